"""The oracle: a CPU restatement of the reference's inference path, used ONLY as the
checker by the tests, by __graft_entry__.smoke() and by bench.py's CPU-baseline leg.
The product (tinybark_b200) never imports it.

- frontend.py: log-mel features (tinybark/audio.py:1-55), numpy.
- encoder.py: the FastConformer encoder and encoder projector, torch fp32 on the CPU,
  on checkpoint-named weights (transformers' ParakeetEncoder, modeling_parakeet.py,
  with tinybark's Bark config: tinybark/tinygrad/model.py:87-158).
- decoder.py: the TDT prediction network, joint and greedy loop, torch fp32 on the
  CPU (tinybark/tinygrad/model.py:162-233, tinybark/ort/__init__.py:55-86,
  tinybark/ort/export.py:28-50).

Parity pins: frontend against tinybark.audio.features itself; the encoder against
transformers' ParakeetEncoder 5.5.0 (the module family ParakeetForTDT wraps); the greedy
loop against tinybark.ort.Bark.tokens run with sessions that call this oracle. The
fixtures and the script that made them are in tests/golden/.
"""
