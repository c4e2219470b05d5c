"""Generates the golden fixtures in this directory from the reference itself. The path of
a tinybark checkout is a required argument (the checkout is not needed afterwards):

    python tests/golden/make_golden.py /path/to/tinybark

- frontend.npz: tinybark.audio.features on short synthetic clips.
- convert.json: shape and checksums of every tensor tinybark.weights._convert produces
  from the 2-layer synthetic state dict (seed 0).
- cache_file.json: sha256 and tensor order of the fp16 cache file tinybark.weights._save
  writes from that conversion.
- text.json: tinybark.text.Tokenizer.decode of seeded id lists (text_cases) under the
  seeded 8193-id tokenizer of tinybark_b200.synthetic.tokenizer.
- lengths.json: tinybark.ort.subsampled and the greedy loop's cap for many lengths.
- encoder.npz: transformers' ParakeetEncoder (the module family ParakeetForTDT wraps)
  with Bark's config on the synthetic weights: 2 layers on a 1 s clip, 24 layers on a 2 s
  clip (hidden states before the projector).
- decode.json: tokens from tinybark.ort.Bark.tokens, the reference's own greedy loop,
  with its ONNX sessions replaced by calls into this repository's oracle prediction
  network and joint (onnxruntime is not installed here).
"""

from __future__ import annotations

import hashlib
import json
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

from oracle import decoder as odec  # noqa: E402
from oracle import encoder as oenc  # noqa: E402
from tinybark_b200 import synthetic  # noqa: E402

# (name, seconds, seed) of the front-end clips: 2 frames, odd lengths, 1 s.
FRONTEND_CLIPS = [("two_frames", 320 / 16000, 11), ("odd", 5333 / 16000, 12), ("one_second", 1.0, 13)]
# Decode cases: seed of the encoder frames, their count, the frame scale, bias edits.
#   mixed: blanks, durations 1-4, ends on frame >= valid; eos: EOS emitted, then stop;
#   cap: duration-0 repeats until the global iteration cap; single: one encoder frame.
DECODE_CASES = {
    "mixed": dict(seed=21, frames=40, scale=2.0, blank=1.5, eos=None, feature_frames=320),
    "eos": dict(seed=22, frames=40, scale=2.0, blank=1.0, eos=1.5, feature_frames=320),
    "cap": dict(seed=27, frames=40, scale=2.0, blank=0.8, eos=None, feature_frames=320),
    "single": dict(seed=24, frames=1, scale=2.0, blank=0.5, eos=None, feature_frames=2),
}


def decode_weights(case: dict) -> dict[str, np.ndarray]:
    """The 2-layer synthetic state dict with the joint biases edited for a decode case."""
    sd = synthetic.state_dict(0, layers=2)
    bias = sd["joint.head.bias"].copy()
    bias[synthetic.BLANK] += case["blank"]
    if case["eos"] is not None:
        bias[3] += case["eos"]
    sd["joint.head.bias"] = bias
    return sd


def decode_frames(case: dict) -> np.ndarray:
    rng = np.random.default_rng(case["seed"])
    return (rng.standard_normal((case["frames"], synthetic.DECODER_HIDDEN)) * case["scale"]).astype(np.float32)


def text_cases(count: int = 300, seed: int = 5) -> list[list[int]]:
    """Seeded id lists for the detokeniser fixture: 0-120 ids each, about 40 % of them
    byte-fallback pieces (ids 3..258, so byte runs, split multi-byte sequences and
    invalid UTF-8 occur), the rest any id of the 8193 (special tokens included)."""
    rng = np.random.default_rng(seed)
    cases = []
    for _ in range(count):
        n = int(rng.integers(0, 121))
        byte = rng.random(n) < 0.4
        ids = np.where(byte, rng.integers(3, 259, n), rng.integers(0, 8193, n))
        cases.append([int(i) for i in ids])
    return cases


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a, np.float32).tobytes()).hexdigest()[:16]


def main(ref: Path) -> None:
    import importlib.machinery

    from transformers import ParakeetEncoder  # noqa: F401  (before the stub below)

    stub = types.ModuleType("onnxruntime")
    stub.__spec__ = importlib.machinery.ModuleSpec("onnxruntime", None)
    sys.modules.setdefault("onnxruntime", stub)
    sys.path.insert(0, str(ref))
    from tinybark import audio, ort, text, weights

    torch.set_num_threads(8)

    # Front-end.
    out = {}
    for name, seconds, seed in FRONTEND_CLIPS:
        x = synthetic.to_float(synthetic.clip(seconds, seed))
        out[f"{name}_samples"] = x
        out[f"{name}_features"] = audio.features(x)
    np.savez_compressed(HERE / "frontend.npz", **out)

    # Converter.
    sd = synthetic.state_dict(0, layers=2)
    conv = weights._convert(dict(sd), synthetic.config(2))
    summary = {k: {"shape": list(v.shape), "sha": digest(v), "sum": float(np.nansum(v[np.isfinite(v)]))}
               for k, v in conv.items()}
    (HERE / "convert.json").write_text(json.dumps(summary, indent=1, sort_keys=True))
    import tempfile

    with tempfile.TemporaryDirectory() as d:
        path = Path(d) / "bark.safetensors"
        weights._save(conv, path)
        sha = hashlib.sha256(path.read_bytes()).hexdigest()
        (HERE / "cache_file.json").write_text(json.dumps({"sha256": sha, "order": list(conv)}, indent=1))

        # Detokeniser: the reference's Tokenizer on the seeded tokenizer.
        tok = text.Tokenizer(synthetic.tokenizer(Path(d) / "tokenizer.json"))
        texts = [tok.decode(ids) for ids in text_cases()]
    (HERE / "text.json").write_text(json.dumps({"texts": texts}, ensure_ascii=False, indent=0))

    # Length helpers.
    ns = list(range(0, 70)) + [99, 100, 101, 255, 256, 257, 1000, 3000, 60000]
    lengths = {"n": ns, "subsampled": [ort.subsampled(n) for n in ns],
               "cap": [10 * ort.subsampled(n + 1) - 1 for n in ns]}
    (HERE / "lengths.json").write_text(json.dumps(lengths))

    # Encoder: transformers' module on the synthetic weights.
    enc = {}
    for layers, seconds, seed in ((2, 1.0, 31), (24, 2.0, 32)):
        sd = synthetic.state_dict(0, layers=layers)
        x = synthetic.to_float(synthetic.clip(seconds, seed))
        feats = audio.features(x)
        model = oenc.hf_encoder(sd, layers)
        with torch.inference_mode():
            hidden = model(torch.from_numpy(feats)[None]).last_hidden_state[0].numpy()
        enc[f"l{layers}_samples"] = x
        enc[f"l{layers}_hidden"] = hidden
    np.savez_compressed(HERE / "encoder.npz", **enc)

    # Decode: the reference's greedy loop with stub sessions around the oracle.
    result = {}
    for name, case in DECODE_CASES.items():
        sd = decode_weights(case)
        dec = odec.Decoder(sd)
        frames = decode_frames(case)
        bark = ort.Bark.__new__(ort.Bark)
        bark.blank, bark.durations, bark.max_symbols = synthetic.BLANK, list(synthetic.DURATIONS), 10
        bark.state_shape = (2, 1, synthetic.DECODER_HIDDEN)

        class Encoder:
            def run(self, _, inputs):
                return [frames]

        class DecoderSession:
            def run(self, _, inputs):
                h = torch.from_numpy(inputs["h"][:, 0].copy())
                c = torch.from_numpy(inputs["c"][:, 0].copy())
                out, h, c = dec.step(int(inputs["token"][0, 0]), h, c)
                return out.numpy(), h.numpy()[:, None], c.numpy()[:, None]

        class Joint:
            def run(self, _, inputs):
                tok, d, _ = dec.joint(torch.from_numpy(inputs["encoded"]), torch.from_numpy(inputs["decoded"]))
                return np.array(tok), np.array(d)

        bark.encoder, bark.decoder, bark.joint = Encoder(), DecoderSession(), Joint()
        # Bark.tokens computes features only to count frames; give it samples of the
        # requested feature-frame count.
        ort.audio = types.SimpleNamespace(features=lambda s: np.zeros((case["feature_frames"], 128), np.float32))
        tokens = bark.tokens(np.zeros(case["feature_frames"] * 160, np.float32))
        ort.audio = audio
        result[name] = {"case": case, "tokens": [int(t) for t in tokens]}
        print(name, len(tokens), tokens[:20])
    (HERE / "decode.json").write_text(json.dumps(result, indent=1))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden.py /path/to/tinybark")
    main(Path(sys.argv[1]))
