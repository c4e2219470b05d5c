"""Host-side logic of the cuda backend, without a GPU: batch planning, the weight
repacking rules, the detokeniser and the backend registry."""

import json

import numpy as np
import pytest

from tinybark_b200 import backends, lengths
from tinybark_b200.engine import plan_arrays
from tinybark_b200.text import Tokenizer


def test_plan_offsets_and_tiles():
    frames = [2, 100, 1000, 3, 257]
    p = plan_arrays(frames, 2, 32)
    t3 = [lengths.subsampled(f) for f in frames]
    assert p["t3"].tolist() == t3
    assert p["frame_off"].tolist() == [0, 2, 102, 1102, 1105, 1362]
    assert p["t3_off"][-1] == sum(t3)
    assert p["t3_clip"].tolist() == sum(([i] * n for i, n in enumerate(t3)), [])
    assert p["caps"].tolist() == [lengths.decode_cap(f) for f in frames]
    # Every attention row covered exactly once, longest clip first.
    att = p["attn_tiles"].reshape(-1, 2)
    assert att[0, 0] == int(np.argmax(t3))
    covered = {(c, r + k) for c, r in att for k in range(32) if r + k < t3[c]}
    assert covered == {(c, r) for c in range(len(frames)) for r in range(t3[c])}
    t2 = [lengths.subsampled(f, 2) for f in frames]
    sub = p["sub_tiles"].reshape(-1, 2)
    covered = {(c, r + k) for c, r in sub for k in range(2) if r + k < t2[c]}
    assert covered == {(c, r) for c in range(len(frames)) for r in range(t2[c])}


def test_plan_rejects_short_clips():
    with pytest.raises(ValueError):
        plan_arrays([5, 1], 2, 32)


def test_lstm_gate_interleave():
    """Row 4u+g of the repacked LSTM weight is gate g of unit u (PyTorch order i, f, g, o)."""
    w = np.arange(4 * 640 * 3, dtype=np.float32).reshape(4 * 640, 3)
    packed = w.reshape(4, 640, 3).transpose(1, 0, 2).reshape(4 * 640, 3)
    for u in (0, 5, 639):
        for g in range(4):
            np.testing.assert_array_equal(packed[4 * u + g], w[g * 640 + u])


def test_glu_pair_interleave():
    w = np.arange(2048 * 2, dtype=np.float32).reshape(2048, 2)
    packed = np.stack([w[:1024], w[1024:]], 1).reshape(2048, 2)
    for c in (0, 7, 1023):
        np.testing.assert_array_equal(packed[2 * c], w[c])
        np.testing.assert_array_equal(packed[2 * c + 1], w[1024 + c])


def test_subsampling_linear_permutation():
    """Linear input columns go from (channel, frequency) to (frequency, channel), so the
    kernels' [time][frequency][channel] activations multiply the same weights."""
    rng = np.random.default_rng(0)
    w = rng.standard_normal((8, 256 * 16)).astype(np.float32)
    x = rng.standard_normal((256, 16)).astype(np.float32)  # (channel, frequency)
    perm = w.reshape(8, 256, 16).transpose(0, 2, 1).reshape(8, -1)
    np.testing.assert_allclose(perm @ x.T.reshape(-1), w @ x.reshape(-1), rtol=1e-5, atol=1e-4)


def test_tokenizer_decodes_pieces_bytes_and_specials(tmp_path):
    spec = {
        "model": {"vocab": {"<unk>": 0, "▁Hel": 1, "lo": 2, "▁w": 3, "<0xC3>": 4, "<0xA9>": 5, "rld": 6}},
        "added_tokens": [{"id": 7, "content": "<|endoftext|>", "special": True}],
    }
    path = tmp_path / "tokenizer.json"
    path.write_text(json.dumps(spec))
    tok = Tokenizer(str(path))
    assert tok.decode([1, 2, 3, 4, 5, 6, 7]) == "Hello wérld"
    assert tok.decode([7]) == ""


def test_joined_piece_bytes_are_the_tokenizers_text(tmp_path):
    """The GPU's join, restated: every id's bytes from Tokenizer.table joined and finished
    once give Tokenizer.decode's text, over random id lists heavy in byte-fallback runs
    (invalid UTF-8 included) and special tokens between them."""
    import random

    from conftest import synthetic_tokenizer
    from tinybark_b200.text import finish

    tok = Tokenizer(synthetic_tokenizer(tmp_path / "tokenizer.json", vocab=600))
    off, data = tok.table()
    assert len(off) == 601 and off[0] == 0 and off[-1] == len(data)
    assert bytes(data[off[3 + 0xC3] : off[4 + 0xC3]]) == b"\xc3" and off[1] == off[0]  # a byte piece; a special
    rng = random.Random(1)
    for _ in range(20000):
        ids = []
        for _ in range(rng.randint(0, 12)):
            r = rng.random()
            ids.append(rng.randrange(3, 259) if r < 0.5 else (rng.choice([0, 1, 2, 599]) if r < 0.6 else rng.randrange(259, 599)))
        joined = b"".join(bytes(data[off[i] : off[i + 1]]) for i in ids)
        assert finish(joined) == tok.decode(ids), ids


def test_registry_has_cuda_backend():
    b = backends.BACKENDS["cuda"]
    assert b.name == "cuda" and set(b.descriptions) <= set(backends.DEVICES)
    assert "gpu" in b.descriptions and b.env("gpu") == {}


def test_cpu_device_is_refused():
    import tinybark_b200

    with pytest.raises(RuntimeError):
        tinybark_b200.Bark("cpu", weights=({}, {}))
