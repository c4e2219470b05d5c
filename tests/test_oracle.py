"""The oracle pinned against the reference's own outputs (tests/golden, made by
tests/golden/make_golden.py from tinybark and transformers). CPU only."""

import numpy as np
import pytest
import torch

from conftest import golden_json, golden_npz, max_rel, state_dict
from oracle import decoder as odec
from oracle import encoder as oenc
from oracle import frontend as ofront
from tinybark_b200 import lengths, synthetic, tables, weights

CLIPS = ("two_frames", "odd", "one_second")


@pytest.mark.parametrize("name", CLIPS)
def test_frontend_matches_reference(name):
    g = golden_npz("frontend.npz")
    ours = ofront.features(g[f"{name}_samples"])
    ref = g[f"{name}_features"]
    assert ours.shape == ref.shape == (len(g[f"{name}_samples"]) // 160, 128)
    np.testing.assert_allclose(ours, ref, rtol=0, atol=1e-6)


def test_frontend_tables_match_oracle():
    np.testing.assert_array_equal(tables.mel_filters(), ofront.MEL)
    np.testing.assert_array_equal(tables.window(), ofront.WINDOW)
    w, start, off = tables.sparse_mel()
    dense = np.zeros((128, 257), np.float32)
    for m in range(128):
        dense[m, start[m] : start[m] + off[m + 1] - off[m]] = w[off[m] : off[m + 1]]
    np.testing.assert_array_equal(dense, ofront.MEL)


def test_synthetic_clips_are_seeded_speech_like():
    a, b = synthetic.clip(1.5, 7), synthetic.clip(1.5, 7)
    np.testing.assert_array_equal(a, b)
    assert a.dtype == np.int16 and len(a) == 24000
    assert 16000 <= np.abs(a).max() <= 16384  # peak at half of full scale
    assert not np.array_equal(a, synthetic.clip(1.5, 8))
    long = synthetic.clip(10.0, 3, segment=2.0)
    assert len(long) == 160000


def test_convert_matches_reference():
    ref = golden_json("convert.json")
    ours = weights.convert(state_dict(2), synthetic.config(2))
    assert set(ours) == set(ref)
    import hashlib

    for k, v in ours.items():
        assert list(v.shape) == ref[k]["shape"], k
        sha = hashlib.sha256(np.ascontiguousarray(v, np.float32).tobytes()).hexdigest()[:16]
        assert sha == ref[k]["sha"], k


def test_converted_cache_roundtrip(tmp_path):
    conv = weights.convert(state_dict(2), synthetic.config(2))
    path = tmp_path / "bark.safetensors"
    weights.save(conv, path)
    back = weights.load(path)
    assert set(back) == set(conv)
    for k in conv:
        np.testing.assert_array_equal(back[k], conv[k].astype(np.float16).astype(np.float32))


def test_lengths_match_reference():
    ref = golden_json("lengths.json")
    assert [lengths.subsampled(n) for n in ref["n"]] == ref["subsampled"]
    assert [lengths.decode_cap(n) for n in ref["n"]] == ref["cap"]
    assert lengths.bucket(1) == 256 and lengths.bucket(256) == 256 and lengths.bucket(257) == 512


def test_rel_shift_index_equals_pad_reshape():
    """The index form of the relative shift equals transformers' pad/reshape form
    (modeling_parakeet.py:348-355) on the first T columns."""
    t = 9
    bd = torch.randn(2, 3, t, 2 * t - 1)
    b, h, q, p = bd.shape
    x = torch.nn.functional.pad(bd, (1, 0)).view(b, h, -1, q)[:, :, 1:].view(b, h, q, p)[..., :t]
    i = torch.arange(t)[:, None]
    j = torch.arange(t)[None, :]
    y = torch.gather(bd, 3, (t - 1 - i + j).expand(b, h, t, t))
    torch.testing.assert_close(x, y, rtol=0, atol=0)


@pytest.mark.parametrize("layers,tol", [(2, 1e-5), (24, 1e-5)])
def test_encoder_matches_transformers(layers, tol):
    g = golden_npz("encoder.npz")
    feats = ofront.features(g[f"l{layers}_samples"])
    _, hidden = oenc.encode(state_dict(layers), feats, hidden=True)
    assert hidden.shape == g[f"l{layers}_hidden"].shape
    assert max_rel(hidden, g[f"l{layers}_hidden"]) < tol


@pytest.mark.parametrize("case", ["mixed", "eos", "cap", "single"])
def test_greedy_loop_matches_reference_loop(case):
    from golden.make_golden import decode_frames, decode_weights

    g = golden_json("decode.json")[case]
    dec = odec.Decoder(decode_weights(g["case"]))
    tokens = dec.greedy(decode_frames(g["case"]), g["case"]["feature_frames"])
    assert tokens == g["tokens"]
