"""The block-scaled format oracle (oracle/mx.py) pinned on the CPU: known E4M3 / E2M1 codes
and ties, every code round-tripping, agreement with torch's float8_e4m3fn conversion, the
MX scale choice, and the error bounds the formats guarantee."""

import numpy as np
import pytest
import torch

from oracle import mx


def test_e4m3_known_codes():
    cases = [(1.0, 0x38), (-2.0, 0xC0), (448.0, 0x7E), (500.0, 0x7E), (-1e9, 0xFE), (2.0**-9, 0x01), (2.0**-6, 0x08),
             (7 * 2.0**-9, 0x07), (0.0, 0x00), (-0.0, 0x80), (1.0625, 0x38), (1.1875, 0x3A), (1.96875, 0x40),
             (2.0**-10, 0x00), (3 * 2.0**-11, 0x01), (240.0, 0x77), (464.0, 0x7E)]
    for x, code in cases:
        assert int(mx.e4m3_encode(x)) == code, (x, hex(int(mx.e4m3_encode(x))))


def test_e4m3_every_code_round_trips():
    codes = np.array([c for c in range(256) if (c & 0x7F) != 0x7F], np.uint8)
    assert np.array_equal(mx.e4m3_encode(mx.e4m3_decode(codes)), codes)
    assert np.isnan(mx.e4m3_decode(np.array([0x7F, 0xFF]))).all()
    assert mx.e4m3_decode(np.array([0x7E]))[0] == 448.0


def test_e4m3_matches_torch_conversion_in_range():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(20000) * s for s in (1e-3, 0.1, 1.0, 30.0, 150.0)])
    x = np.clip(x, -448, 448).astype(np.float32)
    x = np.concatenate([x, np.float32(mx.e4m3_decode(np.arange(0, 126)) + 2.0**-12)])  # just above codes
    want = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(mx.e4m3_encode(x), want)


def test_e2m1_values_ties_and_saturation():
    assert list(mx.e2m1_decode(np.arange(8))) == [0, 0.5, 1, 1.5, 2, 3, 4, 6]
    ties = {0.25: 0.0, 0.75: 1.0, 1.25: 1.0, 1.75: 2.0, 2.5: 2.0, 3.5: 4.0, 5.0: 4.0, 7.0: 6.0, -5.5: -6.0}
    for x, v in ties.items():
        assert mx.e2m1_decode(mx.e2m1_encode(x)) == v, x
    assert int(mx.e2m1_encode(-1.0)) == 0b1010


def test_mxfp8_scale_and_error_bound():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((7, 128)) * np.exp2(rng.integers(-20, 20, (7, 1)))
    x[0, :32] = 0.0  # an all-zero block
    x[1, :32] = 3.0  # max 3 -> scale 2^(1 - 8), 3 / 2^-7 = 384 exactly representable
    codes, e = mx.mxfp8_quantize(x)
    assert codes.shape == x.shape and e.shape == (7, 4)
    assert e[0, 0] == -127 and e[1, 0] == -7
    y = mx.mxfp8_dequantize(codes, e)
    assert np.array_equal(y[:2, :32], x[:2, :32])
    blocks, yb = x.reshape(7, 4, 32), y.reshape(7, 4, 32)
    amax = np.abs(blocks).max(-1, keepdims=True)
    # The scale puts a block's largest value in [256, 512): values above 448 saturate (up
    # to 1/8 relative error, inherent in the format's scale rule); the rest of E4M3's normal
    # range (|x| / 2^e in [2^-6, 448]) is within half a step, 2^-4 relative; the whole block
    # within 2^-9 * 2^e absolute plus that.
    scaled = np.abs(blocks) / np.exp2(e)[..., None]
    err = np.abs(yb - blocks)
    normal, saturated = (scaled >= 2.0**-6) & (scaled <= 448), scaled > 448
    assert saturated.any() and normal.any()
    assert (err[normal] <= np.abs(blocks)[normal] * 2.0**-4).all()
    assert (np.abs(yb)[saturated] == (448 * np.exp2(e)[..., None] * np.ones_like(yb))[saturated]).all()
    assert (err[saturated] <= np.abs(blocks)[saturated] / 8).all()
    assert (err <= np.exp2(e)[..., None] * 2.0**-9 + amax / 8).all()


def test_nvfp4_round_trip_bounds():
    rng = np.random.default_rng(2)
    x = rng.standard_normal((5, 64)) * 3.0
    codes, s, g = mx.nvfp4_quantize(x)
    assert codes.shape == x.shape and s.shape == (5, 4) and codes.max() < 16
    y = mx.nvfp4_dequantize(codes, s, g)
    scale = (mx.e4m3_decode(s) * g)[..., None]
    # Half the largest E2M1 step (2, between 4 and 6) times the block scale, plus the
    # scale's own E4M3 rounding (2^-4 of the block max).
    bound = scale * 1.0 + np.abs(x.reshape(5, 4, 16)).max(-1, keepdims=True) * 2.0**-4
    assert (np.abs(y - x).reshape(5, 4, 16) <= bound).all()
    assert np.allclose(np.abs(y).max(), np.abs(x).max(), rtol=0.1)


@pytest.mark.parametrize("fmt,tol", [("mxfp8", 0.05), ("nvfp4", 0.35)])
def test_block_scaled_gemm_tracks_the_float_product(fmt, tol):
    rng = np.random.default_rng(3)
    a, w = rng.standard_normal((64, 256)), rng.standard_normal((48, 256)) * 0.05
    ref = a @ w.T
    got = mx.block_scaled_gemm(a, w, fmt)
    err = np.abs(got - ref).max() / np.abs(ref).max()
    assert 0 < err < tol
