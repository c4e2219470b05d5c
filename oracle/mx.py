"""Oracle (test infrastructure, not the product): block-scaled low-precision weights for the
FFN GEMMs, restated in numpy from the formats' published definitions. No kernel uses these
formats yet; this fixes the arithmetic a block-scaled FFN GEMM is checked against. The
formats follow the survey of low-bit floats with block scales in the reference's notes
(docs/2026-10-24-learnings.md:133-146).

- FP8 E4M3 (the "FN" variant of OCP's 8-bit floats): sign, 4 exponent bits (bias 7),
  3 mantissa bits; no infinities, largest finite 448 = 1.75 * 2^8, smallest subnormal
  2^-9; code 0x7F / 0xFF is NaN. Conversion rounds to nearest, ties to even, and saturates
  to +-448 (as a satfinite conversion does).
- FP4 E2M1: sign, 2 exponent bits (bias 1), 1 mantissa bit: 0, 0.5, 1, 1.5, 2, 3, 4, 6.
  Same rounding and saturation (to +-6).
- MXFP8 (OCP Microscaling Formats v1.0): each block of 32 consecutive values along the
  reduction axis shares an E8M0 scale 2^e, e = floor(log2(max |x|)) - 8 (8 = the exponent
  of E4M3's largest binade) clamped to [-127, 127]; elements are E4M3 of x / 2^e. An
  all-zero block takes e = -127.
- NVFP4: blocks of 16 share an E4M3 scale, elements E2M1, and the tensor has one fp32
  scale g = amax / (6 * 448) so that every block scale fits E4M3. A block's scale is
  E4M3(max |x| / (6 * g)); its elements are E2M1(x / (scale * g)) (zero where the scale
  rounds to zero).

Codes are uint8 arrays (an E2M1 code in the low nibble).
"""

from __future__ import annotations

import numpy as np

E4M3_MAX = 448.0
E2M1_MAX = 6.0
MX_BLOCK = 32
NV_BLOCK = 16


def _round_even(x: np.ndarray) -> np.ndarray:
    return np.round(x)  # numpy rounds half to even


def _encode(x, exp_bits: int, man_bits: int, bias: int, max_value: float) -> np.ndarray:
    """Round-to-nearest-even, saturating encoding into a small float with subnormals."""
    x = np.asarray(x, np.float64)
    if np.isnan(x).any():
        raise ValueError("NaN has no saturating encoding here")
    sign = np.signbit(x).astype(np.uint8)
    a = np.minimum(np.abs(x), max_value)
    min_normal_exp = 1 - bias
    e = np.floor(np.log2(np.where(a > 0, a, 1.0)))
    e = np.maximum(e, min_normal_exp)  # subnormals share the smallest normal binade's step
    step = np.exp2(e - man_bits)
    q = np.minimum(_round_even(a / step) * step, max_value)
    # Re-derive the binade after rounding (a mantissa can carry into the next one).
    qe = np.floor(np.log2(np.where(q > 0, q, 1.0)))
    normal = q >= 2.0**min_normal_exp
    exp_field = np.where(normal, qe + bias, 0)
    man_field = np.where(normal, q / np.exp2(qe) - 1.0, q / 2.0**min_normal_exp) * 2**man_bits
    code = (exp_field.astype(np.int64) << man_bits) | _round_even(man_field).astype(np.int64)
    return ((sign.astype(np.int64) << (exp_bits + man_bits)) | code).astype(np.uint8)


def _decode(code, exp_bits: int, man_bits: int, bias: int) -> np.ndarray:
    c = np.asarray(code).astype(np.int64)
    sign = np.where((c >> (exp_bits + man_bits)) & 1, -1.0, 1.0)
    e = (c >> man_bits) & ((1 << exp_bits) - 1)
    m = c & ((1 << man_bits) - 1)
    value = np.where(e > 0, (1.0 + m / 2**man_bits) * np.exp2(e - bias), m / 2**man_bits * 2.0 ** (1 - bias))
    return sign * value


def e4m3_encode(x) -> np.ndarray:
    return _encode(x, 4, 3, 7, E4M3_MAX)


def e4m3_decode(code) -> np.ndarray:
    c = np.asarray(code).astype(np.int64)
    v = _decode(c, 4, 3, 7)
    return np.where((c & 0x7F) == 0x7F, np.nan, v)


def e2m1_encode(x) -> np.ndarray:
    return _encode(x, 2, 1, 1, E2M1_MAX)


def e2m1_decode(code) -> np.ndarray:
    return _decode(np.asarray(code) & 0xF, 2, 1, 1)


def _blocks(x: np.ndarray, block: int) -> np.ndarray:
    x = np.asarray(x, np.float64)
    if x.shape[-1] % block:
        raise ValueError(f"the last axis ({x.shape[-1]}) is not a multiple of the block ({block})")
    return x.reshape(*x.shape[:-1], x.shape[-1] // block, block)


def mxfp8_quantize(x) -> tuple[np.ndarray, np.ndarray]:
    """(E4M3 codes [..., K], E8M0 scale exponents [..., K / 32] as int) of x [..., K]."""
    b = _blocks(x, MX_BLOCK)
    amax = np.abs(b).max(-1)
    e = np.where(amax > 0, np.floor(np.log2(np.where(amax > 0, amax, 1.0))) - 8, -127)
    e = np.clip(e, -127, 127).astype(np.int64)
    codes = e4m3_encode(b / np.exp2(e)[..., None])
    return codes.reshape(np.shape(x)), e


def mxfp8_dequantize(codes, scale_exp) -> np.ndarray:
    v = _blocks(e4m3_decode(codes), MX_BLOCK) * np.exp2(np.asarray(scale_exp, np.float64))[..., None]
    return v.reshape(np.shape(codes))


def nvfp4_quantize(x) -> tuple[np.ndarray, np.ndarray, float]:
    """(E2M1 codes [..., K], E4M3 block scale codes [..., K / 16], fp32 tensor scale g)."""
    x = np.asarray(x, np.float64)
    amax = float(np.abs(x).max()) if x.size else 0.0
    g = float(np.float32(amax / (E2M1_MAX * E4M3_MAX))) if amax > 0 else 1.0
    b = _blocks(x, NV_BLOCK)
    scale_codes = e4m3_encode(np.abs(b).max(-1) / (E2M1_MAX * g))
    scale = e4m3_decode(scale_codes) * g
    safe = np.where(scale > 0, scale, 1.0)[..., None]
    codes = np.where(scale[..., None] > 0, e2m1_encode(b / safe), 0).astype(np.uint8)
    return codes.reshape(x.shape), scale_codes, g


def nvfp4_dequantize(codes, scale_codes, g: float) -> np.ndarray:
    v = _blocks(e2m1_decode(codes), NV_BLOCK) * (e4m3_decode(scale_codes) * g)[..., None]
    return v.reshape(np.shape(codes))


def block_scaled_gemm(a, w, fmt: str = "mxfp8") -> np.ndarray:
    """A [M, K] times W [N, K]^T with both operands quantized along K in `fmt` ("mxfp8" or
    "nvfp4"), products summed in float64: the value a block-scaled GEMM approximates with
    fp32 accumulation."""
    if fmt == "mxfp8":
        qa, qw = mxfp8_dequantize(*mxfp8_quantize(a)), mxfp8_dequantize(*mxfp8_quantize(w))
    elif fmt == "nvfp4":
        qa, qw = nvfp4_dequantize(*nvfp4_quantize(a)), nvfp4_dequantize(*nvfp4_quantize(w))
    else:
        raise ValueError(fmt)
    return qa @ qw.T
