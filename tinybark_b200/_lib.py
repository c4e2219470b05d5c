"""ctypes bindings of libtbcuda.so (include/tbcuda.h). The library is required: there
is no CPU fallback, so importing this module without the built library raises."""

from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libtbcuda.so"

F32, BF16 = 0, 1
SRC_F16, SRC_F32 = 0, 1
REPACK_CHUNK = 16384
EPI_STORE, EPI_SILU, EPI_RESIDUAL, EPI_BIAS_RELU, EPI_GLU, EPI_QKV, EPI_ARGMAX, EPI_LSTM, EPI_JOINT_IN = range(9)
STATUS = {0: "ok", 1: "bad argument", 2: "CUDA error", 3: "unsupported shape or dtype", 4: "workspace too small",
          5: "more clips than the library's own scratch holds"}
FRONTEND_STATIC_MAX_CLIPS = 64
DEVICE_ERRORS = {1: "GEMM barrier wait timed out", 2: "attention barrier wait timed out", 4: "decode wait timed out",
                 8: "depthwise conv copy wait timed out", 16: "token id outside the text piece table"}

HIDDEN, HEADS, HEAD_DIM, FFN, KERNEL, CHANNELS, MELS = 1024, 8, 128, 4096, 9, 256, 128
VOCAB, BLANK, EOS, DURATIONS, PRED = 8193, 8192, 3, 5, 640
TOKEN_ROWS, JOINT_ROWS = 8256, 8448

vp, ll, i32, f32 = C.c_void_p, C.c_longlong, C.c_int, C.c_float


class Epilogue(C.Structure):
    _fields_ = [
        ("kind", i32), ("out_dtype", i32), ("out", vp), ("ldo", ll), ("bias", vp), ("alpha", f32),
        ("out2", vp), ("ldo2", ll), ("out3", vp), ("out4", vp), ("bias_u", vp), ("bias_v", vp),
        ("keys", vp), ("keys2", vp), ("split", i32), ("split_end", i32), ("c", vp), ("h", vp), ("mask", vp),
        ("rows", vp), ("gather", vp), ("gather_row", vp),
    ]


class Layer(C.Structure):
    _fields_ = [
        ("norm_w", vp * 5), ("norm_b", vp * 5), ("ff1_w1", vp), ("ff1_w2", vp), ("ff2_w1", vp), ("ff2_w2", vp),
        ("qkv", vp), ("o_proj", vp), ("pw1", vp), ("pw2", vp), ("bias_u", vp), ("bias_v", vp),
        ("dw_w", vp), ("dw_b", vp), ("rel", vp), ("rel_c", vp),
    ]


class Model(C.Structure):
    _fields_ = [
        ("dtype", i32), ("layers", i32), ("max_len", i32),
        ("sub0_w", vp), ("sub0_b", vp), ("sub_dw_w", vp * 2), ("sub_dw_b", vp * 2), ("sub_pw_w", vp * 2),
        ("sub_pw_b", vp * 2), ("sub_linear_w", vp), ("sub_linear_b", vp), ("layer", C.POINTER(Layer)),
        ("enc_proj_w", vp), ("enc_proj_b", vp),
        ("embedding", vp), ("lstm_w", vp * 2), ("lstm_b", vp * 2), ("dec_proj_w", vp), ("dec_proj_b", vp),
        ("joint_w", vp), ("joint_b", vp),
        ("window", vp), ("mel_w", vp), ("mel_start", vp), ("mel_off", vp),
        ("lstm0_hh", vp), ("lstm0_emb", vp), ("ffn_mx", vp),
    ]


class MXWeight(C.Structure):
    """tb_mx_weight: one MXFP8 weight matrix (codes, tiled scales)."""

    _fields_ = [("codes", vp), ("scales", vp)]


class Batch(C.Structure):
    _fields_ = [
        ("clips", i32), ("frames_total", i32), ("t1_total", i32), ("t2_total", i32), ("t3_total", i32),
        ("frame_off", vp), ("t1_off", vp), ("t2_off", vp), ("t3_off", vp), ("t2_clip", vp), ("t3_clip", vp),
        ("sub_tiles", vp), ("n_sub_tiles", i32), ("attn_tiles", vp), ("n_attn_tiles", i32), ("max_t3", i32),
    ]


class RepackJob(C.Structure):
    """tb_repack_job: one destination tensor of tb_repack."""

    _fields_ = [
        ("src_off", ll), ("dst_off", ll), ("stride", ll * 4), ("first_chunk", ll), ("dims", i32 * 4),
        ("src_type", i32), ("dst_type", i32), ("fill", i32), ("value", f32),
    ]


def _load() -> C.CDLL:
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH.name} is not built: run `python -m tinybark_b200.build` (needs nvcc). "
            "The cuda backend has no CPU fallback."
        )
    lib = C.CDLL(str(LIB_PATH))
    sz = C.c_size_t
    P = C.POINTER
    sig = {
        "tb_version": (i32, []),
        "tb_tile_rows": (i32, [i32, P(i32), P(i32)]),
        "tb_launch_count": (ll, []),
        "tb_last_cuda_error": (C.c_char_p, []),
        "tb_sm_count": (i32, [i32, P(i32)]),
        "tb_frontend_workspace_bytes": (sz, [i32, i32]),
        "tb_frontend": (i32, [P(Model), vp, vp, vp, i32, i32, i32, vp, vp, sz, vp]),
        "tb_frontend_pcm16": (i32, [P(Model), vp, vp, vp, i32, i32, i32, vp, vp, sz, vp]),
        "tb_frontend_static": (i32, [P(Model), vp, vp, vp, i32, i32, vp, vp]),
        "tb_layernorm": (i32, [vp, vp, vp, vp, vp, vp, vp, i32, i32, vp]),
        "tb_gemm": (i32, [i32, vp, ll, vp, i32, i32, i32, P(Epilogue), vp, vp]),
        "tb_set_gemm_pairs": (i32, [i32]),
        "tb_relpos_attention": (i32, [i32, vp, vp, vp, vp, vp, vp, i32, P(Batch), vp, vp, vp]),
        "tb_conv_depthwise": (i32, [i32, vp, vp, vp, P(Batch), vp, vp, vp]),
        "tb_subsample_workspace_bytes": (sz, [i32, i32, i32]),
        "tb_subsample": (i32, [P(Model), P(Batch), vp, vp, vp, sz, vp, vp]),
        "tb_encoder_workspace_bytes": (sz, [i32, i32, i32]),
        "tb_encoder_forward": (i32, [P(Model), P(Batch), vp, vp, vp, sz, vp, vp]),
        "tb_decode_workspace_bytes": (sz, [i32, i32, i32]),
        "tb_selftest_wait": (i32, [i32, vp, vp, vp]),
        "tb_selftest_math": (i32, [i32, vp, vp, ll, vp]),
        "tb_decode_lane_iterations": (i32, [vp, i32, i32, i32, vp, vp]),
        "tb_mx_scale_bytes": (sz, [i32, i32]),
        "tb_encoder_workspace_bytes_mx": (sz, [i32, i32]),
        "tb_mx_quantize": (i32, [i32, vp, ll, i32, i32, vp, vp, vp]),
        "tb_gemm_mx": (i32, [vp, vp, vp, vp, i32, i32, i32, P(Epilogue), vp, vp]),
        "tb_tdt_decode": (i32, [P(Model), vp, vp, vp, i32, i32, i32, vp, vp, vp, sz, vp, vp, vp]),
        "tb_repack": (i32, [P(RepackJob), i32, vp, vp, sz, vp, sz, vp]),
        "tb_text_offsets": (i32, [vp, i32, vp, i32, vp, i32, vp, vp, vp]),
        "tb_text_bytes": (i32, [vp, i32, vp, i32, vp, vp, ll, i32, vp, vp, ll, vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args
    return lib


lib = _load()

# Every symbol include/tbcuda.h declares, for the export check.
EXPORTS = (
    "tb_version", "tb_tile_rows", "tb_launch_count", "tb_last_cuda_error", "tb_sm_count", "tb_frontend_workspace_bytes", "tb_frontend",
    "tb_frontend_static", "tb_frontend_pcm16",
    "tb_layernorm", "tb_gemm", "tb_set_gemm_pairs", "tb_relpos_attention", "tb_conv_depthwise", "tb_subsample_workspace_bytes",
    "tb_subsample", "tb_encoder_workspace_bytes", "tb_encoder_forward", "tb_decode_workspace_bytes", "tb_tdt_decode",
    "tb_selftest_wait", "tb_selftest_math", "tb_decode_lane_iterations", "tb_mx_scale_bytes", "tb_mx_quantize", "tb_encoder_workspace_bytes_mx",
    "tb_gemm_mx", "tb_repack", "tb_text_offsets", "tb_text_bytes",
)


def check(status: int, what: str) -> None:
    """Raises RuntimeError on a non-zero status, as the reference's backends raise on failure."""
    if status:
        detail = lib.tb_last_cuda_error().decode() if status == 2 else ""
        raise RuntimeError(f"{what}: {STATUS.get(status, status)} {detail}".strip())


def tile_rows(dtype: int) -> tuple[int, int]:
    a, b = C.c_int(), C.c_int()
    check(lib.tb_tile_rows(dtype, C.byref(a), C.byref(b)), "tb_tile_rows")
    return a.value, b.value
