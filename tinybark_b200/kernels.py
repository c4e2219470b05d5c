"""Single kernels of libtbcuda on torch tensors, for tests and the per-kernel
microbenchmarks. Each call goes through the C ABI on the current stream."""

from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib as L

_ERR: dict[int, torch.Tensor] = {}


def _err(device: torch.device) -> torch.Tensor:
    i = device.index if device.index is not None else torch.cuda.current_device()
    if i not in _ERR:
        _ERR[i] = torch.zeros(1, dtype=torch.int32, device=device)
    return _ERR[i]


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def dtype_of(t: torch.Tensor) -> int:
    return L.BF16 if t.dtype == torch.bfloat16 else L.F32


def gemm(a: torch.Tensor, w: torch.Tensor, ep: L.Epilogue) -> None:
    """A [M, K] times W [N, K]^T with epilogue `ep` (its output pointers set by the caller)."""
    L.check(L.lib.tb_gemm(dtype_of(a), a.data_ptr(), a.stride(0), w.data_ptr(), a.shape[0], w.shape[0], a.shape[1],
                          C.byref(ep), _err(a.device).data_ptr(), _stream()), "tb_gemm")


def layernorm(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, y: torch.Tensor, x_out=None, w2=None, b2=None):
    L.check(L.lib.tb_layernorm(x.data_ptr(), w.data_ptr(), b.data_ptr(), None if x_out is None else x_out.data_ptr(),
                               None if w2 is None else w2.data_ptr(), None if b2 is None else b2.data_ptr(),
                               y.data_ptr(), dtype_of(y), x.shape[0], _stream()), "tb_layernorm")


class Frames:
    """A tb_batch with the encoder-frame fields of clips of lengths `t3` (attention and
    the depthwise conv read only those)."""

    def __init__(self, t3: list[int], dtype: int, device="cuda"):
        t3 = np.asarray(t3, np.int64)
        _, rows = L.tile_rows(dtype)
        off = np.concatenate([[0], np.cumsum(t3)]).astype(np.int32)
        clip = np.repeat(np.arange(len(t3), dtype=np.int32), t3)
        order = np.argsort(-t3, kind="stable")
        tiles = np.array([(c, r) for c in order for r in range(0, int(t3[c]), rows)], np.int32).reshape(-1)
        self.keep = [torch.from_numpy(a).to(device) for a in (off, clip, tiles)]
        self.off = off
        b = L.Batch()
        b.clips, b.t3_total, b.max_t3 = len(t3), int(off[-1]), int(t3.max())
        b.t3_off, b.t3_clip = self.keep[0].data_ptr(), self.keep[1].data_ptr()
        b.attn_tiles, b.n_attn_tiles = self.keep[2].data_ptr(), len(tiles) // 2
        self.batch = b


def rel_bias(rel: torch.Tensor, bias_u: torch.Tensor, bias_v: torch.Tensor) -> torch.Tensor:
    """(bias_v - bias_u)_h . rel[n, head h] as [rows, 128] fp32 (columns 8.. zero): the
    position term the bf16 attention adds to (q + bias_u) . rel, through tb_gemm."""
    w = torch.zeros(128, L.HIDDEN, device=rel.device, dtype=torch.float32)
    diff = (bias_v - bias_u).float().reshape(L.HEADS, L.HEAD_DIM)
    for h in range(L.HEADS):
        w[h, h * L.HEAD_DIM : (h + 1) * L.HEAD_DIM] = diff[h]
    out = torch.empty(rel.shape[0], 128, device=rel.device, dtype=torch.float32)
    ep = L.Epilogue(kind=L.EPI_STORE, out_dtype=L.F32, out=out.data_ptr(), ldo=128)
    gemm(rel, w.to(rel.dtype).contiguous(), ep)
    return out


def attention(qu, qv, k, v, rel, max_len: int, frames: Frames, out, rel_c=None) -> None:
    L.check(L.lib.tb_relpos_attention(dtype_of(qu), qu.data_ptr(), None if qv is None else qv.data_ptr(),
                                      k.data_ptr(), v.data_ptr(), rel.data_ptr(),
                                      None if rel_c is None else rel_c.data_ptr(), max_len, C.byref(frames.batch),
                                      out.data_ptr(), _err(qu.device).data_ptr(), _stream()), "tb_relpos_attention")


def depthwise(x, w, b, frames: Frames, y) -> None:
    L.check(L.lib.tb_conv_depthwise(dtype_of(x), x.data_ptr(), w.data_ptr(), b.data_ptr(), C.byref(frames.batch),
                                    y.data_ptr(), _err(x.device).data_ptr(), _stream()), "tb_conv_depthwise")


class MX:
    """A matrix [rows, K] in MXFP8 on the GPU (tb_mx_quantize): E4M3 codes [rows padded to
    128, K] and E8M0 scales in the MMA's tiled layout (tb_mx_scale_bytes)."""

    def __init__(self, x: torch.Tensor):
        rows, k = x.shape
        pad = -(-rows // 128) * 128
        self.rows, self.k = rows, k
        self.codes = torch.empty(pad, k, dtype=torch.uint8, device=x.device)
        self.scales = torch.empty(L.lib.tb_mx_scale_bytes(rows, k), dtype=torch.uint8, device=x.device)
        L.check(L.lib.tb_mx_quantize(dtype_of(x), x.data_ptr(), x.stride(0), rows, k, self.codes.data_ptr(),
                                     self.scales.data_ptr(), _stream()), "tb_mx_quantize")

    def scale_exponents(self) -> torch.Tensor:
        """The E8M0 scale exponents (byte - 127) as [rows, K / 32] int, untiled."""
        groups = self.k // 512
        t = self.scales.view(-1, groups, 128, 16).permute(0, 2, 1, 3).reshape(-1, self.k // 32)
        return t[: self.rows].to(torch.int32) - 127


def gemm_mx(a: MX, w: MX, ep: L.Epilogue) -> None:
    """A [M, K] times W [N, K]^T, both MXFP8, with epilogue `ep`."""
    L.check(L.lib.tb_gemm_mx(a.codes.data_ptr(), a.scales.data_ptr(), w.codes.data_ptr(), w.scales.data_ptr(), a.rows,
                             w.rows, a.k, C.byref(ep), _err(a.codes.device).data_ptr(), _stream()), "tb_gemm_mx")


def check(device=None) -> None:
    device = torch.device("cuda") if device is None else torch.device(device)
    torch.cuda.synchronize(device)
    e = _err(device)
    code = int(e.item())
    if code:
        e.zero_()
        raise RuntimeError(f"device error {code}")
