"""The packed weights: one device buffer holding every tensor the kernels read, in their
layouts, written by one tb_repack launch from the converted tensors (tinybark's layout,
tinybark/weights.py:62-89) wherever those sit on the GPU: the fp16 cache file's data block
(tinybark/weights.py:92-120) read once, as tinybark/tinygrad/weights.py:10-26 reads it, and
copied up with each tensor on a 16-byte boundary (aligned_runs), or float32 arrays
uploaded one by one.

Each region is one contiguous destination tensor, 256-byte aligned. The reorderings the
kernels want are the strides of the region's jobs:
- subsampling linear: input columns (channel, frequency) to (frequency, channel);
- conv pointwise_conv1: GLU pairs side by side (row 2c is a_c, row 2c+1 its gate g_c);
- LSTM weights and biases: the four gates of a unit side by side (row 4u+g is gate g of
  unit u);
- bf16 only: layer 0's W_hh and W_ih halves of those rows (the persistent decoder takes
  layer 0's gates as E[token] + W_hh . h0, with the table E = embedding . W_ih^T computed
  once from the second);
- joint: the token rows, the 5 duration rows at TOKEN_ROWS, zero rows (bias -inf) up to
  JOINT_ROWS.
Matrices take the engine's type (bf16 or fp32), vectors stay fp32.
"""

from __future__ import annotations

import ctypes as C
import json
import os
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass
from math import prod
from pathlib import Path

import numpy as np
import torch

from . import _lib as L

SRC_TYPES = {"F16": L.SRC_F16, "F32": L.SRC_F32}
SRC_SIZE = {L.SRC_F16: 2, L.SRC_F32: 4}
DST_SIZE = {L.BF16: 2, L.F32: 4}
NORMS = ("norm_feed_forward1", "norm_self_att", "norm_conv", "norm_feed_forward2", "norm_out")


@dataclass(frozen=True)
class Source:
    off: int  # byte offset in the source buffer
    shape: tuple[int, ...]
    type: int  # SRC_F16 or SRC_F32


@dataclass(frozen=True)
class Region:
    off: int  # byte offset in the packed buffer
    shape: tuple[int, ...]
    type: int  # F32 or BF16


def _contiguous(dims: tuple[int, ...]) -> tuple[int, ...]:
    return tuple(prod(dims[i + 1 :]) for i in range(len(dims)))


class Layout:
    """Regions of the packed buffer and the tb_repack jobs that fill them from the
    source tensors of `index`. Matrices get `mat_type`, vectors F32."""

    def __init__(self, index: dict[str, Source], mat_type: int):
        self.index, self.mat_type = index, mat_type
        self.jobs: list[tuple] = []  # (src_off, dst_off, strides[4], dims[4], src_type, dst_type, fill, value)
        self.regions: dict[str, Region] = {}
        self.size = 0

    def _region(self, key: str, shape, mat: bool) -> Region:
        if key in self.regions:
            raise ValueError(f"region {key} defined twice")
        dtype = self.mat_type if mat else L.F32
        off = -(-self.size // 256) * 256
        self.size = off + prod(shape) * DST_SIZE[dtype]
        r = self.regions[key] = Region(off, tuple(int(d) for d in shape), dtype)
        return r

    def _job(self, dst_off: int, dst_type: int, dims, name: str | None = None, strides=None, base: int = 0,
             fill: float = 0.0) -> None:
        dims = tuple(int(d) for d in dims)
        if len(dims) > 4:
            raise ValueError("a job has at most 4 dimensions")
        dims4 = (1,) * (4 - len(dims)) + dims
        if name is None:
            self.jobs.append((0, dst_off, (0, 0, 0, 0), dims4, L.SRC_F32, dst_type, 1, fill))
            return
        src = self.index.get(name)
        if src is None:
            raise KeyError(f"weights have no tensor {name}")
        strides = _contiguous(dims) if strides is None else tuple(int(s) for s in strides)
        strides4 = (0,) * (4 - len(strides)) + strides
        last = base + sum((d - 1) * s for d, s in zip(dims4, strides4))
        if min(dims4) > 0 and (base < 0 or min(strides4) < 0 or last >= prod(src.shape)):
            raise ValueError(f"{name}: job reads outside the tensor of shape {src.shape}")
        self.jobs.append((src.off + base * SRC_SIZE[src.type], dst_off, strides4, dims4, src.type, dst_type, 0, 0.0))

    def tensor(self, key: str, name: str, shape=None, mat: bool = False) -> None:
        """The source tensor as is (reshaped to `shape`, same element count)."""
        src_shape = self.index[name].shape
        shape = src_shape if shape is None else tuple(shape)
        if prod(shape) != prod(src_shape):
            raise ValueError(f"{name}: shape {src_shape} does not reshape to {shape}")
        r = self._region(key, shape, mat)
        self._job(r.off, r.type, (prod(shape),), name)

    def view(self, key: str, name: str, dims, strides, base: int = 0, mat: bool = True) -> None:
        """Region of extents `dims` whose element i is source element base + i . strides."""
        r = self._region(key, dims, mat)
        self._job(r.off, r.type, dims, name, strides, base)

    def rows(self, key: str, shape, parts: list[tuple[str, int]], fill: float, mat: bool) -> None:
        """Region of `shape` whose rows from r0 on are the source tensor of each (name, r0);
        every other row is `fill`."""
        r = self._region(key, shape, mat)
        row = prod(shape[1:])
        at = 0
        for name, r0 in sorted(parts, key=lambda p: p[1]):
            n = prod(self.index[name].shape) // row
            if r0 < at or r0 + n > shape[0] or n * row != prod(self.index[name].shape):
                raise ValueError(f"{name} does not fit rows {r0}.. of {key}")
            if r0 > at:
                self._job(r.off + at * row * DST_SIZE[r.type], r.type, (r0 - at, row), fill=fill)
            self._job(r.off + r0 * row * DST_SIZE[r.type], r.type, (n, row), name)
            at = r0 + n
        if at < shape[0]:
            self._job(r.off + at * row * DST_SIZE[r.type], r.type, (shape[0] - at, row), fill=fill)

    def table(self):
        """The jobs as a tb_repack_job array."""
        arr = (L.RepackJob * len(self.jobs))()
        for j, (src_off, dst_off, strides, dims, st, dt, fill, value) in zip(arr, self.jobs):
            j.src_off, j.dst_off, j.src_type, j.dst_type, j.fill, j.value = src_off, dst_off, st, dt, fill, value
            j.stride[:] = strides
            j.dims[:] = dims
        return arr

    def run(self, source: torch.Tensor, out: torch.Tensor) -> None:
        """Fills `out` (uint8, device, at least `size` bytes) from `source` (uint8, device)
        on the current stream."""
        if out.numel() < self.size:
            raise ValueError("packed buffer smaller than the layout")
        table = self.table()
        jobs_dev = torch.empty(max(1, C.sizeof(table)), dtype=torch.uint8, device=out.device)
        stream = torch.cuda.current_stream(out.device).cuda_stream
        L.check(L.lib.tb_repack(table, len(self.jobs), jobs_dev.data_ptr(), source.data_ptr(), source.numel(),
                                out.data_ptr(), out.numel(), stream), "tb_repack")

    def tensor_of(self, buf: torch.Tensor, key: str) -> torch.Tensor:
        """The region `key` of the packed buffer as a torch tensor (a view)."""
        r = self.regions[key]
        dt = torch.bfloat16 if r.type == L.BF16 else torch.float32
        return buf.narrow(0, r.off, prod(r.shape) * DST_SIZE[r.type]).view(dt).view(r.shape)


def model_layout(index: dict[str, Source], layers: int, dtype: int) -> Layout:
    """Every region the engine's tb_model points at, keyed by field (per layer: "i.field")."""
    H, C_, P, K = L.HIDDEN, L.CHANNELS, L.PRED, L.KERNEL
    lay = Layout(index, dtype)
    p = "encoder.subsampling."
    lay.tensor("sub0_w", p + "layers.0.weight", (C_, 9))
    lay.tensor("sub0_b", p + "layers.0.bias")
    for i, (dw, pw) in enumerate(((2, 3), (5, 6))):
        lay.tensor(f"sub_dw_w{i}", p + f"layers.{dw}.weight", (C_, 9))
        lay.tensor(f"sub_dw_b{i}", p + f"layers.{dw}.bias")
        lay.tensor(f"sub_pw_w{i}", p + f"layers.{pw}.weight", (C_, C_), mat=True)
        lay.tensor(f"sub_pw_b{i}", p + f"layers.{pw}.bias")
    # Input columns (channel c, frequency f) -> (f, c): element [o, f, c] is source [o, c, f].
    lay.view("sub_linear_w", p + "linear.weight", (H, 16, C_), (C_ * 16, 1, 16))
    lay.tensor("sub_linear_b", p + "linear.bias")
    for i in range(layers):
        q = f"encoder.layers.{i}."
        for j, n in enumerate(NORMS):
            lay.tensor(f"{i}.norm_w{j}", q + n + ".weight")
            lay.tensor(f"{i}.norm_b{j}", q + n + ".bias")
        for f in (1, 2):
            lay.tensor(f"{i}.ff{f}_w1", q + f"feed_forward{f}.linear1.weight", mat=True)
            lay.tensor(f"{i}.ff{f}_w2", q + f"feed_forward{f}.linear2.weight", mat=True)
        a = q + "self_attn."
        lay.tensor(f"{i}.qkv", a + "qkv", mat=True)
        lay.tensor(f"{i}.o_proj", a + "o_proj.weight", mat=True)
        lay.tensor(f"{i}.bias_u", a + "bias_u", (H,))
        lay.tensor(f"{i}.bias_v", a + "bias_v", (H,))
        lay.tensor(f"{i}.rel_w", a + "relative_k_proj.weight", mat=True)
        c = q + "conv."
        # GLU pairs side by side: element [ch, j, k] is source row j * H + ch.
        lay.view(f"{i}.pw1", c + "pointwise_conv1.weight", (H, 2, H), (H, H * H, 1))
        lay.tensor(f"{i}.pw2", c + "pointwise_conv2.weight", (H, H), mat=True)
        lay.tensor(f"{i}.dw_w", c + "depthwise.weight", (H, K))
        lay.tensor(f"{i}.dw_b", c + "depthwise.bias")
    lay.tensor("enc_proj_w", "encoder_projector.weight", mat=True)
    lay.tensor("enc_proj_b", "encoder_projector.bias")
    lay.tensor("embedding", "decoder.embedding.weight", mat=True)
    for l in range(2):
        # Gates side by side per unit: element [u, g, k] is source row g * P + u.
        lay.view(f"lstm_w{l}", f"decoder.lstm.weight_l{l}", (P, 4, 2 * P), (2 * P, 2 * P * P, 1))
        lay.view(f"lstm_b{l}", f"decoder.lstm.bias_l{l}", (P, 4), (1, P), mat=False)
    if dtype == L.BF16:
        lay.view("lstm0_hh", "decoder.lstm.weight_l0", (P, 4, P), (2 * P, 2 * P * P, 1), base=P)
        lay.view("lstm0_ih", "decoder.lstm.weight_l0", (P, 4, P), (2 * P, 2 * P * P, 1))
    lay.tensor("dec_proj_w", "decoder.decoder_projector.weight", mat=True)
    lay.tensor("dec_proj_b", "decoder.decoder_projector.bias")
    lay.rows("joint_w", (L.JOINT_ROWS, P),
             [("joint.token_head.weight", 0), ("joint.duration_head.weight", L.TOKEN_ROWS)], 0.0, mat=True)
    lay.rows("joint_b", (L.JOINT_ROWS,),
             [("joint.token_head.bias", 0), ("joint.duration_head.bias", L.TOKEN_ROWS)], float("-inf"), mat=False)
    return lay


def upload_arrays(tensors: dict[str, np.ndarray], device) -> tuple[torch.Tensor, dict[str, Source]]:
    """Float arrays into one device buffer (float32, each at a 256-byte boundary)."""
    index, off = {}, 0
    for name, a in tensors.items():
        index[name] = Source(off, tuple(np.shape(a)), L.SRC_F32)
        off += -(-int(np.size(a)) * 4 // 256) * 256
    source = torch.empty(max(off, 256), dtype=torch.uint8, device=device)
    for name, a in tensors.items():
        s, n = index[name], int(np.size(a))
        if n:
            flat = torch.from_numpy(np.ascontiguousarray(a, np.float32).reshape(-1))
            source.narrow(0, s.off, 4 * n).view(torch.float32).copy_(flat)
    return source, index


def cache_index(path: str | Path) -> tuple[int, int, dict[str, Source]]:
    """(data block offset, data block bytes, tensors) of a safetensors file of F16 / F32
    tensors, as tinybark writes its cache (tinybark/weights.py:92-103)."""
    size = Path(path).stat().st_size
    with open(path, "rb") as f:
        n = int.from_bytes(f.read(8), "little")
        if n <= 0 or 8 + n > size:
            raise ValueError(f"{path}: not a safetensors file")
        header = json.loads(f.read(n))
    body = 8 + n
    index = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        t = SRC_TYPES.get(info["dtype"])
        if t is None:
            raise ValueError(f"{name}: unsupported dtype {info['dtype']}")
        start, end = info["data_offsets"]
        shape = tuple(info["shape"])
        if end - start != prod(shape) * SRC_SIZE[t] or end > size - body or start % SRC_SIZE[t]:
            raise ValueError(f"{name}: data offsets {start}..{end} do not hold {info['dtype']} {shape}")
        index[name] = Source(start, shape, t)
    spans = sorted((s.off, s.off + prod(s.shape) * SRC_SIZE[s.type], n) for n, s in index.items())
    for (_, end, a), (start, _, b) in zip(spans, spans[1:]):
        if start < end:
            raise ValueError(f"{a} and {b} overlap in the data block")
    return body, size - body, index


def aligned_runs(index: dict[str, Source]) -> tuple[list[tuple[int, int, int]], int, dict[str, Source]]:
    """Where each tensor of a file's data block goes in device memory so that every one
    starts 16-byte aligned: tensors in file order form runs of equal offset mod 16, and
    each run is moved as a whole, by at most 15 bytes more than the run before it (the
    cache tinybark writes has one 5-element f16 tensor, the duration bias, after which
    every tensor is 10 bytes off a boundary). Returns the runs as (start, end, device
    start) byte ranges of the block, the device bytes, and the tensors at their device
    offsets."""
    names = sorted(index, key=lambda k: index[k].off)
    runs: list[list[int]] = []  # [start, end, shift]
    moved: dict[str, Source] = {}
    for name in names:
        s = index[name]
        end = s.off + prod(s.shape) * SRC_SIZE[s.type]
        if runs and (s.off + runs[-1][2]) % 16 == 0:
            runs[-1][1] = max(runs[-1][1], end)
        else:
            shift = runs[-1][2] if runs else 0
            shift += -(s.off + shift) % 16
            runs.append([s.off, end, shift])
        moved[name] = Source(s.off + runs[-1][2], s.shape, s.type)
    pieces = [(a, b, a + d) for a, b, d in runs]
    return pieces, (pieces[-1][2] + pieces[-1][1] - pieces[-1][0]) if pieces else 0, moved


def slice_copies(start: int, length: int, pieces) -> list[tuple[int, int, int]]:
    """The copies that move bytes [start, start + length) of a block to device memory, as
    (offset in the slice, device offset, bytes): the part of each piece (start, end,
    device start) that the slice holds."""
    out = []
    for a, e, d in pieces:
        lo, hi = max(a, start), min(e, start + length)
        if lo < hi:
            out.append((lo - start, d + lo - a, hi - lo))
    return out


def upload_file(path: str | Path, offset: int, nbytes: int, device, pieces=None, dev_bytes: int | None = None,
                slice_bytes: int = 8 << 20, threads: int | None = None) -> torch.Tensor:
    """Bytes [offset, offset + nbytes) of a file in device memory (uint8): each piece
    (start, end, device start) of that range at its device offset (default: the whole range
    at 0). Worker threads (by default one per core, at most 12) read slices into a ring of
    two pinned buffers per thread while the slices already read are copied to the GPU on a
    copy stream; a buffer is read into again once its copies have finished. A 1.25 GB file
    in the page cache moves at about 34 GB/s with 12 threads on a 16-core host (23 GB/s
    with 4)."""
    pieces = [(0, nbytes, 0)] if pieces is None else pieces
    threads = threads or max(2, min(12, os.cpu_count() or 4))
    buffers = 2 * threads
    dst = torch.empty(max(nbytes if dev_bytes is None else dev_bytes, 256), dtype=torch.uint8, device=device)
    n_slices = -(-nbytes // slice_bytes)
    if n_slices == 0:
        return dst
    nbuf = min(buffers, n_slices)
    bufs = [torch.empty(slice_bytes, dtype=torch.uint8, pin_memory=True) for _ in range(nbuf)]
    views = [memoryview(b.numpy()) for b in bufs]
    copied: list[torch.cuda.Event | None] = [None] * nbuf
    stream = torch.cuda.Stream(device)
    fd = os.open(path, os.O_RDONLY)

    def read(k: int) -> tuple[int, int, int]:
        b = k % nbuf
        if copied[b] is not None:
            copied[b].synchronize()
        start, length = k * slice_bytes, min(slice_bytes, nbytes - k * slice_bytes)
        got = 0
        while got < length:
            r = os.preadv(fd, [views[b][got:length]], offset + start + got)
            if r <= 0:
                raise OSError(f"{path}: file ends before byte {offset + start + length}")
            got += r
        return b, start, length

    try:
        with ThreadPoolExecutor(threads) as pool:
            pending = [pool.submit(read, k) for k in range(nbuf)]
            for k in range(n_slices):
                b, start, length = pending[k].result()
                with torch.cuda.stream(stream):
                    for at, to, n in slice_copies(start, length, pieces):
                        dst.narrow(0, to, n).copy_(bufs[b].narrow(0, at, n), non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(stream)
                copied[b] = ev
                if k + nbuf < n_slices:
                    pending.append(pool.submit(read, k + nbuf))
    finally:
        os.close(fd)
    torch.cuda.current_stream(device).wait_stream(stream)
    return dst


def upload_cache(path: str | Path, device) -> tuple[torch.Tensor, dict[str, Source]]:
    """The cache file's tensors on the GPU, each 16-byte aligned (aligned_runs), with their
    index."""
    offset, nbytes, index = cache_index(path)
    pieces, dev_bytes, moved = aligned_runs(index)
    return upload_file(path, offset, nbytes, device, pieces, dev_bytes), moved
