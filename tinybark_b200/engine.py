"""Host side of the cuda backend: the converted weights repacked on the GPU for the
kernels, batch planning, and the front-end -> encoder -> TDT decode pipeline, all
through libtbcuda's C ABI. torch only allocates device memory and supplies the stream.

Clips of a batch are packed end to end at every stage (no padding): the reference pads
to multiples of 2.56 s and masks (tinybark/tinygrad/model.py:15-20,140-158), and on
valid frames both give the same values, since every masked position the reference
zeroes is a zero-padding position here.
"""

from __future__ import annotations

import ctypes as C
import os
import time
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib as L
from . import lengths, pack, tables

DTYPES = {"fp32": L.F32, "bf16": L.BF16}
MAX_DECODE_GROUPS = 8
# Smallest part upload_parts makes (samples; 60 s of audio, about 750 encoder rows). The
# residual GEMMs of at most 256 rows (about 20 s of audio) split K over several CTAs whose
# sums land in the order their atomic adds take, so their last bits can differ from call
# to call. A batch of more than 256 encoder rows is cut only into parts of more than 256
# rows, so its encoder gives the same bits on every call.
MIN_PART_SAMPLES = 60 * 16000
# Every token id as a Python int, gathered by token rows: a lane's list then shares these
# objects instead of creating one int per emitted token (half the conversion time).
_TOKEN_INTS = np.array(range(L.VOCAB), dtype=object)


def token_list(row: np.ndarray) -> list[int]:
    """A row of token ids (ints below the vocabulary size) as a list of Python ints."""
    return _TOKEN_INTS[row].tolist()


def part_edges(off: np.ndarray, fractions, min_samples: int = MIN_PART_SAMPLES) -> list[int]:
    """Clip indices where upload_parts cuts a batch whose clips start at sample offsets
    `off` [clips + 1]: [0, ..., clips], each cut at the first clip boundary at or past a
    fraction of the samples, except that no part is shorter than `min_samples` (a cut that
    would leave one is dropped, its clips going with the next part)."""
    clips, total = len(off) - 1, int(off[-1])
    cuts = np.searchsorted(off, [f * total for f in fractions]).tolist()
    edges = [0]
    for c in sorted(set(c for c in cuts if 0 < c < clips)):
        if off[c] - off[edges[-1]] >= min_samples and total - off[c] >= min_samples:
            edges.append(c)
    edges.append(clips)
    return edges


def lane_order(idx: list[int], frames: list[int], groups: int | None = None) -> list[int]:
    """Orders clips `idx` (frame counts `frames[i]`) for the decoder: longest first, and
    for the graph decoder with `groups` > 1 concurrent groups, dealt round-robin into
    the groups, the groups concatenated. Each group then holds clips of every length,
    and within a group the lanes finish from its end, so its GEMMs shrink to the lanes
    still running."""
    order = sorted(idx, key=lambda i: -frames[i])
    g = max(1, groups or 1)
    return [i for k in range(g) for i in order[k::g]]


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def positions(length: int) -> torch.Tensor:
    """(2*length-1, 1024) float32: row n is relative position length-1-n as interleaved
    [sin, cos] (tinybark/tinygrad/model.py:30-34), computed in float32 as
    transformers' ParakeetEncoderRelPositionalEncoding does."""
    inv_freq = 1.0 / (10000.0 ** (torch.arange(0, L.HIDDEN, 2, dtype=torch.int64).float() / L.HIDDEN))
    pos = torch.arange(length - 1, -length, -1).float()
    freqs = pos[:, None] * inv_freq[None, :]
    return torch.stack([freqs.sin(), freqs.cos()], -1).reshape(2 * length - 1, L.HIDDEN)


@dataclass
class Plan:
    """Offsets and work lists of one batch, on the device, behind a tb_batch."""

    frames: np.ndarray
    t3: np.ndarray
    batch: L.Batch
    meta: torch.Tensor
    t3_off: torch.Tensor
    frame_off: torch.Tensor
    caps: torch.Tensor
    max_cap: int


def plan_arrays(frames, sub_rows: int, attn_rows: int) -> dict[str, np.ndarray]:
    """Host-side metadata of a packed batch: cumulative row offsets at each subsampling
    stage, the clip of every row, the (clip, first row) work items of the subsampling
    and attention kernels (longest clips first) and each clip's greedy-loop cap."""
    f = np.asarray(frames, np.int64)
    if len(f) == 0 or f.min() < 2:
        raise ValueError("every clip needs at least 2 feature frames")
    t1 = (f - 1) // 2 + 1
    t2 = (t1 - 1) // 2 + 1
    t3 = (t2 - 1) // 2 + 1
    off = lambda n: np.concatenate([[0], np.cumsum(n)]).astype(np.int32)
    ids = np.arange(len(f), dtype=np.int32)
    order = np.argsort(-t3, kind="stable")
    def tiles(n, step):  # (clip, first row) of every `step`-row work item, clips in `order`
        per = (n[order] + step - 1) // step
        clip = np.repeat(order, per)
        first = np.arange(int(per.sum())) - np.repeat(np.cumsum(per) - per, per)
        return np.stack([clip, first * step], 1).astype(np.int32).reshape(-1)

    return {
        "frames": f, "t3": t3,
        "frame_off": off(f), "t1_off": off(t1), "t2_off": off(t2), "t3_off": off(t3),
        "t2_clip": np.repeat(ids, t2), "t3_clip": np.repeat(ids, t3),
        "sub_tiles": tiles(t2, sub_rows), "attn_tiles": tiles(t3, attn_rows),
        "caps": np.array([lengths.decode_cap(int(n)) for n in f], np.int32),
    }


class Engine:
    """The model on one GPU. `tensors` is the converted layout (tinybark/weights.py:62-89):
    the path of tinybark's fp16 cache file of it (tinybark/weights.py:92-120), read
    straight into GPU memory, or a dict of float32 arrays; `dtype` is "fp32" (parity) or
    "bf16" (throughput). `ffn` "mxfp8" (bf16 only) runs the FFN GEMMs block-scaled: their
    weights quantized to MXFP8 at load, their inputs at run time (a lower-precision option,
    tinybark/docs/2026-10-24-learnings.md:133-146; "bf16", the default, keeps them bf16)."""

    def __init__(self, tensors: dict[str, np.ndarray], config: dict, dtype: str = "bf16", device="cuda",
                 max_len: int = 512, ffn: str = "bf16"):
        if ffn not in ("bf16", "mxfp8") or (ffn == "mxfp8" and dtype != "bf16"):
            raise ValueError(f"ffn must be 'bf16', or 'mxfp8' with dtype 'bf16' (got {ffn!r}, {dtype!r})")
        if not torch.cuda.is_available():
            raise RuntimeError("the cuda backend needs a CUDA GPU")
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.dtype = DTYPES[dtype]
        self.tdtype = torch.bfloat16 if self.dtype == L.BF16 else torch.float32
        self.layers = config["encoder_config"]["num_hidden_layers"]
        self.sub_rows, self.attn_rows = L.tile_rows(self.dtype)
        self._keep: list[torch.Tensor] = []
        self._pinned: torch.Tensor | None = None  # sample staging buffer of upload()
        self._staged = None  # event after the last copy out of it
        self._threads = None
        self._side: torch.cuda.Stream | None = None  # copies of finished lanes during decode
        self._copy: torch.cuda.Stream | None = None  # sample copies of upload_parts()
        self._tok_host: torch.Tensor | None = None  # pinned token rows of decode_lists()
        with torch.cuda.device(self.device):
            self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
            self.host_flag = torch.zeros(2 * MAX_DECODE_GROUPS, dtype=torch.int32).pin_memory()
            self._pack(tensors)
            self.ffn = ffn
            if ffn == "mxfp8":
                self._quantize_ffn()
            self.max_len = 0
            self.ensure_len(max_len)

    # ------------------------------------------------------------------ weights

    def _vec(self, a: np.ndarray, dtype=torch.float32) -> torch.Tensor:
        t = torch.from_numpy(np.ascontiguousarray(a)).to(self.device, dtype).contiguous()
        self._keep.append(t)
        return t

    def _pack(self, w) -> None:
        """The weights into one packed device buffer (pack.model_layout), from a path of
        tinybark's fp16 cache file (its data block uploaded as is) or from a dict of the
        converted tensors; then the kernels' pointers into it."""
        t0 = time.perf_counter()
        if isinstance(w, (str, os.PathLike)):
            source, index = pack.upload_cache(w, self.device)
        else:
            source, index = pack.upload_arrays(w, self.device)
        lay = pack.model_layout(index, self.layers, self.dtype)
        blob = torch.zeros(lay.size, dtype=torch.uint8, device=self.device)
        torch.cuda.synchronize(self.device)
        t1 = time.perf_counter()
        lay.run(source, blob)
        torch.cuda.synchronize(self.device)
        t2 = time.perf_counter()
        del source
        self.layout, self._blob = lay, blob
        base = blob.data_ptr()

        def at(key: str) -> int:
            return base + lay.regions[key].off

        m = L.Model()
        m.dtype, m.layers = self.dtype, self.layers
        m.sub0_w, m.sub0_b = at("sub0_w"), at("sub0_b")
        for i in range(2):
            m.sub_dw_w[i], m.sub_dw_b[i] = at(f"sub_dw_w{i}"), at(f"sub_dw_b{i}")
            m.sub_pw_w[i], m.sub_pw_b[i] = at(f"sub_pw_w{i}"), at(f"sub_pw_b{i}")
        m.sub_linear_w, m.sub_linear_b = at("sub_linear_w"), at("sub_linear_b")

        self._layer_arr = (L.Layer * self.layers)()
        self._rel_w: list[torch.Tensor] = []
        self._pos_bias: list[tuple[torch.Tensor, torch.Tensor]] = []
        for i in range(self.layers):
            lay_i = self._layer_arr[i]
            for j in range(len(pack.NORMS)):
                lay_i.norm_w[j], lay_i.norm_b[j] = at(f"{i}.norm_w{j}"), at(f"{i}.norm_b{j}")
            lay_i.ff1_w1, lay_i.ff1_w2 = at(f"{i}.ff1_w1"), at(f"{i}.ff1_w2")
            lay_i.ff2_w1, lay_i.ff2_w2 = at(f"{i}.ff2_w1"), at(f"{i}.ff2_w2")
            lay_i.qkv, lay_i.o_proj = at(f"{i}.qkv"), at(f"{i}.o_proj")
            lay_i.bias_u, lay_i.bias_v = at(f"{i}.bias_u"), at(f"{i}.bias_v")
            self._pos_bias.append((lay.tensor_of(blob, f"{i}.bias_u"), lay.tensor_of(blob, f"{i}.bias_v")))
            self._rel_w.append(lay.tensor_of(blob, f"{i}.rel_w"))
            lay_i.pw1, lay_i.pw2 = at(f"{i}.pw1"), at(f"{i}.pw2")
            lay_i.dw_w, lay_i.dw_b = at(f"{i}.dw_w"), at(f"{i}.dw_b")
        m.layer = C.cast(self._layer_arr, C.POINTER(L.Layer))
        m.enc_proj_w, m.enc_proj_b = at("enc_proj_w"), at("enc_proj_b")
        m.embedding = at("embedding")
        for l in range(2):
            m.lstm_w[l], m.lstm_b[l] = at(f"lstm_w{l}"), at(f"lstm_b{l}")
        if self.dtype == L.BF16:
            # The persistent decoder takes layer 0's gates as E[token] + W_hh . h0: the
            # input term of every token, E = embedding . W_ih^T, computed once here.
            m.lstm0_hh = at("lstm0_hh")
            emb = lay.tensor_of(blob, "embedding")
            w_ih = lay.tensor_of(blob, "lstm0_ih").view(4 * L.PRED, L.PRED)
            table = torch.empty(L.VOCAB, 4 * L.PRED, device=self.device, dtype=torch.float32)
            self._keep.append(table)
            from . import kernels

            kernels.gemm(emb, w_ih, L.Epilogue(kind=L.EPI_STORE, out_dtype=L.F32, out=table.data_ptr(),
                                               ldo=4 * L.PRED))
            m.lstm0_emb = _ptr(table)
        m.dec_proj_w, m.dec_proj_b = at("dec_proj_w"), at("dec_proj_b")
        m.joint_w, m.joint_b = at("joint_w"), at("joint_b")

        mel_w, mel_start, mel_off = tables.sparse_mel()
        m.window = _ptr(self._vec(tables.window()))
        m.mel_w = _ptr(self._vec(mel_w))
        m.mel_start = _ptr(self._vec(mel_start, torch.int32))
        m.mel_off = _ptr(self._vec(mel_off, torch.int32))
        self.model = m
        self.load_seconds = {"upload": t1 - t0, "repack": t2 - t1}

    def _quantize_ffn(self) -> None:
        """The FFN weights of every layer to MXFP8 on the GPU (tb_mx_quantize of the packed
        bf16 matrices), pointed at by tb_model.ffn_mx."""
        from . import kernels

        self._mx = []
        arr = (L.MXWeight * (4 * self.layers))()
        for i in range(self.layers):
            for j, key in enumerate(("ff1_w1", "ff1_w2", "ff2_w1", "ff2_w2")):
                q = kernels.MX(self.layout.tensor_of(self._blob, f"{i}.{key}"))
                self._mx.append(q)
                arr[4 * i + j].codes, arr[4 * i + j].scales = q.codes.data_ptr(), q.scales.data_ptr()
        self._mx_arr = arr
        self.model.ffn_mx = C.cast(arr, C.c_void_p)
        torch.cuda.synchronize(self.device)

    def ensure_len(self, t3: int) -> None:
        """Projected position tables (pos @ relative_k_proj^T, one per layer) covering
        clips of up to `t3` encoder frames; computed once per length, off the per-clip
        path, as tinybark/tinygrad/model.py:130-138 caches them per bucket."""
        if t3 <= self.max_len:
            return
        n = max(-(-t3 // 128) * 128, 128)
        pos = positions(n).to(self.device, self.tdtype).contiguous()
        rows = 2 * n - 1
        from . import kernels

        self._rel = []
        for i in range(self.layers):
            r = torch.empty(rows, L.HIDDEN, device=self.device, dtype=self.tdtype)
            ep = L.Epilogue(kind=L.EPI_STORE, out_dtype=self.dtype, out=r.data_ptr(), ldo=L.HIDDEN)
            self._gemm(pos, self._rel_w[i], ep)
            c = kernels.rel_bias(r, *self._pos_bias[i])
            self._rel.append((r, c))
            self._layer_arr[i].rel = r.data_ptr()
            self._layer_arr[i].rel_c = c.data_ptr()
        self.max_len = n
        self.model.max_len = n
        self.check()

    def _gemm(self, a: torch.Tensor, w: torch.Tensor, ep: L.Epilogue) -> None:
        L.check(L.lib.tb_gemm(self.dtype, a.data_ptr(), a.stride(0), w.data_ptr(), a.shape[0], w.shape[0], a.shape[1],
                              C.byref(ep), self.err.data_ptr(), _stream(self.device)), "tb_gemm")

    def check(self) -> None:
        """Synchronises and raises if a kernel reported a device-side timeout."""
        torch.cuda.synchronize(self.device)
        code = int(self.err.item())
        if code:
            self.err.zero_()
            names = [v for k, v in L.DEVICE_ERRORS.items() if code & k]
            raise RuntimeError("device error: " + ", ".join(names or [str(code)]))

    # ------------------------------------------------------------------ batches

    def plan(self, frames: list[int] | np.ndarray) -> Plan:
        """Packed offsets and work lists for clips of the given feature-frame counts
        (each at least 2), uploaded in one copy."""
        parts = plan_arrays(frames, self.sub_rows, self.attn_rows)
        self.ensure_len(int(parts["t3"].max()))
        names = ("frame_off", "t1_off", "t2_off", "t3_off", "t2_clip", "t3_clip", "sub_tiles", "attn_tiles", "caps")
        host = np.concatenate([parts[n] for n in names]).astype(np.int32)
        meta = torch.from_numpy(host).pin_memory().to(self.device, non_blocking=True)
        views, start = {}, 0
        for n in names:
            views[n] = meta[start : start + len(parts[n])]
            start += len(parts[n])
        b = L.Batch()
        b.clips = len(parts["frames"])
        b.frames_total, b.t1_total = int(parts["frame_off"][-1]), int(parts["t1_off"][-1])
        b.t2_total, b.t3_total = int(parts["t2_off"][-1]), int(parts["t3_off"][-1])
        for n in names[:6]:
            setattr(b, n, views[n].data_ptr())
        b.sub_tiles, b.n_sub_tiles = views["sub_tiles"].data_ptr(), len(parts["sub_tiles"]) // 2
        b.attn_tiles, b.n_attn_tiles = views["attn_tiles"].data_ptr(), len(parts["attn_tiles"]) // 2
        b.max_t3 = int(parts["t3"].max())
        return Plan(parts["frames"], parts["t3"], b, meta, views["t3_off"], views["frame_off"], views["caps"],
                    int(parts["caps"].max()))

    # ------------------------------------------------------------------ stages

    def features(self, samples: torch.Tensor, sample_off: torch.Tensor, plan: Plan) -> torch.Tensor:
        """Packed samples (device; float32, or int16 PCM converted on the device) to packed
        normalised log-mel features [frames, 128]."""
        b = plan.batch
        feats = torch.empty(b.frames_total, L.MELS, device=self.device, dtype=torch.float32)
        nbytes = L.lib.tb_frontend_workspace_bytes(b.clips, b.frames_total)
        ws = torch.empty(nbytes, device=self.device, dtype=torch.uint8)
        fn = L.lib.tb_frontend_pcm16 if samples.dtype == torch.int16 else L.lib.tb_frontend
        L.check(fn(C.byref(self.model), samples.data_ptr(), sample_off.data_ptr(), plan.frame_off.data_ptr(), b.clips,
                   b.frames_total, int(plan.frames.max()), feats.data_ptr(), ws.data_ptr(), nbytes,
                   _stream(self.device)), "tb_frontend")
        return feats

    def encode(self, feats: torch.Tensor, plan: Plan, out: torch.Tensor | None = None) -> torch.Tensor:
        """Packed features to packed encoder frames projected for the joint, [t3_total, 640]
        float32 (into `out` if given: contiguous rows of that shape)."""
        b = plan.batch
        enc = torch.empty(b.t3_total, L.PRED, device=self.device, dtype=torch.float32) if out is None else out
        if enc.shape != (b.t3_total, L.PRED) or not enc.is_contiguous() or enc.dtype != torch.float32:
            raise ValueError("encode: out must be a contiguous float32 [t3_total, 640] tensor")
        if self.ffn == "mxfp8":
            nbytes = L.lib.tb_encoder_workspace_bytes_mx(b.t2_total, b.t3_total)
        else:
            nbytes = L.lib.tb_encoder_workspace_bytes(self.dtype, b.t2_total, b.t3_total)
        ws = torch.empty(nbytes, device=self.device, dtype=torch.uint8)
        L.check(L.lib.tb_encoder_forward(C.byref(self.model), C.byref(b), feats.data_ptr(), enc.data_ptr(),
                                         ws.data_ptr(), nbytes, self.err.data_ptr(), _stream(self.device)),
                "tb_encoder_forward")
        return enc

    def decode(self, enc: torch.Tensor, plan: Plan, early_exit: bool = True,
               groups: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """Greedy TDT decoding of every clip; returns device (tokens [clips, max_cap], counts [clips]).
        `groups` None or 0: the library's default decoder (bf16: one persistent kernel for
        the whole loop; fp32: graph-replayed GEMM kernels); 1..8: the graph decoder with
        that many concurrent lane groups (clips in lane_order for balanced groups). Every
        choice gives the same tokens."""
        b = plan.batch
        g = 0 if groups is None else int(groups)
        tokens = torch.empty(b.clips, plan.max_cap, device=self.device, dtype=torch.int32)
        counts = torch.empty(b.clips, device=self.device, dtype=torch.int32)
        nbytes = L.lib.tb_decode_workspace_bytes(self.dtype, b.clips, g)
        ws = torch.empty(nbytes, device=self.device, dtype=torch.uint8)
        flag = self.host_flag.data_ptr() if early_exit else None
        L.check(L.lib.tb_tdt_decode(C.byref(self.model), enc.data_ptr(), plan.t3_off.data_ptr(), plan.caps.data_ptr(),
                                    b.clips, plan.max_cap, g, tokens.data_ptr(), counts.data_ptr(), ws.data_ptr(),
                                    nbytes, flag, self.err.data_ptr(), _stream(self.device)), "tb_tdt_decode")
        self._last_decode = (ws, b.clips, g)
        return tokens, counts

    def lane_iterations(self) -> torch.Tensor:
        """Greedy-loop iterations each lane ran in the last decode (groups 0 or 1), [clips]
        int32 on the device: the decode's algorithmic work is their sum times the work of
        one iteration."""
        ws, lanes, g = self._last_decode
        it = torch.empty(lanes, dtype=torch.int32, device=self.device)
        L.check(L.lib.tb_decode_lane_iterations(ws.data_ptr(), self.dtype, lanes, g, it.data_ptr(),
                                                _stream(self.device)), "tb_decode_lane_iterations")
        return it

    # ------------------------------------------------------------------ end to end

    def upload(self, clips: list[np.ndarray]) -> tuple[torch.Tensor, torch.Tensor]:
        """Packs sample arrays (all float32, or all int16 PCM) into the engine's pinned
        staging buffer (kept and grown across calls: pinning memory is slow) with a few
        host threads, in slices whose copy to the device starts as soon as each is packed,
        so packing and the transfer overlap."""
        pcm = len(clips) > 0 and all(c.dtype == np.int16 for c in clips)
        tdt = torch.int16 if pcm else torch.float32
        sizes = np.array([len(c) for c in clips], np.int64)
        off = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
        total = int(off[-1])
        if self._staged is not None:
            self._staged.synchronize()  # the previous transfer out of the buffer is done
        nbytes = (total + 1) * (2 if pcm else 4)
        if self._pinned is None or self._pinned.numel() < nbytes:
            self._pinned = torch.empty(max(nbytes, int(nbytes * 1.25)), dtype=torch.uint8).pin_memory()
        staged = self._pinned[: (total + 1) * (2 if pcm else 4)].view(tdt)
        hv = staged.numpy()
        hv[total] = 0

        def pack(i: int) -> None:
            hv[off[i] : off[i + 1]] = clips[i]

        samples = torch.empty(total, device=self.device, dtype=tdt)
        if total >= 1 << 22:
            # About eight slices of whole clips; each copied once packed.
            bounds = np.searchsorted(off, np.linspace(0, total, 9)[1:-1]).tolist()
            edges = [0, *sorted(set(b for b in bounds if 0 < b < len(clips))), len(clips)]
            for a, b in zip(edges[:-1], edges[1:]):
                list(self._pool().map(pack, range(a, b)))
                samples[off[a] : off[b]].copy_(staged[off[a] : off[b]], non_blocking=True)
        else:
            for i in range(len(clips)):
                pack(i)
            samples.copy_(staged[:total], non_blocking=True)
        self._staged = torch.cuda.Event()
        self._staged.record()
        sample_off = torch.from_numpy(off).pin_memory().to(self.device, non_blocking=True)
        return samples, sample_off

    def upload_parts(self, clips: list[np.ndarray], fractions=(1 / 64, 1 / 16, 1 / 4, 1 / 2), slice_bytes=64 << 20):
        """upload() in parts, for callers that start on each part while the next is still
        on its way: yields (first clip, end clip, samples, sample_off) per part, the copy
        of each part (on the engine's copy stream) ordered before the current stream's
        next work. Parts are contiguous clip ranges ending at these fractions of the
        samples: a small first part leaves little of the transfer exposed, and each later
        part (at most about three times the one before, the ratio of encoder time to transfer
        time) is packed and copied while the previous one is computed. Within a part the
        clips are packed in slices of about `slice_bytes`, each copied as soon as it is
        packed, so packing and copying overlap. No part is shorter than MIN_PART_SAMPLES
        (unless the whole batch is)."""
        pcm = len(clips) > 0 and all(c.dtype == np.int16 for c in clips)
        tdt = torch.int16 if pcm else torch.float32
        sizes = np.array([len(c) for c in clips], np.int64)
        off = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
        total = int(off[-1])
        if self._staged is not None:
            self._staged.synchronize()
        nbytes = (total + 1) * (2 if pcm else 4)
        if self._pinned is None or self._pinned.numel() < nbytes:
            self._pinned = torch.empty(max(nbytes, int(nbytes * 1.25)), dtype=torch.uint8).pin_memory()
        staged = self._pinned[:nbytes].view(tdt)
        hv = staged.numpy()
        samples = torch.empty(total, device=self.device, dtype=tdt)
        if self._copy is None:
            self._copy = torch.cuda.Stream(self.device)
        cur = torch.cuda.current_stream(self.device)
        self._copy.wait_stream(cur)
        edges = part_edges(off, fractions)

        def pack(i: int) -> None:
            hv[off[i] : off[i + 1]] = clips[i]

        per = 2 if pcm else 4
        for a, b in zip(edges[:-1], edges[1:]):
            # Slices of whole clips, about slice_bytes each.
            want = max(1, int((off[b] - off[a]) * per // slice_bytes))
            marks = np.searchsorted(off, np.linspace(off[a], off[b], want + 1)[1:-1]).tolist()
            sl = [a, *sorted(set(m for m in marks if a < m < b)), b]
            for c, d in zip(sl[:-1], sl[1:]):
                list(self._pool().map(pack, range(c, d)))
                with torch.cuda.stream(self._copy):
                    samples[off[c] : off[d]].copy_(staged[off[c] : off[d]], non_blocking=True)
            with torch.cuda.stream(self._copy):
                ready = torch.cuda.Event()
                ready.record(self._copy)
            cur.wait_event(ready)
            sub_off = torch.from_numpy(off[a : b + 1] - off[a]).pin_memory().to(self.device, non_blocking=True)
            yield a, b, samples[off[a] : off[b]], sub_off
        self._staged = ready
        samples.record_stream(self._copy)

    def _pool(self):
        if self._threads is None:
            from concurrent.futures import ThreadPoolExecutor

            self._threads = ThreadPoolExecutor(max_workers=8)
        return self._threads

    def _encode_batch(self, clips: list[np.ndarray]):
        """Front-end and encoder of every clip of at least 2 frames: (kept clip indices in
        lane order, encoder rows, plan), or None if no clip is kept."""
        clips = [np.asarray(c).reshape(-1) for c in clips]
        if not all(c.dtype == np.int16 for c in clips):  # 16-bit PCM stays 16-bit up to the GPU
            clips = [np.asarray(c, np.float32) for c in clips]
        frames = [lengths.frames(len(c)) for c in clips]
        keep = lane_order([i for i, f in enumerate(frames) if f >= 2], frames)
        if not keep:
            return None
        kf = [frames[i] for i in keep]
        t3 = np.asarray(kf, np.int64)
        for _ in range(3):
            t3 = (t3 - 1) // 2 + 1  # the three stride-2 subsampling stages
        t3_off = np.concatenate([[0], np.cumsum(t3)]).astype(np.int64)
        enc = torch.empty(int(t3_off[-1]), L.PRED, device=self.device, dtype=torch.float32)
        # Front-end and encoder part by part, each part's samples copied while the
        # previous part is computed. The whole batch's plan (for the decode) is built once
        # the first part's work is queued.
        plan = None
        for a, b, samples, sample_off in self.upload_parts([clips[i] for i in keep]):
            whole = (a, b) == (0, len(keep))
            sub = self.plan(kf if whole else kf[a:b])
            feats = self.features(samples, sample_off, sub)
            self.encode(feats, sub, out=enc[t3_off[a] : t3_off[b]])
            if plan is None:
                plan = sub if whole else self.plan(kf)
        return keep, enc, plan

    def tokens_batch(self, clips: list[np.ndarray]) -> list[list[int]]:
        """Token ids of every clip (16 kHz mono float32 samples), as the reference's
        Bark.tokens returns them one clip at a time (tinybark/tinygrad/model.py:196-234)."""
        out: list[list[int]] = [[] for _ in clips]
        with torch.cuda.device(self.device):
            batch = self._encode_batch(clips)
            if batch is None:
                return out
            keep, enc, plan = batch
            lists = self.decode_lists(enc, plan)
        for j, i in enumerate(keep):
            out[i] = lists[j]
        return out

    def text_table(self, off: np.ndarray, data: np.ndarray) -> tuple[torch.Tensor, torch.Tensor]:
        """A tokenizer's piece table (text.Tokenizer.table) on this GPU."""
        return (torch.from_numpy(np.ascontiguousarray(off, np.int32)).to(self.device),
                torch.from_numpy(np.ascontiguousarray(data, np.uint8)).to(self.device))

    def texts(self, tokens: torch.Tensor, counts: torch.Tensor, table) -> list[bytes]:
        """Each lane's piece bytes joined on the GPU (tb_text_offsets, tb_text_bytes):
        token rows [lanes, ld] and counts [lanes] int32 on this GPU, `table` from
        text_table. text.finish turns one into its text."""
        off_t, data = table
        n, ld = tokens.shape
        stream = _stream(self.device)
        off = torch.empty(n + 1, dtype=torch.int64, device=self.device)
        L.check(L.lib.tb_text_offsets(tokens.data_ptr(), ld, counts.data_ptr(), n, off_t.data_ptr(), off_t.numel() - 1,
                                      off.data_ptr(), self.err.data_ptr(), stream), "tb_text_offsets")
        o = off.cpu().numpy()
        text = torch.empty(max(int(o[-1]), 1), dtype=torch.uint8, device=self.device)
        L.check(L.lib.tb_text_bytes(tokens.data_ptr(), ld, counts.data_ptr(), n, off_t.data_ptr(), data.data_ptr(),
                                    data.numel(), off_t.numel() - 1, off.data_ptr(), text.data_ptr(), int(o[-1]),
                                    stream), "tb_text_bytes")
        raw = text[: int(o[-1])].cpu().numpy().tobytes()
        self.check()
        return [raw[o[i] : o[i + 1]] for i in range(n)]

    def texts_batch(self, clips: list[np.ndarray], table) -> list[bytes]:
        """The joined piece bytes of every clip's transcript: the tokens_batch pipeline, with
        the token rows turned into bytes on the GPU instead of copied out as lists."""
        out = [b"" for _ in clips]
        with torch.cuda.device(self.device):
            batch = self._encode_batch(clips)
            if batch is None:
                return out
            keep, enc, plan = batch
            flag = self.host_flag.numpy()
            flag[0], flag[1] = plan.batch.clips, -1
            tokens, counts = self.decode(enc, plan)
            texts = self.texts(tokens, counts, table)
        for j, i in enumerate(keep):
            out[i] = texts[j]
        return out

    def decode_lists(self, enc: torch.Tensor, plan: Plan) -> list[list[int]]:
        """decode(), with each lane's tokens as a Python list. With the persistent decoder
        (bf16) the lanes that have stopped are copied out and converted while the loop is
        still running: the kernel publishes a row bound every few iterations (lanes at or
        above it are final), so little conversion is left once it ends."""
        n, cap = plan.batch.clips, plan.max_cap
        if self.dtype != L.BF16:
            tokens, counts = self.decode(enc, plan)
            tok, cnt = tokens.cpu().numpy(), counts.cpu().numpy()
            self.check()
            return [token_list(tok[j, : cnt[j]]) for j in range(n)]
        flag = self.host_flag.numpy()
        flag[0], flag[1] = n, -1
        tokens, counts = self.decode(enc, plan)
        done = torch.cuda.Event()
        done.record()
        if self._side is None:
            self._side = torch.cuda.Stream(self.device)
        if self._tok_host is None or self._tok_host.numel() < n * cap + n:
            self._tok_host = torch.empty(int((n * cap + n) * 1.25), dtype=torch.int32).pin_memory()
        tok_h = self._tok_host[: n * cap].view(n, cap)
        cnt_h = self._tok_host[n * cap : n * cap + n]
        tk, cn = tok_h.numpy(), cnt_h.numpy()
        lists: list[list[int]] = [[] for _ in range(n)]
        hi = n  # lanes [hi, n) are converted
        while hi > 0:
            finished = done.query()
            bound = 0 if finished else max(0, min(int(flag[0]), hi))
            if bound < hi:
                with torch.cuda.stream(self._side):
                    tok_h[bound:hi].copy_(tokens[bound:hi], non_blocking=True)
                    cnt_h[bound:hi].copy_(counts[bound:hi], non_blocking=True)
                    copied = torch.cuda.Event()
                    copied.record(self._side)
                copied.synchronize()
                for j in range(bound, hi):
                    lists[j] = token_list(tk[j, : cn[j]])
                hi = bound
            elif not finished:
                time.sleep(2e-4)
        self.check()
        return lists
