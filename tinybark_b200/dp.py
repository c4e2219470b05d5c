"""Data parallelism over clips: one process per GPU, each transcribing its own shard of
the clips end to end (front-end, encoder, TDT decode), with no collective on the data
path. Clips are independent units: nothing in the greedy loop
(tinybark/tinygrad/model.py:196-233) reads another clip.

`deal` splits a clip list into shards of equal predicted time: the clips sorted by length
(tinybark sorts clips into 256-frame length buckets, tinybark/tinygrad/model.py:15-20;
this build packs clips without padding, so the deal works on exact lengths) and cut into
contiguous ranges, the cuts placed so that the largest predicted shard time is as small
as it can be. A shard's time is not a sum over its clips: the encoder's is (FLOPs), but
the greedy loop runs all of a shard's lanes together for as many iterations as its
longest clip needs, each iteration costing a fixed latency plus a little per lane. So a
shard of only short clips ends its loop early and can take more clips, and contiguous
length ranges beat dealing every shard the same mix of lengths (`deal_lpt`, longest
processing time first on additive costs), which gives every shard a full-length loop.

`MultiGPU` runs the shards: one spawned process per GPU (pinned with
CUDA_VISIBLE_DEVICES, as tinybark's benchmark isolates each backend in a process of its
own, bench/__main__.py:45-57), the samples passed through one shared-memory block and the
token lists gathered over pipes.
"""

from __future__ import annotations

import heapq
import multiprocessing as mp
import os
from multiprocessing import shared_memory
from typing import Callable, Sequence

import numpy as np

from . import lengths

# Predicted cost of a clip: encoder work per encoder frame and per squared length
# (linears and subsampling 1.26 GFLOP per frame, attention 6 T^2 1024 FLOP per layer over
# 24 layers), and decoder work per greedy-loop iteration (24.6 MFLOP per lane).
ENC_FLOP_PER_FRAME = 1.26e9
ATTN_FLOP_PER_FRAME2 = 6 * 1024 * 24
DEC_FLOP_PER_ITER = 24.6e6


# Predicted seconds on one B200, bf16, measured: the front-end and encoder at 0.88 PFLOP/s
# of clip_encoder_flop (154 ms for a 512-clip batch of 2-30 s clips), and one iteration of
# the persistent decoder at 25.1 us plus 27.9 ns per running lane (a least-squares fit to
# the whole greedy loop of 512, 1024, 2048 and 4096 lanes: 118, 157, 208, 319 ms).
ENC_S_PER_FLOP = 1.0 / 0.88e15
ITER_S = 25.1e-6
ITER_S_PER_LANE = 27.9e-9


def clip_encoder_flop(frames: int) -> float:
    t = lengths.subsampled(frames, 3)
    return ENC_FLOP_PER_FRAME * t + ATTN_FLOP_PER_FRAME2 * t * t


def predicted_seconds(frames: Sequence[int]) -> float:
    """Predicted time of one GPU transcribing these clips as one batch: encoder work, then
    the greedy loop, iteration by iteration at the latency of the lanes still running."""
    f = np.asarray(frames, np.int64)
    if f.size == 0:
        return 0.0
    t = f
    for _ in range(3):
        t = (t - 1) // 2 + 1  # encoder frames (lengths.subsampled)
    enc = float(np.sum(ENC_FLOP_PER_FRAME * t + ATTN_FLOP_PER_FRAME2 * t.astype(np.float64) ** 2)) * ENC_S_PER_FLOP
    u = f + 1
    for _ in range(3):
        u = (u - 1) // 2 + 1
    caps = np.sort(lengths.MAX_SYMBOLS * u - 1)[::-1]  # lengths.decode_cap, longest first
    # The k longest lanes run for iterations caps[k] .. caps[k - 1].
    lanes = np.arange(1, len(caps) + 1)
    steps = caps - np.append(caps[1:], 0)
    return enc + float(np.sum(steps * (ITER_S + ITER_S_PER_LANE * lanes)))


# The token ids (8192 pieces and the blank) as Python ints, gathered by token rows: a list
# then shares these objects instead of creating an int per token (half the conversion
# time). Rows holding anything else convert as they are.
_TOKEN_INTS = np.array(range(8193), dtype=object)


def _id_list(row: np.ndarray) -> list[int]:
    if row.size and 0 <= int(row.min()) and int(row.max()) < len(_TOKEN_INTS):
        return _TOKEN_INTS[row].tolist()
    return row.tolist()


def clip_cost(frames: int) -> float:
    """Predicted FLOPs of one clip of `frames` feature frames through the whole path."""
    t = lengths.subsampled(frames, 3)
    return ENC_FLOP_PER_FRAME * t + ATTN_FLOP_PER_FRAME2 * t * t + DEC_FLOP_PER_ITER * lengths.decode_cap(frames)


def deal(frames: Sequence[int], parts: int) -> list[list[int]]:
    """Indices of the clips (feature-frame counts `frames`) in each of `parts` shards:
    contiguous ranges of the clips in decreasing length (ties by index), the first shard
    the longest clips, cut so that the largest `predicted_seconds` of a shard is the
    smallest the cuts allow (a bisection on that time; each shard takes as many clips as
    fit under it). Deterministic, so every rank computes the same deal."""
    if parts < 1:
        raise ValueError("parts must be at least 1")
    order = sorted(range(len(frames)), key=lambda i: (-int(frames[i]), i))
    f = [int(frames[i]) for i in order]
    if not f:
        return [[] for _ in range(parts)]

    def cuts(limit: float) -> list[int] | None:
        """Shard ends filling each shard up to `limit`, or None if `parts` do not suffice."""
        ends, start = [], 0
        for _ in range(parts):
            if start == len(f):
                break
            lo, hi = start + 1, len(f)  # the largest end with the shard's time <= limit
            if predicted_seconds(f[start:lo]) > limit:
                return None
            while lo < hi:
                mid = (lo + hi + 1) // 2
                if predicted_seconds(f[start:mid]) <= limit:
                    lo = mid
                else:
                    hi = mid - 1
            ends.append(lo)
            start = lo
        return ends if start == len(f) else None

    lo, hi = max(predicted_seconds([x]) for x in f), predicted_seconds(f)
    for _ in range(40):
        mid = (lo + hi) / 2
        if cuts(mid) is None:
            lo = mid
        else:
            hi = mid
    ends = cuts(hi)
    shards, start = [], 0
    for e in ends:
        shards.append(order[start:e])
        start = e
    return shards + [[] for _ in range(parts - len(shards))]


def deal_lpt(frames: Sequence[int], parts: int) -> list[list[int]]:
    """Longest processing time first on additive costs (clip_cost): clips in decreasing
    cost (ties by index), each to the shard of least cost so far (ties to the lowest
    shard). Every shard gets the same mix of lengths; kept to compare with `deal`."""
    if parts < 1:
        raise ValueError("parts must be at least 1")
    order = sorted(range(len(frames)), key=lambda i: (-clip_cost(int(frames[i])), i))
    heap = [(0.0, p) for p in range(parts)]
    shards: list[list[int]] = [[] for _ in range(parts)]
    for i in order:
        cost, p = heapq.heappop(heap)
        shards[p].append(i)
        heapq.heappush(heap, (cost + clip_cost(int(frames[i])), p))
    return shards


def shard_costs(frames: Sequence[int], shards: list[list[int]]) -> list[float]:
    return [sum(clip_cost(int(frames[i])) for i in s) for s in shards]


# ---------------------------------------------------------------------------- processes


def _worker(gpu: int, weights, dtype: str, conn, run: Callable | None) -> None:
    """One GPU's process: loads the model once, then transcribes each shard it is sent
    (shared-memory name, dtype, per-clip offsets) and sends back (token ids, counts)."""
    os.environ["CUDA_VISIBLE_DEVICES"] = str(gpu)
    try:
        if run is None:
            from . import load

            bark = load("gpu", dtype=dtype, weights=weights() if callable(weights) else weights)
            run = bark.tokens_batch
        conn.send(("ready", None))
    except Exception as e:  # reported to the caller, which raises
        conn.send(("error", repr(e)))
        return
    while True:
        msg = conn.recv()
        if msg is None:
            break
        name, dt, offs = msg
        shm = shared_memory.SharedMemory(name=name)
        try:
            data = np.ndarray((int(offs[-1]),), dtype=dt, buffer=shm.buf)
            clips = [data[offs[i] : offs[i + 1]] for i in range(len(offs) - 1)]
            lists = run(clips)
            del clips, data
            counts = np.array([len(x) for x in lists], np.int64)
            flat = np.fromiter((t for x in lists for t in x), np.int32, int(counts.sum()))
            conn.send(("ok", (flat, counts)))
        except Exception as e:
            conn.send(("error", repr(e)))
        finally:
            shm.close()


class MultiGPU:
    """Transcription on several GPUs of one host, one process per GPU.

        with MultiGPU([0, 1, 2, 3], weights=path) as m:
            ids = m.tokens_batch(clips)   # clips: 16 kHz mono float32 or int16 arrays

    `weights` is what tinybark_b200.load takes (a cache-file path, or (tensors, config)),
    or a picklable zero-argument callable returning it (each process calls it once).
    `run` replaces each process's transcription (clips -> token lists), for tests
    without a GPU."""

    def __init__(self, gpus: Sequence[int], weights=None, dtype: str = "bf16", run: Callable | None = None):
        self.gpus = list(gpus)
        if not self.gpus:
            raise ValueError("no GPUs")
        ctx = mp.get_context("spawn")
        self._conns, self._procs = [], []
        for g in self.gpus:
            parent, child = ctx.Pipe()
            p = ctx.Process(target=_worker, args=(g, weights, dtype, child, run), daemon=True)
            p.start()
            self._conns.append(parent)
            self._procs.append(p)
        for g, c in zip(self.gpus, self._conns):
            status, info = c.recv()
            if status != "ready":
                self.close()
                raise RuntimeError(f"GPU {g}: {info}")

    def tokens_batch(self, clips: Sequence[np.ndarray]) -> list[list[int]]:
        """Token ids of every clip, as Bark.tokens_batch returns them, the clips dealt to
        the GPUs by `deal`."""
        clips = [np.asarray(c).reshape(-1) for c in clips]
        pcm = len(clips) > 0 and all(c.dtype == np.int16 for c in clips)
        dt = np.dtype(np.int16 if pcm else np.float32)
        frames = [lengths.frames(len(c)) for c in clips]
        shards = deal(frames, len(self.gpus))
        out: list[list[int]] = [[] for _ in clips]
        total = sum(len(c) for c in clips)
        shm = shared_memory.SharedMemory(create=True, size=max(total * dt.itemsize, 1))
        try:
            data = np.ndarray((total,), dtype=dt, buffer=shm.buf)
            pos = 0
            sent = []
            for conn, shard in zip(self._conns, shards):
                offs = [pos]
                for i in shard:
                    data[pos : pos + len(clips[i])] = clips[i]
                    pos += len(clips[i])
                    offs.append(pos)
                # Offsets into the whole block: each process maps it and views its clips.
                conn.send((shm.name, dt.str, np.asarray(offs, np.int64)))
                sent.append(shard)
            errors = []
            for g, conn, shard in zip(self.gpus, self._conns, sent):
                status, info = conn.recv()
                if status != "ok":
                    errors.append(f"GPU {g}: {info}")
                    continue
                flat, counts = info
                ends = np.cumsum(counts)
                for j, i in enumerate(shard):
                    out[i] = _id_list(flat[ends[j] - counts[j] : ends[j]])
            del data
            if errors:
                raise RuntimeError("; ".join(errors))
        finally:
            shm.close()
            shm.unlink()
        return out

    def close(self) -> None:
        for c in self._conns:
            try:
                c.send(None)
            except (OSError, BrokenPipeError):
                pass
        for p in self._procs:
            p.join(timeout=30)
            if p.is_alive():
                p.terminate()
        self._conns, self._procs = [], []

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
