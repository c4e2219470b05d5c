"""Data parallelism over clips: one process per GPU, each transcribing its own shard of
the clips end to end (front-end, encoder, TDT decode), with no collective on the data
path. Clips are independent units: nothing in the greedy loop
(tinybark/tinygrad/model.py:196-233) reads another clip.

`deal` splits a clip list into balanced shards: clips by predicted cost, longest first,
each to the shard with the least predicted cost so far (longest processing time first;
tinybark sorts clips into 256-frame length buckets, tinybark/tinygrad/model.py:15-20,
and this build packs clips without padding, so the deal works on exact lengths). Taking
the longest clips first also gives every shard one of the longest clips, so the shards'
greedy loops, whose length is set by their longest clip, end together.

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


def clip_cost(frames: int) -> float:
    """Predicted FLOPs of one clip of `frames` feature frames through the whole path."""
    t = lengths.subsampled(frames, 3)
    return ENC_FLOP_PER_FRAME * t + ATTN_FLOP_PER_FRAME2 * t * t + DEC_FLOP_PER_ITER * lengths.decode_cap(frames)


def deal(frames: Sequence[int], parts: int) -> list[list[int]]:
    """Indices of the clips (feature-frame counts `frames`) in each of `parts` shards,
    longest processing time first: clips in decreasing predicted cost (ties by index),
    each to the shard of least cost so far (ties to the lowest shard). Deterministic, so
    every rank computes the same deal; each shard lists its clips in dealing order."""
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
                    out[i] = flat[ends[j] - counts[j] : ends[j]].tolist()
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
