"""The multi-rank host logic of bench.py on CPU: two gloo ranks, as torchrun launches the
GPU ranks. The whole-box set is dealt over the ranks (every clip on exactly one rank, the
same clip audio whichever rank draws it; no collective on the data path), the step time
is the max over ranks and the audio total the sum."""

import os
import socket
import sys
from pathlib import Path

import numpy as np
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, out) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    sys.path.insert(0, str(ROOT))
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    import bench
    from tinybark_b200 import dp

    dist.init_process_group("gloo", timeout=timedelta(seconds=60))
    try:
        r, w, local = bench.rank_info()
        clips, durs = bench.shard(r, w, 24)
        step_ms = 100.0 + 10.0 * r  # rank 1 is the slower one
        ids = torch.zeros(24, dtype=torch.int64)
        mine = dp.deal(bench.box_frames(24), w)[r]
        ids[mine] = 1
        dist.all_reduce(ids)  # how many ranks hold each clip
        out.put({
            "rank": r, "world": w, "local": local,
            "durs": [float(d) for d in durs],
            "lens": [len(c) for c in clips],
            "holders": ids.tolist(),
            "max": bench.reduce_over_ranks(step_ms, "max", torch.device("cpu")),
            "sum": bench.reduce_over_ranks(float(np.sum(durs)), "sum", torch.device("cpu")),
        })
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_shard_and_reduce():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = sorted((q.get(timeout=180) for _ in procs), key=lambda d: d["rank"])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [g["rank"] for g in got] == [0, 1] and all(g["world"] == 2 for g in got)
    # Every clip of the set on exactly one rank; shards longest first, 2-30 s of 16 kHz
    # audio, balanced in predicted time to within one clip (the longest clips on rank 0).
    from tinybark_b200 import dp, lengths

    assert all(h == 1 for h in got[0]["holders"]) and got[0]["holders"] == got[1]["holders"]
    frames = [[lengths.frames(n) for n in g["lens"]] for g in got]
    times = [dp.predicted_seconds(f) for f in frames]
    assert abs(times[0] - times[1]) <= max(dp.predicted_seconds([x]) for f in frames for x in f)
    assert min(frames[0]) >= max(frames[1])
    for g in got:
        assert g["durs"] == sorted(g["durs"], reverse=True)
        assert all(2.0 <= d < 30.0 for d in g["durs"])
        assert all(abs(n - 16000 * d) <= 1 for n, d in zip(g["lens"], g["durs"]))
    # Max over ranks for the time, sum for the audio, the same on every rank.
    assert all(g["max"] == 110.0 for g in got)
    total = sum(sum(g["durs"]) for g in got)
    assert all(abs(g["sum"] - total) < 1e-6 for g in got)


def test_shard_is_deterministic_and_independent_of_the_deal():
    """A clip's audio depends only on its index in the set: rank 0 of 1 holds every
    clip, and the clips rank 1 of 2 draws are the same arrays."""
    sys.path.insert(0, str(ROOT))
    import bench
    from tinybark_b200 import dp

    a, da = bench.shard(0, 1, 12)
    b, db = bench.shard(0, 1, 12)
    assert list(da) == list(db) and len(a) == 12
    assert all(np.array_equal(x, y) for x, y in zip(a, b))
    assert all(x.dtype == np.int16 for x in a)
    c, dc = bench.shard(1, 2, 12)
    whole = {(len(x), x[:64].tobytes()) for x in a}
    assert all((len(x), x[:64].tobytes()) in whole for x in c)
    assert len(c) == len(dp.deal(bench.box_frames(12), 2)[1])
