"""Data parallelism over clips (tinybark_b200.dp): the longest-processing-time deal of the
whole-box workload (4096 clips of 2-30 s) and the one-process-per-GPU runner, on CPU."""

import numpy as np

from tinybark_b200 import dp, lengths, synthetic


def box_frames(count=4096, seed=4000):
    return [lengths.frames(int(round(d * 16000))) for d in synthetic.durations(count, seed)]


def test_deal_covers_every_clip_once_and_balances():
    frames = box_frames()
    for parts in (1, 2, 4, 8):
        shards = dp.deal(frames, parts)
        assert sorted(i for s in shards for i in s) == list(range(len(frames)))
        costs = dp.shard_costs(frames, shards)
        assert max(costs) / (sum(costs) / parts) < 1.001
        # Every shard starts with one of the `parts` costliest clips (the longest, up to
        # lengths of equal cost), so the greedy loops (as long as each shard's longest
        # clip) end together.
        costliest = sorted(range(len(frames)), key=lambda i: (-dp.clip_cost(frames[i]), i))[:parts]
        assert sorted(s[0] for s in shards) == sorted(costliest)
        caps = [max(lengths.decode_cap(frames[i]) for i in s) for s in shards]
        assert max(caps) - min(caps) <= 20
    assert dp.deal(frames, 4) == dp.deal(list(frames), 4)  # deterministic


def test_deal_edge_cases():
    assert dp.deal([], 3) == [[], [], []]
    assert dp.deal([500], 2) == [[0], []]
    equal = dp.deal([300] * 10, 4)
    assert [len(s) for s in equal] == [3, 3, 2, 2]


def _fake_run(clips):
    # Stands in for a GPU's transcription: a clip's "tokens" are its length and first sample.
    return [[len(c), int(c[0]) if len(c) else -1] for c in clips]


def test_multi_gpu_runner_deals_and_gathers_in_order():
    rng = np.random.default_rng(2)
    clips = [rng.integers(-3000, 3000, int(n), dtype=np.int16) for n in rng.integers(400, 40000, 37)]
    clips[5] = np.zeros(0, np.int16)
    with dp.MultiGPU([0, 1, 2], run=_fake_run) as m:
        got = m.tokens_batch(clips)
        assert got == _fake_run(clips)
        flt = [c.astype(np.float32) / 32768 for c in clips[:4]]
        assert m.tokens_batch(flt) == [[len(c), 0 if len(c) and abs(c[0]) < 1 else -1] for c in flt]
