"""Data parallelism over clips (tinybark_b200.dp): the longest-processing-time deal of the
whole-box workload (4096 clips of 2-30 s) and the one-process-per-GPU runner, on CPU."""

import numpy as np

from tinybark_b200 import dp, lengths, synthetic


def box_frames(count=4096, seed=4000):
    return [lengths.frames(int(round(d * 16000))) for d in synthetic.durations(count, seed)]


def test_deal_covers_every_clip_once_and_balances():
    frames = box_frames()
    order = sorted(range(len(frames)), key=lambda i: (-frames[i], i))
    for parts in (1, 2, 4, 8):
        shards = dp.deal(frames, parts)
        assert len(shards) == parts
        assert sorted(i for s in shards for i in s) == list(range(len(frames)))
        # Contiguous ranges of the clips by decreasing length, longest first.
        assert [i for s in shards for i in s] == order
        times = [dp.predicted_seconds([frames[i] for i in s]) for s in shards]
        lpt = [dp.predicted_seconds([frames[i] for i in s]) for s in dp.deal_lpt(frames, parts)]
        # No worse than dealing every shard the same mix of lengths.
        assert max(times) <= max(lpt) * (1 + 1e-9)
    assert dp.deal(frames, 4) == dp.deal(list(frames), 4)  # deterministic


def test_lpt_deal_balances_additive_costs():
    frames = box_frames()
    for parts in (2, 8):
        shards = dp.deal_lpt(frames, parts)
        assert sorted(i for s in shards for i in s) == list(range(len(frames)))
        costs = dp.shard_costs(frames, shards)
        assert max(costs) / (sum(costs) / parts) < 1.001


def test_predicted_seconds_counts_each_iteration_at_its_lanes():
    # Two clips: both lanes run to the shorter cap, then one lane alone.
    a, b = 3000, 800
    ca, cb = lengths.decode_cap(a), lengths.decode_cap(b)
    dec = cb * (dp.ITER_S + 2 * dp.ITER_S_PER_LANE) + (ca - cb) * (dp.ITER_S + dp.ITER_S_PER_LANE)
    enc = (dp.clip_encoder_flop(a) + dp.clip_encoder_flop(b)) * dp.ENC_S_PER_FLOP
    assert abs(dp.predicted_seconds([b, a]) - (enc + dec)) < 1e-12


def test_deal_edge_cases():
    assert dp.deal([], 3) == [[], [], []]
    assert dp.deal([500], 2) == [[0], []]
    shards = dp.deal([300] * 10, 4)
    assert sorted(i for s in shards for i in s) == list(range(10)) and len(shards) == 4
    assert dp.deal([100, 900, 500], 1) == [[1, 2, 0]]


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
