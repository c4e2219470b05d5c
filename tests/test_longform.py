"""Cut points and token joining of the long-recording path (Bark.tokens_long): host logic,
no GPU."""

import numpy as np

from tinybark_b200 import longform

SR = longform.SAMPLE_RATE


def test_pieces_cover_the_recording_and_respect_the_limit():
    rng = np.random.default_rng(1)
    x = rng.standard_normal(SR * 200 + 123).astype(np.float32)
    cuts = longform.cut_points(x, max_seconds=30.0)
    assert cuts[0] == 0 and cuts[-1] == len(x)
    sizes = np.diff(cuts)
    assert (sizes > 0).all() and (sizes <= 30 * SR).all()
    assert (sizes[:-1] >= 28 * SR).all()  # every cut in the last 2 s of its piece


def test_cut_falls_in_the_quiet_window():
    rng = np.random.default_rng(2)
    x = rng.standard_normal(SR * 70).astype(np.float32)
    quiet = 29 * SR + 4000
    x[quiet : quiet + SR // 10] *= 1e-3
    cuts = longform.cut_points(x, max_seconds=30.0)
    assert cuts[1] == quiet + SR // 20  # the centre of the 100 ms window


def test_short_recording_is_one_piece():
    x = np.zeros(SR * 12, np.float32)
    assert longform.cut_points(x, max_seconds=30.0) == [0, len(x)]
    assert longform.cut_points(x[:0]) == [0, 0]


def test_join_keeps_eos_only_at_the_end():
    assert longform.join([[5, 3], [7, 8], [9, 3]]) == [5, 7, 8, 9, 3]
    assert longform.join([[3, 4]]) == [3, 4]
    assert longform.join([]) == []
