"""Long audio in pieces of bounded length: the chunked inference that tinybark leaves for
later (its backends take one clip in full context; the production use is dictation of up to
30 s, tinybark/tinygrad/__init__.py:38-39).

Full context over ten minutes means T = 7500 encoder frames: attention over all of them,
and one decoder lane that steps through the whole recording alone (about 75 000 greedy
iterations). Cut into pieces of at most 30 s, the recording becomes a batch of lanes that
the encoder and the decoder process side by side. Each piece is transcribed on its own, as
tinybark transcribes a clip, so words are not split if the cuts fall in pauses: each cut is
placed at the quietest short window near the end of its piece.
"""

from __future__ import annotations

import numpy as np

SAMPLE_RATE = 16000  # tinybark/audio.py:5-10
EOS = 3  # tinybark/tinygrad/model.py:63-75


def cut_points(samples: np.ndarray, max_seconds: float = 30.0, search_seconds: float = 2.0,
               window_seconds: float = 0.1) -> list[int]:
    """Sample offsets [0, c1, ..., len] splitting `samples` into pieces of at most
    `max_seconds`. Each cut lies in the last `search_seconds` of its piece, at the centre of
    the `window_seconds` window with the least energy there (the first such window on a
    tie)."""
    x = np.asarray(samples).reshape(-1)
    n = len(x)
    max_n = int(round(max_seconds * SAMPLE_RATE))
    search_n = min(int(round(search_seconds * SAMPLE_RATE)), max_n // 2)
    win = max(1, int(round(window_seconds * SAMPLE_RATE)))
    if max_n <= 0 or search_n < win:
        raise ValueError("max_seconds must leave room for a search window of window_seconds")
    energy = np.concatenate([[0.0], np.cumsum(np.square(x, dtype=np.float64))])
    cuts = [0]
    start = 0
    while n - start > max_n:
        lo, hi = start + max_n - search_n, start + max_n  # windows [s, s + win) inside [lo, hi)
        s = np.arange(lo, hi - win + 1)
        best = int(s[np.argmin(energy[s + win] - energy[s])])
        start = best + win // 2
        cuts.append(start)
    cuts.append(n)
    return cuts


def join(pieces: list[list[int]]) -> list[int]:
    """The pieces' token lists as one: an end-of-sequence token ends only its own piece, so
    it is kept only where it ends the last one."""
    out: list[int] = []
    for i, toks in enumerate(pieces):
        last = i == len(pieces) - 1
        out.extend(toks if last else [t for t in toks if t != EOS])
    return out
