"""Integer length arithmetic of the path: feature frames per clip, the length after
the three stride-2 subsampling convolutions, padding buckets and the greedy loop's
iteration cap.

Reference: tinybark/tinygrad/model.py:16-27 (BUCKET, bucket, subsampled),
tinybark/audio.py:52 (frames = samples // HOP), tinybark/tinygrad/model.py:222 (cap).
"""

HOP = 160
BUCKET = 256
MAX_SYMBOLS = 10


def frames(samples: int) -> int:
    """Feature frames of a clip of `samples` samples (tinybark/audio.py:52)."""
    return samples // HOP


def subsampled(frames: int, convs: int = 3) -> int:
    """Length after `convs` convolutions with kernel 3, stride 2 and padding 1
    (tinybark/tinygrad/model.py:23-27)."""
    for _ in range(convs):
        frames = (frames - 1) // 2 + 1
    return frames


def bucket(frames: int) -> int:
    """Frames padded up to a multiple of BUCKET (tinybark/tinygrad/model.py:19-20)."""
    return -(-frames // BUCKET) * BUCKET


def decode_cap(frames: int) -> int:
    """Iterations of the greedy loop for a clip of `frames` feature frames: the cap is
    global to the clip, not per encoder frame (tinybark/tinygrad/model.py:222)."""
    return MAX_SYMBOLS * subsampled(frames + 1, 3) - 1
