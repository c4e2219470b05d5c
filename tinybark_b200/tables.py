"""Constant tables of the log-mel front-end kernel: the 400-tap Hann window centred in
the 512-sample frame (tinybark/audio.py:37-39) and the 128 slaney mel filters of
librosa.filters.mel(sr=16000, n_fft=512, n_mels=128, norm="slaney")
(tinybark/audio.py:13-33), stored sparsely: each filter's first FFT bin and its
non-zero weights. The filters are built in float64 and stored as float32, as the
reference stores them."""

from __future__ import annotations

import numpy as np

SAMPLE_RATE, N_FFT, WIN, N_MELS = 16_000, 512, 400, 128


def _hz_to_mel(f):
    f = np.asarray(f, np.float64)
    step = np.log(6.4) / 27.0  # slaney: linear below 1 kHz, log above
    return np.where(f >= 1000.0, 15.0 + np.log(np.maximum(f, 1e-10) / 1000.0) / step, 3.0 * f / 200.0)


def _mel_to_hz(m):
    step = np.log(6.4) / 27.0
    return np.where(m >= 15.0, 1000.0 * np.exp(step * (m - 15.0)), 200.0 * m / 3.0)


def mel_filters() -> np.ndarray:
    """(128, 257) float32 triangular filters, each scaled to unit area (slaney norm)."""
    bins = np.linspace(0, SAMPLE_RATE / 2, N_FFT // 2 + 1)
    edges = _mel_to_hz(np.linspace(_hz_to_mel(0.0), _hz_to_mel(SAMPLE_RATE / 2), N_MELS + 2))
    gap = edges[:, None] - bins[None, :]
    width = np.diff(edges)
    up = -gap[:-2] / width[:-1, None]
    down = gap[2:] / width[1:, None]
    filt = np.maximum(0, np.minimum(up, down)) * (2.0 / (edges[2:] - edges[:-2]))[:, None]
    return filt.astype(np.float32)


def window() -> np.ndarray:
    w = np.zeros(N_FFT, np.float32)
    w[(N_FFT - WIN) // 2 : (N_FFT + WIN) // 2] = np.hanning(WIN)
    return w


def sparse_mel() -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """(weights, first bin per filter, offsets [129]) of the non-zero span of each filter."""
    filt = mel_filters()
    weights, start, off = [], [], [0]
    for row in filt:
        nz = np.nonzero(row)[0]
        lo, hi = (int(nz[0]), int(nz[-1]) + 1) if len(nz) else (0, 0)
        weights.append(row[lo:hi])
        start.append(lo)
        off.append(off[-1] + hi - lo)
    return np.concatenate(weights).astype(np.float32), np.array(start, np.int32), np.array(off, np.int32)
