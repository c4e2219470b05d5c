"""Oracle (test infrastructure only): log-mel features, a numpy restatement of
tinybark/audio.py:42-55 with the slaney mel filterbank of tinybark/audio.py:13-33 and
the centred 400-tap Hann window of tinybark/audio.py:37-39."""

import numpy as np

SAMPLE_RATE = 16_000
N_FFT, HOP, WIN = 512, 160, 400
N_MELS = 128
PREEMPHASIS = 0.97
LOG_GUARD = 2.0**-24
EPSILON = 1e-5


def mel_filters() -> np.ndarray:
    """Slaney-normalised triangular filters on the slaney mel scale, (N_MELS, N_FFT//2+1),
    built in float64 and stored as float32 (tinybark/audio.py:13-33)."""

    def to_mel(f):
        f = np.asarray(f, np.float64)
        logstep = np.log(6.4) / 27.0
        return np.where(f >= 1000.0, 15.0 + np.log(np.maximum(f, 1e-10) / 1000.0) / logstep, 3.0 * f / 200.0)

    def to_hz(m):
        logstep = np.log(6.4) / 27.0
        return np.where(m >= 15.0, 1000.0 * np.exp(logstep * (m - 15.0)), 200.0 * m / 3.0)

    bins = np.linspace(0, SAMPLE_RATE / 2, N_FFT // 2 + 1)
    edges = to_hz(np.linspace(to_mel(0.0), to_mel(SAMPLE_RATE / 2), N_MELS + 2))
    diff = edges[:, None] - bins[None, :]
    width = np.diff(edges)
    rising = -diff[:-2] / width[:-1, None]
    falling = diff[2:] / width[1:, None]
    w = np.maximum(0, np.minimum(rising, falling))
    w *= (2.0 / (edges[2:] - edges[:-2]))[:, None]
    return w.astype(np.float32)


def window() -> np.ndarray:
    """np.hanning(400) centred in a 512-sample frame (tinybark/audio.py:37-39)."""
    w = np.zeros(N_FFT, np.float32)
    w[(N_FFT - WIN) // 2 : (N_FFT + WIN) // 2] = np.hanning(WIN)
    return w


MEL = mel_filters()
WINDOW = window()


def features(samples: np.ndarray) -> np.ndarray:
    """(samples // 160, 128) float32 normalised log-mel features (tinybark/audio.py:42-55)."""
    x = np.asarray(samples, np.float32)
    x = np.concatenate([x[:1], x[1:] - np.float32(PREEMPHASIS) * x[:-1]])
    x = np.pad(x, N_FFT // 2)
    count = len(samples) // HOP
    idx = np.arange(N_FFT)[None, :] + HOP * np.arange(count)[:, None]
    spec = np.fft.rfft(x[idx] * WINDOW, axis=-1)
    power = (spec.real**2 + spec.imag**2).astype(np.float32)
    mel = np.log(power @ MEL.T + np.float32(LOG_GUARD))
    mean = mel.mean(0)
    std = np.sqrt(((mel - mean) ** 2).sum(0) / (count - 1))
    return ((mel - mean) / (std + np.float32(EPSILON))).astype(np.float32)
