"""Seeded synthetic inputs for the Parakeet-TDT-0.6B-v3 / Underdog Bark architecture:
speech-like 16 kHz int16 clips and a random-init state dict in the checkpoint's own
(Bark / transformers) tensor names.

The real checkpoint and real speech are not used: the clips stand in for the
reference's recordings (tinybark/clips/*.pcm, 16 kHz s16le), and the state dict stands
in for what Bark's loader decodes (tinybark/weights.py:44-59), with the same names and
shapes so that the converted layout (tinybark/weights.py:62-89) follows from it.
"""

from __future__ import annotations

import numpy as np

SAMPLE_RATE = 16_000

# Architecture of Parakeet-TDT-0.6B-v3 (tinybark/mojo/bark/model.mojo:29-43).
HIDDEN = 1024
HEADS = 8
HEAD_DIM = HIDDEN // HEADS
FFN = 4096
KERNEL = 9
CHANNELS = 256
N_MELS = 128
VOCAB = 8193
BLANK = 8192
DURATIONS = (0, 1, 2, 3, 4)
DECODER_HIDDEN = 640
DECODER_LAYERS = 2
LAYERS = 24


def config(layers: int = LAYERS) -> dict:
    """The model config in the checkpoint's JSON shape: the keys the converter and the
    greedy loop read (tinybark/weights.py:66,79; tinybark/tinygrad/model.py:63-72)."""
    return {
        "encoder_config": {
            "num_hidden_layers": layers,
            "hidden_size": HIDDEN,
            "num_attention_heads": HEADS,
            "intermediate_size": FFN,
            "conv_kernel_size": KERNEL,
            "subsampling_conv_channels": CHANNELS,
            "subsampling_factor": 8,
            "num_mel_bins": N_MELS,
            "attention_bias": False,
            "convolution_bias": False,
            "scale_input": False,
        },
        "vocab_size": VOCAB,
        "blank_token_id": BLANK,
        "pad_token_id": 2,
        "durations": list(DURATIONS),
        "num_decoder_layers": DECODER_LAYERS,
        "decoder_hidden_size": DECODER_HIDDEN,
        "max_symbols_per_step": 10,
    }


# ---------------------------------------------------------------------------
# Audio


def clip(seconds: float, seed: int, segment: float | None = None) -> np.ndarray:
    """A speech-like int16 clip: a harmonic series (f0 ~ U(100, 250) Hz, 10 partials at
    1/k amplitude) under a 4 Hz syllabic amplitude envelope, white noise 30 dB below
    the signal's RMS, peak normalised to half of full scale. With `segment`, f0 is drawn
    again every `segment` seconds (phase kept continuous)."""
    rng = np.random.default_rng(seed)
    n = int(round(seconds * SAMPLE_RATE))
    if n == 0:
        return np.zeros(0, np.int16)
    if segment:
        per = int(round(segment * SAMPLE_RATE))
        f0 = np.repeat(rng.uniform(100.0, 250.0, -(-n // per)), per)[:n]
    else:
        f0 = np.full(n, rng.uniform(100.0, 250.0))
    phase = np.cumsum(f0)
    phase *= 2.0 * np.pi / SAMPLE_RATE
    offsets = rng.uniform(0.0, 2.0 * np.pi, 10)
    # sin(k phase + o_k) = sin(k phase) cos(o_k) + cos(k phase) sin(o_k), with sin and cos
    # of k phase from those of (k-1) phase by the angle-addition formulas: two
    # transcendental evaluations per sample instead of ten, in place.
    s1, c1 = np.sin(phase), np.cos(phase)
    sk, ck, t1, t2 = s1.copy(), c1.copy(), np.empty(n), np.empty(n)
    signal = sk * np.cos(offsets[0])
    signal += ck * np.sin(offsets[0])
    for k in range(2, 11):
        np.multiply(sk, c1, out=t1)
        t1 += ck * s1
        np.multiply(ck, c1, out=t2)
        t2 -= sk * s1
        sk, t1 = t1, sk
        ck, t2 = t2, ck
        signal += sk * (np.cos(offsets[k - 1]) / k)
        signal += ck * (np.sin(offsets[k - 1]) / k)
    env = np.arange(n, dtype=np.float64)
    env *= 2.0 * np.pi * 4.0 / SAMPLE_RATE
    env += rng.uniform(0.0, 2.0 * np.pi)
    np.cos(env, out=env)
    signal *= 0.5 * (1.0 - env)
    rms = np.sqrt(np.mean(signal**2)) or 1.0
    signal += rng.standard_normal(n) * (rms * 10.0 ** (-30.0 / 20.0))
    signal *= 0.5 * 32767.0 / max(np.abs(signal).max(), 1e-12)
    return np.round(signal).astype(np.int16)


def to_float(pcm: np.ndarray) -> np.ndarray:
    """int16 samples to float32 in [-1, 1), as the backends read s16le PCM
    (tinybark/pytorch/__init__.py:50)."""
    return pcm.astype(np.float32) / 32768


def durations(count: int, seed: int, low: float = 2.0, high: float = 30.0) -> np.ndarray:
    """Clip durations in seconds, uniform in [low, high), rounded to whole samples."""
    rng = np.random.default_rng(seed)
    return np.round(rng.uniform(low, high, count) * SAMPLE_RATE) / SAMPLE_RATE


# ---------------------------------------------------------------------------
# Weights


def _xavier(rng: np.random.Generator, shape: tuple[int, ...]) -> np.ndarray:
    """Xavier-uniform with torch's fan convention: fan_in = shape[1] * receptive field,
    fan_out = shape[0] * receptive field."""
    receptive = int(np.prod(shape[2:])) if len(shape) > 2 else 1
    fan_in, fan_out = shape[1] * receptive, shape[0] * receptive
    bound = np.float32(np.sqrt(6.0 / (fan_in + fan_out)))
    return (rng.random(shape, dtype=np.float32) * 2 - 1) * bound


def state_dict(seed: int = 0, layers: int = LAYERS) -> dict[str, np.ndarray]:
    """Random-init weights in the checkpoint's names: Xavier-uniform linears, convs,
    LSTM and embedding; LayerNorm gamma 1, beta 0; BatchNorm gamma 1, beta 0, running
    mean 0, variance 1; biases 0; the positional biases bias_u / bias_v ~ N(0, 0.02)."""
    rng = np.random.default_rng(seed)
    sd: dict[str, np.ndarray] = {}
    zeros = lambda *s: np.zeros(s, np.float32)
    ones = lambda *s: np.ones(s, np.float32)

    p = "encoder.subsampling."
    sd[p + "layers.0.weight"] = _xavier(rng, (CHANNELS, 1, 3, 3))
    sd[p + "layers.0.bias"] = zeros(CHANNELS)
    for dw, pw in ((2, 3), (5, 6)):
        sd[p + f"layers.{dw}.weight"] = _xavier(rng, (CHANNELS, 1, 3, 3))
        sd[p + f"layers.{dw}.bias"] = zeros(CHANNELS)
        sd[p + f"layers.{pw}.weight"] = _xavier(rng, (CHANNELS, CHANNELS, 1, 1))
        sd[p + f"layers.{pw}.bias"] = zeros(CHANNELS)
    sd[p + "linear.weight"] = _xavier(rng, (HIDDEN, CHANNELS * (N_MELS // 8)))
    sd[p + "linear.bias"] = zeros(HIDDEN)

    for i in range(layers):
        p = f"encoder.layers.{i}."
        for ff in ("feed_forward1", "feed_forward2"):
            sd[p + ff + ".linear1.weight"] = _xavier(rng, (FFN, HIDDEN))
            sd[p + ff + ".linear2.weight"] = _xavier(rng, (HIDDEN, FFN))
        a = p + "self_attn."
        for n in ("q", "k", "v", "o"):
            sd[a + f"{n}_proj.weight"] = _xavier(rng, (HIDDEN, HIDDEN))
        sd[a + "relative_k_proj.weight"] = _xavier(rng, (HIDDEN, HIDDEN))
        sd[a + "bias_u"] = (rng.standard_normal((HEADS, HEAD_DIM)) * 0.02).astype(np.float32)
        sd[a + "bias_v"] = (rng.standard_normal((HEADS, HEAD_DIM)) * 0.02).astype(np.float32)
        c = p + "conv."
        sd[c + "pointwise_conv1.weight"] = _xavier(rng, (2 * HIDDEN, HIDDEN, 1))
        sd[c + "depthwise_conv.weight"] = _xavier(rng, (HIDDEN, 1, KERNEL))
        sd[c + "norm.weight"] = ones(HIDDEN)
        sd[c + "norm.bias"] = zeros(HIDDEN)
        sd[c + "norm.running_mean"] = zeros(HIDDEN)
        sd[c + "norm.running_var"] = ones(HIDDEN)
        sd[c + "pointwise_conv2.weight"] = _xavier(rng, (HIDDEN, HIDDEN, 1))
        for n in ("norm_feed_forward1", "norm_self_att", "norm_conv", "norm_feed_forward2", "norm_out"):
            sd[p + n + ".weight"] = ones(HIDDEN)
            sd[p + n + ".bias"] = zeros(HIDDEN)

    sd["encoder_projector.weight"] = _xavier(rng, (DECODER_HIDDEN, HIDDEN))
    sd["encoder_projector.bias"] = zeros(DECODER_HIDDEN)
    sd["decoder.embedding.weight"] = _xavier(rng, (VOCAB, DECODER_HIDDEN))
    for l in range(DECODER_LAYERS):
        sd[f"decoder.lstm.weight_ih_l{l}"] = _xavier(rng, (4 * DECODER_HIDDEN, DECODER_HIDDEN))
        sd[f"decoder.lstm.weight_hh_l{l}"] = _xavier(rng, (4 * DECODER_HIDDEN, DECODER_HIDDEN))
        sd[f"decoder.lstm.bias_ih_l{l}"] = zeros(4 * DECODER_HIDDEN)
        sd[f"decoder.lstm.bias_hh_l{l}"] = zeros(4 * DECODER_HIDDEN)
    sd["decoder.decoder_projector.weight"] = _xavier(rng, (DECODER_HIDDEN, DECODER_HIDDEN))
    sd["decoder.decoder_projector.bias"] = zeros(DECODER_HIDDEN)
    sd["joint.head.weight"] = _xavier(rng, (VOCAB + len(DURATIONS), DECODER_HIDDEN))
    sd["joint.head.bias"] = zeros(VOCAB + len(DURATIONS))
    return sd


def tokenizer(path, vocab: int = 8193, seed: int = 0) -> str:
    """A tokenizer.json of `vocab` ids in the Parakeet tokenizer's form, since no real
    vocabulary is available offline: the 256 byte-fallback pieces <0x00>..<0xFF> at ids
    3..258, special tokens at ids 0-2 and the last id, and seeded pieces of 1-4 characters
    from a set with "▁", multi-byte and combining characters elsewhere. Returns the path."""
    import json
    import random
    from pathlib import Path

    rng = random.Random(seed)
    chars = ["a", "e", "n", "t", "é", "ß", "中", "😀", "▁", "▁", "x", "\u0301", "\ufffd", " "]
    special = {0: "<unk>", 1: "<pad>", 2: "<|endoftext|>", vocab - 1: "<blank>"}
    pieces, used = {}, set()
    for i in range(vocab):
        if 3 <= i < 259:
            p = f"<0x{i - 3:02X}>"
        else:
            p = "".join(rng.choice(chars) for _ in range(rng.randint(1, 4)))
            while p in used:
                p += rng.choice(chars)
        used.add(p)
        if i not in special:
            pieces[p] = i
    spec = {
        "model": {"vocab": pieces},
        "added_tokens": [{"id": i, "content": c, "special": True} for i, c in special.items()],
    }
    Path(path).write_text(json.dumps(spec))
    return str(path)
