"""Parakeet-TDT-0.6B-v3 / Underdog Bark speech-to-text on NVIDIA B200: the `cuda`
backend of tinybark. Python host code calls hand-written sm_100a kernels through
libtbcuda's C ABI; torch only allocates device memory.

    bark = tinybark_b200.load()            # the converted weights tinybark caches
    text = bark.transcribe(samples)        # 16 kHz mono float32 NumPy array
    ids = bark.tokens_batch([a, b, c])     # many clips in one pass

Same API as tinybark's backends (tinybark/backends.py:21-26; tinybark/tinygrad/__init__.py:21-35):
`device`, `tokens`, `transcribe`, `transcribe_pcm`, plus `tokens_batch`, `transcribe_batch`
(transcripts joined into bytes on the GPU), `tokens_long` /
`transcribe_long` (long recordings in pieces of at most 30 s) and `close`.
"""

from __future__ import annotations

import json
import os
from pathlib import Path

import numpy as np

__all__ = ["Bark", "load"]

# Where tinybark caches the converted weights (tinybark/weights.py:17-21,106-120).
CACHE = Path(os.environ.get("XDG_CACHE_HOME", Path.home() / ".cache")) / "tinybark"
CONVERTED = "bark-6d34ed8639b2-v2"
TOKENIZER_REPO = "nvidia/parakeet-tdt-0.6b-v3"


def converted(path: str | Path | None = None) -> tuple[Path, dict]:
    """tinybark's converted fp16 cache file and its config (tinybark/weights.py:106-120),
    as tinybark's weights.converted() returns them."""
    base = Path(path) if path else CACHE / CONVERTED
    tensors_path, config_path = base.with_suffix(".safetensors"), base.with_suffix(".json")
    if not tensors_path.exists() or not config_path.exists():
        raise FileNotFoundError(
            f"{tensors_path} not found: run tinybark's weights.converted() once, or pass weights=(tensors, config)"
        )
    return tensors_path, json.loads(config_path.read_text())


def converted_weights(path: str | Path | None = None) -> tuple[dict[str, np.ndarray], dict]:
    """The converted cache's tensors as float32 arrays, and its config."""
    from . import weights

    tensors_path, config = converted(path)
    return weights.load(tensors_path), config


class Bark:
    def __init__(self, device: str = "gpu", dtype: str = "bf16", weights=None, tokenizer: str | None = None,
                 max_seconds: float = 30.0, ffn: str = "bf16"):
        if device != "gpu":
            raise RuntimeError(f"the cuda backend runs on the gpu, not {device!r}")
        import torch

        from . import lengths
        from .engine import Engine

        # The cache file goes to the GPU as it is and is repacked there.
        tensors, config = weights if weights is not None else converted()
        max_len = lengths.subsampled(int(max_seconds * 100), 3)
        self.engine = Engine(tensors, config, dtype=dtype, device="cuda", max_len=max_len, ffn=ffn)
        self.device = torch.cuda.get_device_name(self.engine.device)
        self._tokenizer_path = tokenizer
        self._tokenizer = None
        self._text_table = None

    def tokens(self, samples: np.ndarray) -> list[int]:
        """Token ids of one clip (16 kHz mono float32), without start/blank/pad; EOS kept if hit."""
        return self.engine.tokens_batch([samples])[0]

    def tokens_batch(self, clips: list[np.ndarray]) -> list[list[int]]:
        """Token ids of many clips, packed into one GPU pass: float32 samples, or int16 PCM
        (then moved to the GPU as 16-bit and converted there, as pcm / 32768)."""
        return self.engine.tokens_batch(clips)

    def tokens_long(self, samples: np.ndarray, max_seconds: float = 30.0) -> list[int]:
        """Token ids of a recording of any length, transcribed in pieces of at most
        `max_seconds` (cut at the quietest 100 ms near each piece's end) that are decoded
        together as one batch. Up to `max_seconds` this is `tokens`; beyond it, each piece
        has its own context (no reference counterpart: tinybark transcribes a clip in full
        context, which for ten minutes means one decoder lane of some 75 000 steps)."""
        from . import longform

        x = np.asarray(samples).reshape(-1)
        cuts = longform.cut_points(x, max_seconds)
        return longform.join(self.engine.tokens_batch([x[a:b] for a, b in zip(cuts[:-1], cuts[1:])]))

    def transcribe_long(self, samples: np.ndarray, max_seconds: float = 30.0) -> str:
        return self.tokenizer.decode(self.tokens_long(samples, max_seconds))

    @property
    def tokenizer(self):
        if self._tokenizer is None:
            from .text import Tokenizer

            path = self._tokenizer_path
            if path is None:
                from huggingface_hub import hf_hub_download

                path = hf_hub_download(TOKENIZER_REPO, "tokenizer.json")
            self._tokenizer = Tokenizer(path)
        return self._tokenizer

    def transcribe(self, samples: np.ndarray) -> str:
        return self.transcribe_batch([samples])[0]

    def transcribe_batch(self, clips: list[np.ndarray]) -> list[str]:
        """The text of many clips in one pass: each clip's tokens are joined into bytes on
        the GPU (the tokenizer's piece table held there), and only the bytes come back."""
        from .text import finish

        if self._text_table is None:
            self._text_table = self.engine.text_table(*self.tokenizer.table())
        return [finish(raw) for raw in self.engine.texts_batch(clips, self._text_table)]

    def transcribe_pcm(self, pcm: bytes) -> str:
        """16 kHz s16le mono PCM (tinybark/tinygrad/__init__.py:33-35), converted to float on
        the GPU."""
        return self.transcribe(np.frombuffer(pcm, dtype="<i2").astype(np.int16))

    def close(self) -> None:
        self.engine = None


def load(device: str = "gpu", dtype: str = "bf16", weights=None, tokenizer: str | None = None,
         ffn: str = "bf16") -> Bark:
    """The cuda backend on this process's current GPU, bf16 by default ("fp32" for the
    fp32 parity path). `weights` is (tensors, config): tensors the path of a converted
    fp16 cache file or a dict of the converted arrays; by default tinybark's own cache.
    `ffn="mxfp8"` runs the FFN GEMMs on block-scaled FP8 weights (bf16 only)."""
    return Bark(device, dtype=dtype, weights=weights, tokenizer=tokenizer, ffn=ffn)
