"""The backend registry of tinybark (tinybark/backends.py:1-142) with the `cuda` backend
this package adds. `Model`, `Backend` and `DEVICES` mirror the reference's definitions
(tinybark/backends.py:18-39) so the entry reads as it will in tinybark's own registry, where
a maintainer adds that one entry.

    bark = BACKENDS["cuda"].load("gpu")
    text = bark.transcribe(samples)  # 16 kHz mono float32 NumPy array
"""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass
from typing import Protocol

import numpy as np

DEVICES = ("gpu", "cpu")


class Model(Protocol):
    device: str

    def tokens(self, samples: np.ndarray) -> list[int]: ...

    def transcribe(self, samples: np.ndarray) -> str: ...


@dataclass(frozen=True)
class Backend:
    name: str
    descriptions: dict[str, str]
    prepare: Callable[[], object]
    load: Callable[[str], Model]
    envs: dict[str, dict[str, str]] | None = None

    def env(self, device: str) -> dict[str, str]:
        return (self.envs or {}).get(device, {})


def _cuda(device: str) -> Model:
    from . import load

    return load(device)


def _prepare_cuda() -> None:
    from . import build

    build.build()


BACKENDS = {
    "cuda": Backend(
        "cuda",
        {"gpu": "hand-written sm_100a CUDA kernels through a C ABI, bf16 tensor cores, NVIDIA B200"},
        _prepare_cuda,
        _cuda,
    )
}
