import json
import sys
from functools import lru_cache
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA GPU (sm_100a); run with -m gpu")


@lru_cache(maxsize=None)
def golden_npz(name: str) -> dict[str, np.ndarray]:
    with np.load(GOLDEN / name) as z:
        return {k: z[k] for k in z.files}


@lru_cache(maxsize=None)
def golden_json(name: str):
    return json.loads((GOLDEN / name).read_text())


@lru_cache(maxsize=None)
def state_dict(layers: int, seed: int = 0):
    from tinybark_b200 import synthetic

    return synthetic.state_dict(seed, layers=layers)


def max_rel(a, b) -> float:
    """max |a - b| / max |b|: the tolerance metric of the parity checks."""
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.fixture(scope="session")
def sd2():
    return state_dict(2)


@pytest.fixture(scope="session")
def sd24():
    return state_dict(24)


def repack_numpy(jobs, source: np.ndarray, size: int) -> np.ndarray:
    """tb_repack's job semantics restated in numpy (the checker of its kernel and of the
    packed layout): jobs as pack.Layout.jobs tuples, `source` the source bytes (uint8);
    returns the `size` destination bytes, zero where no job writes."""
    import torch

    out = np.zeros(size, np.uint8)
    for src_off, dst_off, strides, dims, src_type, dst_type, fill, value in jobs:
        n = int(np.prod(dims))
        if n == 0:
            continue
        if fill:
            vals = np.full(n, value, np.float32)
        else:
            dt = np.float16 if src_type == 0 else np.float32
            src = source[src_off : src_off + (len(source) - src_off) // dt().itemsize * dt().itemsize].view(dt)
            idx = np.zeros((1, 1, 1, 1), np.int64)
            for k, (d, s) in enumerate(zip(dims, strides)):
                shape = [1, 1, 1, 1]
                shape[k] = d
                idx = idx + (np.arange(d, dtype=np.int64) * s).reshape(shape)
            vals = src[idx.reshape(-1)].astype(np.float32)
        if dst_type == 1:
            raw = torch.from_numpy(vals).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint8)
        else:
            raw = vals.view(np.uint8)
        out[dst_off : dst_off + raw.size] = raw
    return out



def synthetic_tokenizer(path, vocab: int = 8193, seed: int = 0) -> str:
    from tinybark_b200 import synthetic

    return synthetic.tokenizer(path, vocab, seed)
