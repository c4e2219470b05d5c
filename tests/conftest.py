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
