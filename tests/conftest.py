"""Shared pytest setup: the ``gpu`` marker, package loading and golden fixtures."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = Path(__file__).resolve().parent / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

from __graft_entry__ import load_package  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def gdn():
    """The GDN library package (loaded from its in-tree directory)."""
    return load_package()


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


def rel_err(x: np.ndarray, ref: np.ndarray) -> float:
    """max |x - ref| / max |ref| (0 when both are zero)."""
    den = float(np.max(np.abs(ref))) if ref.size else 0.0
    num = float(np.max(np.abs(x - ref))) if ref.size else 0.0
    return num / den if den > 0 else num


def state_close(x: np.ndarray, ref: np.ndarray, rtol: float = 1e-3) -> tuple[bool, float]:
    """Final-state tolerance used throughout: per (sequence, head),
    max|x - ref| <= rtol * max|ref| and ||x - ref||_F <= rtol * ||ref||_F."""
    x = x.reshape(-1, x.shape[-2] * x.shape[-1]).astype(np.float64)
    ref = ref.reshape(-1, ref.shape[-2] * ref.shape[-1]).astype(np.float64)
    worst = 0.0
    for xi, ri in zip(x, ref):
        den_max = np.max(np.abs(ri))
        den_fro = np.linalg.norm(ri)
        if den_max == 0:
            e = float(np.max(np.abs(xi)))
        else:
            e = max(float(np.max(np.abs(xi - ri)) / den_max),
                    float(np.linalg.norm(xi - ri) / den_fro))
        worst = max(worst, e)
    return worst <= rtol, worst
