"""Test setup: the `gpu` marker, the package import, and shared fixtures.

Tests marked `gpu` run the CUDA path on a B200 and compare it with the CPU oracle (oracle/); the
rest run anywhere: the oracle against tgtts-v4's own known answers, the host logic, and that the
C-ABI library loads and exports what include/tgcuda.h declares.
"""

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import __graft_entry__ as entry  # noqa: E402

entry.load_package()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA kernels)")


@pytest.fixture(scope="session")
def pkg():
    return entry.load_package()


@pytest.fixture(scope="session")
def syn():
    from tgtts_v4_b200 import synthetic

    return synthetic


@pytest.fixture(scope="session")
def ctx(pkg):
    c = pkg.Context(0)
    yield c
    c.close()


def distance(got, want):
    """max |d|, relative RMS of d, and the cosine of got against want (f64)."""
    import numpy as np

    g = np.asarray(got, np.float64).ravel()
    w = np.asarray(want, np.float64).ravel()
    d = g - w
    max_abs = float(np.max(np.abs(d))) if d.size else 0.0
    rel = float(np.sqrt(np.sum(d * d) / max(np.sum(w * w), 1e-300)))
    cos = float(np.dot(g, w) / max(np.sqrt(np.dot(g, g) * np.dot(w, w)), 1e-300))
    return max_abs, rel, cos
