import pathlib
import sys

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")
    config.addinivalue_line("markers", "slow: long-running CPU check")


def reference_compare(actual, expected, tol):
    """tests/conformance.js:7-10: |a - e| <= tol * (1 + |e|) for every element; returns max error."""
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    assert a.shape == e.shape, "length mismatch"
    err = np.abs(a - e)
    bad = ~(np.isfinite(a) & (err <= tol * (1 + np.abs(e))))
    assert not bad.any(), f"first bad index {int(np.argmax(bad))}: {a[bad][:4]} vs {e[bad][:4]}"
    return float(err.max()) if err.size else 0.0


def rel_l2(actual, expected):
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    return float(np.linalg.norm(a - e) / max(np.linalg.norm(e), 1e-30))


@pytest.fixture(scope="session")
def golden():
    return {p.stem: dict(np.load(p)) for p in GOLDEN.glob("*.npz")}


@pytest.fixture(scope="session")
def port():
    from oracle.oracle import Oracle
    return Oracle("port")
