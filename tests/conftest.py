"""Shared test setup: import paths, the `gpu` marker, and a per-session engine."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT / "ai-research_b200", ROOT):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (run with -m gpu on a GPU box)")


@pytest.fixture(scope="session")
def engine():
    import sx

    eng = sx.Engine(0)
    yield eng
    eng.close()


@pytest.fixture(scope="session")
def engine_f32kv():
    import sx

    eng = sx.Engine(0, kv_f32=True)
    yield eng
    eng.close()


def assert_close(got, want, atol=1e-3, rtol=1e-2, what="values"):
    """The path's float tolerance: |a - b| <= atol + rtol * |b| elementwise."""
    import numpy as np

    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, f"{what}: shape {got.shape} != {want.shape}"
    err = np.abs(got - want)
    tol = atol + rtol * np.abs(want)
    bad = np.nonzero(err > tol)[0] if got.ndim == 1 else np.argwhere(err > tol)
    assert bad.size == 0, (
        f"{what}: {len(bad)} elements out of tolerance; worst err {err.max():.3e} "
        f"at {np.unravel_index(np.argmax(err - tol), err.shape)}"
    )
