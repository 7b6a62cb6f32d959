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


def assert_close_bf16_operands(got, want, what="values", frac=1e-2, scale_tol=1e-3):
    """The f32 tolerance for a path that multiplies bf16 operands (the batched prefill), with
    an allowance for double rounding: the path and the checker each round their own f32 value
    to bf16, and where those f32 values straddle a bf16 rounding boundary (a 1-ulp difference
    before rounding) one operand differs by 2^-8, which attention at scale 1.0 can amplify.
    A flip in a late layer moves many logits a little (measured on the 3-layer test model:
    7 of 4096 logits past the elementwise bound, worst 6e-3 at a scale of 110, i.e. 6e-5 of
    it), while a wrong operand, slot or head moves them by the order of the scale.  So: all
    but a fraction `frac` of the elements must meet |a - b| <= 1e-3 + 1e-2 |b|, and every
    element must lie within scale_tol of the vector's scale max |b|."""
    import numpy as np

    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, f"{what}: shape {got.shape} != {want.shape}"
    err = np.abs(got - want)
    bad = int(np.count_nonzero(err > 1e-3 + 1e-2 * np.abs(want)))
    scale = float(np.abs(want).max())
    stats = (f"{bad} of {err.size} elements past the elementwise bound, worst err "
             f"{err.max():.3e} = {err.max() / max(scale, 1e-30):.2e} of the scale {scale:.3e}")
    assert bad <= max(1, int(frac * err.size)), f"{what}: {stats} (allowed fraction {frac})"
    assert err.max() <= scale_tol * scale, f"{what}: {stats} (allowed {scale_tol} of the scale)"


# With a bf16 KV cache on top of bf16 operands, every cached K/V element is a second place
# where the two sides round f32 values that may differ by an ulp: more elements move a little
# (measured on the bf16-cache prefill test, 8 q heads per kv head: 41 of 4096 logits past the
# elementwise bound), while the scale bound, which a wrong slot, head or operand breaks by
# orders of magnitude, stays as tight.
BF16_KV_FRAC = 5e-2
