"""Shared test set-up.

* registers the ``gpu`` marker (tests that need a B200; the CPU suite runs with
  ``-m "not gpu"``) and the ``new_on_gpu`` marker (GPU tests not yet run on a B200,
  ordered after the rest);
* builds the oracle (oracle/libsmol_oracle.so) and the product library
  (smol-genius_b200/libsmol_b200.so) when they are missing, so a fresh checkout
  can run the suite directly;
* puts the oracle and the binding on sys.path.
"""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_DIR = os.path.join(ROOT, "oracle")
PKG_DIR = os.path.join(ROOT, "smol-genius_b200")
GOLDEN = os.path.join(ROOT, "tests", "golden", "reference_cases.npz")

for p in (ORACLE_DIR, PKG_DIR):
    if p not in sys.path:
        sys.path.insert(0, p)

# Tolerances of the north star: attention outputs vs the fp32 reference fed the same
# bf16-rounded inputs.
REL_L2_TOL = 1e-3
MAX_ABS_TOL = 1e-2


def _ensure_built() -> None:
    if not os.path.exists(os.path.join(ORACLE_DIR, "libsmol_oracle.so")):
        subprocess.run(["make", "-C", ORACLE_DIR, "oracle"], check=True, capture_output=True)
    if not os.path.exists(os.path.join(PKG_DIR, "libsmol_b200.so")):
        subprocess.run(["make", "-C", PKG_DIR, "-j8"], check=True, capture_output=True)


_ensure_built()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) CUDA device")
    config.addinivalue_line("markers", "new_on_gpu(stage=0): a GPU test not yet run on a B200; runs after the rest")


def pytest_collection_modifyitems(config, items):
    """Tests marked new_on_gpu run after the established ones (the sort is stable), so
    that under -x a failure in one of them cannot keep the established tests from
    running; among them by `stage` (default 0): unit tests of a new kernel before the
    tests built on it.  test_zz_no_alloc.py stays the very last file: the
    allocation-free entry point's tests must find every other test already run."""
    def key(item):
        if os.path.basename(str(item.fspath)) == "test_zz_no_alloc.py":
            return (2, 0)
        mark = item.get_closest_marker("new_on_gpu")
        return (0, 0) if mark is None else (1, mark.kwargs.get("stage", 0))
    items.sort(key=key)


@pytest.fixture(scope="session")
def golden():
    return np.load(GOLDEN)


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def assert_close(got, want, what=""):
    import pyoracle
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, f"{what}: shape {got.shape} vs {want.shape}"
    assert np.all(np.isfinite(got)), f"{what}: non-finite values"
    e = pyoracle.rel_l2(got, want)
    m = float(np.abs(got - want).max()) if got.size else 0.0
    assert e <= REL_L2_TOL and m <= MAX_ABS_TOL, f"{what}: rel-L2 {e:.3e} (tol {REL_L2_TOL}), max-abs {m:.3e}"
    return e, m


def assert_within_bf16_truncation(got, ref_bits, rel_tol, abs_tol=1e-6, what=""):
    """The reference's bf16 decoder truncates its fp32 results toward zero
    (qkn_bf16_decoder.c:30-35), so the value it computed lies in [|t|, |t| + ulp(t)) with
    t's sign, t the stored bf16.  `got` (fp32) passes when its distance to that interval
    is at most rel_tol * |got| + abs_tol everywhere.  Returns the largest distance
    relative to |got| + 1e-30."""
    got = np.asarray(got, np.float64)
    bits = np.asarray(ref_bits, np.uint16).astype(np.uint32)
    t = (bits << 16).view(np.float32).astype(np.float64)
    exp = (bits >> 7) & 0xFF
    ulp = np.where(exp > 0, np.ldexp(1.0, exp.astype(np.int64) - 127 - 7), np.ldexp(1.0, -133))
    lo, hi = np.abs(t), np.abs(t) + ulp
    same = (np.sign(got) == np.sign(t)) | (t == 0) | (got == 0)
    a = np.abs(got)
    dist = np.where(same, np.maximum(0.0, np.maximum(lo - a, a - hi)), a + np.abs(t))
    bad = dist > rel_tol * a + abs_tol
    if bad.any():
        i = int(np.argmax(np.where(bad, dist - rel_tol * a, -1.0)))
        raise AssertionError(f"{what}: {int(bad.sum())} of {bad.size} outside the truncation interval; worst at "
                             f"{i}: got {got.flat[i]:.6g}, reference {t.flat[i]:.6g}, distance {dist.flat[i]:.3e}")
    return float((dist / (a + 1e-30)).max())
