"""Shared test set-up: import paths, the `gpu` marker, and fp16 comparison helpers."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "wzy-flash-serve_b200")
for p in (ROOT, PKG, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU; run with -m gpu")


# Tolerance of the north star for norms / activation / RoPE: within 2 fp16 ulp of the reference math.
ULP_TOL = 2
# Results below the fp16 normal range (|x| < 2^-14) arise only from cancellation of O(1) terms (e.g.
# a*cos - d*sin), where the ulp of the result says nothing about the computation's accuracy: they are
# checked with an absolute bound of 2^-22 (two fp32 ulps of a unit-size term) instead.
SUBNORMAL_ABS_TOL = 2.0 ** -22
F16_MIN_NORMAL = 2.0 ** -14


def f16_ulp_distance(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Distance in units in the last place between two fp16 arrays, on the monotone integer line
    of binary16 (so +0/-0 are 0 apart and a sign change counts every representable step)."""
    ai = np.ascontiguousarray(a, dtype=np.float16).view(np.int16).astype(np.int32)
    bi = np.ascontiguousarray(b, dtype=np.float16).view(np.int16).astype(np.int32)
    ai = np.where(ai < 0, -0x8000 - ai, ai)
    bi = np.where(bi < 0, -0x8000 - bi, bi)
    return np.abs(ai - bi)


def f16_report(got: np.ndarray, want: np.ndarray) -> dict:
    g = np.asarray(got, dtype=np.float32).reshape(-1)
    w = np.asarray(want, dtype=np.float32).reshape(-1)
    d = np.abs(g - w)
    rel = d / np.maximum(np.abs(w), 1e-3)
    ulp = f16_ulp_distance(got, want).reshape(-1)
    tiny = np.abs(w) < F16_MIN_NORMAL
    ulp_normal = np.where(tiny, 0, ulp)
    return {
        "max_abs": float(d.max()) if d.size else 0.0,
        "max_rel": float(rel.max()) if rel.size else 0.0,
        "max_ulp": int(ulp_normal.max()) if ulp.size else 0,  # over |want| >= 2^-14
        "max_abs_tiny": float(d[tiny].max()) if tiny.any() else 0.0,  # over |want| < 2^-14
        "max_ulp_incl_tiny": int(ulp.max()) if ulp.size else 0,
        "frac_exact": float((ulp == 0).mean()) if ulp.size else 1.0,
        "n": int(d.size),
    }


def assert_f16_close(got, want, tol_ulp: int = ULP_TOL, what: str = ""):
    r = f16_report(got, want)
    assert r["max_ulp"] <= tol_ulp and r["max_abs_tiny"] <= SUBNORMAL_ABS_TOL, f"{what}: {r}"
    return r


def assert_f32_in_f16_out_close(got16, want32, atol: float, what: str = ""):
    """fp16 outputs of fp32-input rows (the 4-stream norms). v = R + bo * gate cancels to arbitrarily
    small values, where an fp32-level error (the gate's exponential, ~1e-7 absolute) is many fp16 ulps
    of a result just above 2^-14; the bound is therefore the fp32 test's absolute tolerance plus the
    fp16 rounding of the result: |got - want32| <= atol + ulp16(want32). Elsewhere (|want| >= 2^-6,
    where atol is below a quarter ulp) it is still <= 2 fp16 ulp, asserted separately."""
    g = np.asarray(got16, dtype=np.float32).reshape(-1)
    w = np.asarray(want32, dtype=np.float32).reshape(-1)
    ulp16 = np.spacing(np.abs(w).astype(np.float16)).astype(np.float32)
    err = np.abs(g - w)
    worst = float((err - (atol + ulp16)).max()) if err.size else 0.0
    assert worst <= 0.0, f"{what}: max |err| - (atol + ulp16) = {worst}"
    big = np.abs(w) >= 2.0 ** -6
    if big.any():
        ulp = f16_ulp_distance(g[big].astype(np.float16), w[big].astype(np.float16))
        assert int(ulp.max()) <= ULP_TOL, f"{what}: {int(ulp.max())} fp16 ulp at |want| >= 2^-6"


@pytest.fixture(scope="session")
def orc():
    import oracle as o

    o.lib()
    return o


@pytest.fixture(scope="session")
def wz():
    import wzyb200

    wzyb200.lib()
    return wzyb200
