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


def f16_ulp_distance(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Distance in units in the last place between two fp16 arrays, on the monotone integer line
    of binary16 (so +0/-0 are 0 apart and a sign change counts every representable step)."""
    ai = np.ascontiguousarray(a, dtype=np.float16).view(np.int16).astype(np.int32)
    bi = np.ascontiguousarray(b, dtype=np.float16).view(np.int16).astype(np.int32)
    ai = np.where(ai < 0, -0x8000 - ai, ai)
    bi = np.where(bi < 0, -0x8000 - bi, bi)
    return np.abs(ai - bi)


def f16_report(got: np.ndarray, want: np.ndarray) -> dict:
    g = np.asarray(got, dtype=np.float32)
    w = np.asarray(want, dtype=np.float32)
    d = np.abs(g - w)
    rel = d / np.maximum(np.abs(w), 1e-3)
    ulp = f16_ulp_distance(got, want)
    return {
        "max_abs": float(d.max()) if d.size else 0.0,
        "max_rel": float(rel.max()) if rel.size else 0.0,
        "max_ulp": int(ulp.max()) if ulp.size else 0,
        "frac_exact": float((ulp == 0).mean()) if ulp.size else 1.0,
        "n": int(d.size),
    }


def assert_f16_close(got, want, tol_ulp: int = ULP_TOL, what: str = ""):
    r = f16_report(got, want)
    assert r["max_ulp"] <= tol_ulp, f"{what}: {r}"
    return r


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
