"""The 64-bit remainder the kernels use for the PLE fp8 hash and the KV ring cell (mod_u64 in
csrc/common.cuh): q = mulhi(x, m) with m = floor((2^64 - 1) / d), r = x - q*d, then at most two
subtractions of d. Checked here in exact integer arithmetic on the bound it relies on (q never above
x // d and at most two below), over the reference's PLE vocab sizes, ring sizes and random divisors."""
from __future__ import annotations

import numpy as np

M64 = (1 << 64) - 1


def mod_u64(x: int, d: int) -> int:
    m = M64 // d
    q = (x * m) >> 64
    r = (x - q * d) & M64
    assert 0 <= x // d - q <= 2
    if r >= d:
        r -= d
    if r >= d:
        r -= d
    return r


def test_mod_u64_matches_remainder():
    r = np.random.default_rng(5)
    divisors = [1, 2, 3, 127, 4096, 8192, 28672, 20000003, 20000023, 20000077, (1 << 32) - 1, (1 << 32) + 15,
                (1 << 63) + 9, M64] + [int(v) for v in r.integers(1, 1 << 62, 200)]
    xs = [0, 1, M64, M64 - 1, 1 << 63] + [int(v) for v in r.integers(0, 1 << 63, 300)] + \
         [int(v) * 2 + 1 for v in r.integers(0, 1 << 62, 300)]
    for d in divisors:
        for x in xs + [d - 1, d, d + 1, (M64 // d) * d, (M64 // d) * d - 1]:
            x &= M64
            assert mod_u64(x, d) == x % d, (x, d)
