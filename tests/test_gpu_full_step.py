"""GPU parity of the benchmark's timed step at its full size: configs[4], the configs[1]+[2] bundles on
262,144 tokens, through the same buffers, host-built RoPE table and entry points (`wzyb_attn_prep_f16`,
`wzyb_act_f16`) that `bench.py` times.

At this size both bundles issue their ops' own launches, and the RoPE positions run to 262,143, the last
row of the table. The whole step is ~20 GB on the device; the oracle checks a sample of tokens spread over
the range (and the rows at power-of-two boundaries and the last token), each against the oracle with its own
position: the residual bit-exact, the norm, q/k norm + RoPE, SwiGLU and the GDN gated norm within 2 fp16
ulp, as the smaller parity tests do.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import bench
from conftest import ULP_TOL, assert_f16_close

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _sample(t: torch.Tensor, idx: torch.Tensor, shape) -> np.ndarray:
    return t.view(shape).index_select(0, idx).cpu().numpy()


def test_configs4_step_sampled_against_oracle(wz, orc):
    torch.cuda.set_device(0)
    wz.read_faults(clear=True)
    T = bench.TOKENS
    c_h, s_h = wz.rope_table_host(T, bench.ROT, bench.THETA)
    cos, sin = torch.from_numpy(c_h).to(DEV), torch.from_numpy(s_h).to(DEV)
    sh = bench.Shard(wz, torch, T, 0, 1000, DEV, cos, sin)
    rows = sorted(r for r in set(np.linspace(0, T - 1, 64).astype(np.int64).tolist())
                  | {1, 4095, 4096, 65535, 65536, 131071, 131072, T - 1} if r < T)
    idx = torch.tensor(rows, dtype=torch.int64, device=DEV)
    H, QH, KH, HD = bench.HIDDEN, bench.QH, bench.KH, bench.HD
    ER, FFN, GH, GHD = bench.EXPERT_ROWS, bench.FFN, bench.GDN_H, bench.GDN_HD
    pre = {
        "x": _sample(sh.x, idx, (T, H)), "res": _sample(sh.res, idx, (T, H)),
        "q": _sample(sh.q, idx, (T, QH * HD)), "k": _sample(sh.k, idx, (T, KH * HD)),
        "gate": _sample(sh.gate, idx, (T, ER * FFN)), "up": _sample(sh.up, idx, (T, ER * FFN)),
        "o": _sample(sh.o, idx, (T, GH * GHD)), "z": _sample(sh.z, idx, (T, GH * GHD)),
    }
    w, gq, gk, gg = (t.cpu().numpy() for t in (sh.w, sh.gq, sh.gk, sh.gg))

    s = torch.cuda.current_stream()
    for i in range(len(bench.STEP_BUNDLES)):
        sh.launch(i, s)
    torch.cuda.synchronize()
    assert wz.read_faults() == 0
    got = {
        "y": _sample(sh.y, idx, (T, H)), "res": _sample(sh.res, idx, (T, H)),
        "q": _sample(sh.q, idx, (T, QH * HD)), "k": _sample(sh.k, idx, (T, KH * HD)),
        "act": _sample(sh.act, idx, (T, ER * FFN)), "gy": _sample(sh.gy, idx, (T, GH * GHD)),
    }
    del sh
    torch.cuda.empty_cache()

    S = len(rows)
    y_ref, res_ref = orc.add_rmsnorm_f16(pre["x"], pre["res"], w, bench.EPS, 1.0)
    assert np.array_equal(got["res"].view(np.uint16), res_ref.view(np.uint16)), "residual sum"
    assert_f16_close(got["y"], y_ref, ULP_TOL, "add+RMSNorm at 262,144 tokens")
    for i, t in enumerate(rows):
        q_ref = orc.head_norm_rope(pre["q"][i], gq, c_h, s_h, 1, QH, HD, HD, QH * HD, bench.ROT, bench.EPS, 1.0, t)
        k_ref = orc.head_norm_rope(pre["k"][i], gk, c_h, s_h, 1, KH, HD, HD, KH * HD, bench.ROT, bench.EPS, 1.0, t)
        assert_f16_close(got["q"][i], q_ref, ULP_TOL, f"q norm + RoPE at position {t}")
        assert_f16_close(got["k"][i], k_ref, ULP_TOL, f"k norm + RoPE at position {t}")
    assert_f16_close(got["act"], orc.swiglu(pre["gate"], pre["up"]), ULP_TOL, "SwiGLU at 262,144 tokens")
    gy_ref = orc.gdn_gated_norm(pre["o"], pre["z"], gg, S, GH, GHD, bench.EPS, 0.0, wz.GATE_SIGMOID)
    assert_f16_close(got["gy"], gy_ref, ULP_TOL, "GDN gated norm at 262,144 tokens")
