"""CPU: the oracle against golden outputs of the reference's own kernels (generated on a B200 by
tests/golden/make_golden.py from the reference's unmodified headers)."""
from __future__ import annotations

import os

import numpy as np
import pytest

from conftest import GOLDEN, assert_f16_close

PATH = os.path.join(GOLDEN, "ref_kernels_golden.npz")


@pytest.fixture(scope="module")
def gold():
    if not os.path.exists(PATH):
        pytest.skip("golden fixture not generated yet")
    return dict(np.load(PATH))


def test_golden_add_rmsnorm(orc, gold):
    y, res = orc.add_rmsnorm_f16(gold["addnorm_x"], gold["addnorm_res"], gold["addnorm_w"], 1e-6, 1.0)
    assert np.array_equal(res, gold["addnorm_R"].astype(np.float16))
    assert_f16_close(y, gold["addnorm_y"], 1, "add_rmsnorm")


def test_golden_hyper_connection_norm(orc, gold):
    T, n, hc = 4, 256, 4
    xn, _, R = orc.gr_norm_f32(gold["hc_R"], gold["hc_w"], gold["hc_bo"], gold["hc_inj"], T, n, hc)
    np.testing.assert_allclose(R, gold["hc_Rout"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(xn, gold["hc_xn"], rtol=2e-6, atol=2e-6)


def test_golden_head_norm_rope(orc, gold):
    q = gold["rope_q"]
    T, heads, hd = q.shape
    c, s = orc.rope_table(1100, 64, 1e7)
    out = orc.head_norm_rope(q.reshape(-1), gold["rope_gamma"], c, s, T, heads, hd, hd, heads * hd, 64, 1e-6, 1.0,
                             1000)
    assert_f16_close(out, gold["rope_out"].reshape(-1).astype(np.float16), 1, "head_norm_rope")
    out32 = orc.head_norm_rope(q.astype(np.float32).reshape(-1),
                               (np.float32(1) + gold["rope_gamma"].astype(np.float32)).astype(np.float32), c, s, T,
                               heads, hd, hd, heads * hd, 64, 1e-6, 0.0, 1000)
    np.testing.assert_allclose(out32, gold["rope_out"].reshape(-1), rtol=1e-5, atol=2e-6)


def test_golden_gdn(orc, gold):
    o = gold["gdn_o"]
    T, H, hd = o.shape
    y = orc.gdn_gated_norm(o, gold["gdn_z"], gold["gdn_gamma"], T, H, hd, 1e-6, 0.0, 0)
    assert_f16_close(y, gold["gdn_y"], 1, "gdn")


def test_golden_swiglu(orc, gold):
    g, u = gold["swiglu_g"].astype(np.float32), gold["swiglu_u"].astype(np.float32)
    np.testing.assert_allclose(orc.swiglu(g, u), gold["swiglu_out"], rtol=2e-6, atol=2e-6)
    gu = gold["swil_gu"]
    out = orc.swiglu_interleaved(gu, gu.shape[0], gu.shape[1] // 2).astype(np.float16)
    assert_f16_close(out, gold["swil_out"], 1, "swiglu interleaved")


def test_golden_rope_table(orc, gold):
    c, s = orc.rope_table(262144, 64, 1e7)
    pos = gold["ropetab_pos"]
    assert np.array_equal(c[pos].view(np.uint32), gold["ropetab_cos"].view(np.uint32))
    assert np.array_equal(s[pos].view(np.uint32), gold["ropetab_sin"].view(np.uint32))
