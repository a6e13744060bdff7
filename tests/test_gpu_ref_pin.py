"""GPU: pin the oracle (and the CUDA path) against the reference's OWN kernels, compiled from its
unmodified headers into oracle/_ref/libwzyref.so and launched with the reference's launch shapes.

Inputs are fp16-exact values fed to the reference's fp32 kernels; the zero-centred weight (1+w) is
handed to the reference as g = 1.0f + w computed in fp32, since the reference applies raw weights.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import ULP_TOL, assert_f16_close

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module")
def ref(orc):
    if not orc.ref_available():
        pytest.skip("oracle/_ref/libwzyref.so not built (needs the reference sources at build time)")
    return orc.ref_lib()


_KEEP = []


@pytest.fixture(autouse=True)
def _keep_alive():
    yield
    torch.cuda.synchronize()
    _KEEP.clear()


def dev(a):
    # Kept alive until the test ends: a raw pointer taken from a temporary tensor would otherwise let
    # the caching allocator hand the same block to the next tensor before the kernel has run.
    t = torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    _KEEP.append(t)
    return t


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def sp():
    return torch.cuda.current_stream().cuda_stream


def test_pin_add_rmsnorm_baseline(ref, orc, wz):
    """configs[1] add+RMSNorm [4096, 2048] vs pf_gr_norm_fp16 (hc=1, gate 1.0)."""
    r = np.random.default_rng(201)
    T, n = 4096, 2048
    x = r.standard_normal((T, n)).astype(np.float16)
    res = r.standard_normal((T, n)).astype(np.float16)
    w = (0.02 * r.standard_normal(n)).astype(np.float16)
    g32 = (np.float32(1.0) + w.astype(np.float32)).astype(np.float32)
    dR = dev(res.astype(np.float32))
    dxn = torch.empty((T, n), dtype=torch.float16, device=DEV)
    inj0 = torch.zeros(T, dtype=torch.float32, device=DEV)
    assert ref.ref_pf_gr_norm_fp16(dR.data_ptr(), dev(g32).data_ptr(), dev(x.astype(np.float32)).data_ptr(),
                                   inj0.data_ptr(), dxn.data_ptr(), T, n, 1, 1e-6, sp()) == 0
    ref_y, ref_R = host(dxn), host(dR)
    y_or, res_or = orc.add_rmsnorm_f16(x, res, w, 1e-6, 1.0)
    assert np.array_equal(res_or, ref_R.astype(np.float16))
    assert_f16_close(y_or, ref_y, 1, "oracle vs reference pf_gr_norm_fp16")
    dres, dy = dev(res), torch.empty((T, n), dtype=torch.float16, device=DEV)
    wz.add_rmsnorm_f16(dev(x), dres, dev(w), dy, 1e-6, 1.0)
    assert np.array_equal(host(dres), res_or)
    assert_f16_close(host(dy), ref_y, ULP_TOL, "CUDA vs reference pf_gr_norm_fp16")


def test_pin_gr_norm_hyper_connection(ref, orc, wz):
    """fused_gr_norm_multi with 4 streams and learned inject gates (fp32)."""
    r = np.random.default_rng(202)
    T, n, hc = 8, 2560, 4
    R = r.standard_normal((T * hc, n)).astype(np.float32)
    bo = r.standard_normal((T, n)).astype(np.float32)
    inj = r.standard_normal((T * hc,)).astype(np.float32)
    w = (1 + 0.02 * r.standard_normal((hc, n))).astype(np.float32)
    dR, dxn = dev(R), torch.empty((T * hc, n), dtype=torch.float32, device=DEV)
    assert ref.ref_fused_gr_norm_multi(dR.data_ptr(), dev(w).data_ptr(), dev(bo).data_ptr(), dev(inj).data_ptr(),
                                       dxn.data_ptr(), T, n, hc, 1e-6, sp()) == 0
    ref_xn, ref_R = host(dxn), host(dR)
    xn_or, _, R_or = orc.gr_norm_f32(R, w, bo, inj, T, n, hc)
    np.testing.assert_allclose(R_or, ref_R, rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(xn_or, ref_xn, rtol=2e-6, atol=2e-6)
    dR2, dxn2 = dev(R), torch.empty((T * hc, n), dtype=torch.float32, device=DEV)
    wz.gr_norm_f32(dR2, dev(w), dev(bo), dev(inj), dxn2, T, n, hc)
    np.testing.assert_allclose(host(dR2), ref_R, rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(host(dxn2), ref_xn, rtol=2e-6, atol=2e-6)


@pytest.mark.parametrize("heads,hd", [(16, 256), (2, 256), (4, 128)])
def test_pin_head_norm_rope(ref, orc, wz, heads, hd):
    """fused_head_norm_rope_multi (rot 64, theta 1e7) at the configs[1] token count."""
    r = np.random.default_rng(203 + heads)
    T = 4096
    x = r.standard_normal((T, heads, hd)).astype(np.float16)
    gam = (0.02 * r.standard_normal(hd)).astype(np.float16)
    g32 = (np.float32(1.0) + gam.astype(np.float32)).astype(np.float32)
    c, s = orc.ref_rope_table(T + 100, 1e7)
    dc, ds = dev(c), dev(s)
    base = torch.tensor([100], dtype=torch.int32, device=DEV)
    d32 = dev(x.astype(np.float32))
    assert ref.ref_fused_head_norm_rope_multi(d32.data_ptr(), dev(g32).data_ptr(), dc.data_ptr(), ds.data_ptr(),
                                              base.data_ptr(), T, heads, hd, hd, heads * hd, 1e-6, sp()) == 0
    ref_out = host(d32).reshape(-1)
    # oracle fp32 path vs the reference, then the fp16 outputs
    or32 = orc.head_norm_rope(x.astype(np.float32).reshape(-1), g32, c, s, T, heads, hd, hd, heads * hd, 64, 1e-6,
                              0.0, 100)
    np.testing.assert_allclose(or32, ref_out, rtol=1e-5, atol=2e-6)
    or16 = orc.head_norm_rope(x.reshape(-1), gam, c, s, T, heads, hd, hd, heads * hd, 64, 1e-6, 1.0, 100)
    # fp32 results agree to ~1e-6; after rounding both to fp16 a value can land 1 ulp apart on either
    # side of a binade boundary, i.e. 2 ulp on the fp16 integer line.
    assert_f16_close(or16, ref_out.astype(np.float16), ULP_TOL, "oracle vs reference head norm rope")
    d16 = dev(x)
    wz.head_norm_rope(d16, dev(gam), dc, ds, T, heads, hd, hd, heads * hd, 64, 1e-6, 1.0, d_base_pos=base)
    assert_f16_close(host(d16).reshape(-1), ref_out.astype(np.float16), ULP_TOL, "CUDA vs reference")


def test_pin_gdn_gated_norm(ref, orc, wz):
    """configs[2] GDN gated norm [4096, 32, 128] vs pf_gdn_rmsnorm_gate_parallel (sigmoid gate)."""
    r = np.random.default_rng(204)
    T, H, hd = 4096, 32, 128
    o = r.standard_normal((T, H, hd)).astype(np.float16)
    z = r.standard_normal((T, H, hd)).astype(np.float16)
    gm = (1 + 0.02 * r.standard_normal(hd)).astype(np.float16)
    dy = torch.empty((T, H, hd), dtype=torch.float16, device=DEV)
    assert ref.ref_pf_gdn_rmsnorm_gate_parallel(dev(o.astype(np.float32)).data_ptr(),
                                                dev(z.astype(np.float32)).data_ptr(),
                                                dev(gm.astype(np.float32)).data_ptr(), dy.data_ptr(), T, H, 1e-6,
                                                sp()) == 0
    ref_y = host(dy)
    assert_f16_close(orc.gdn_gated_norm(o, z, gm, T, H, hd, 1e-6, 0.0, 0), ref_y, 1, "oracle vs reference gdn")
    dy2 = torch.empty_like(dy)
    wz.gdn_gated_norm(dev(o), dev(z), dev(gm), dy2, T, H, hd, 1e-6, 0.0, 0)
    assert_f16_close(host(dy2), ref_y, ULP_TOL, "CUDA vs reference gdn")


def test_pin_swiglu(ref, orc, wz):
    """configs[2] SwiGLU [45056, 512] vs silu_mul_multi; interleaved vs pf_silu_mul_interleaved_to_fp16."""
    r = np.random.default_rng(205)
    rows, cols = 4096 * 11, 512
    g = r.standard_normal((rows, cols)).astype(np.float16)
    u = r.standard_normal((rows, cols)).astype(np.float16)
    out = torch.empty((rows, cols), dtype=torch.float32, device=DEV)
    assert ref.ref_silu_mul_multi(dev(g.astype(np.float32)).data_ptr(), dev(u.astype(np.float32)).data_ptr(),
                                  out.data_ptr(), rows * cols, sp()) == 0
    ref_o = host(out)
    np.testing.assert_allclose(orc.swiglu(g.astype(np.float32), u.astype(np.float32)), ref_o, rtol=2e-6, atol=2e-6)
    assert_f16_close(orc.swiglu(g, u), ref_o.astype(np.float16), 1, "oracle vs reference silu_mul")
    o16 = torch.empty((rows, cols), dtype=torch.float16, device=DEV)
    wz.swiglu(dev(g), dev(u), o16)
    assert_f16_close(host(o16), ref_o.astype(np.float16), ULP_TOL, "CUDA vs reference silu_mul")
    T, nff = 4096, 640
    gu = r.standard_normal((T, 2 * nff)).astype(np.float32)
    ro = torch.empty((T, nff), dtype=torch.float16, device=DEV)
    assert ref.ref_pf_silu_mul_interleaved_to_fp16(dev(gu).data_ptr(), ro.data_ptr(), T, nff, sp()) == 0
    mine = torch.empty_like(ro)
    wz.swiglu_interleaved(dev(gu), mine, T, nff)
    assert_f16_close(host(mine), host(ro), ULP_TOL, "CUDA vs reference interleaved")
    assert_f16_close(orc.swiglu_interleaved(gu, T, nff).astype(np.float16), host(ro), 1, "oracle vs reference il")


def test_pin_bf16_embedding_gather(ref, orc, wz):
    """mtp_gather_bf16_emb at its own hard-wired shape [248320, 2560], incl. out-of-range ids."""
    ne, nv = ctypes_dims(ref)
    gen = torch.Generator(device=DEV).manual_seed(206)
    table = torch.randint(-32768, 32767, (nv, ne), generator=gen, device=DEV, dtype=torch.int32).to(torch.int16)
    ids = np.concatenate([np.random.default_rng(206).integers(0, nv, 60), [-7, nv, nv + 100, 0]]).astype(np.int32)
    dids = dev(ids)
    ro = torch.empty((ids.size, ne), dtype=torch.float32, device=DEV)
    assert ref.ref_mtp_gather_bf16_emb(table.data_ptr(), dids.data_ptr(), ro.data_ptr(), ids.size, sp()) == 0
    mine = torch.empty_like(ro)
    wz.embed_gather_bf16_f32(table, dids, mine, wz.OOB_CLAMP)
    assert np.array_equal(host(mine).view(np.uint32), host(ro).view(np.uint32))
    want, _ = orc.embed_gather_bf16_f32(host(table).view(np.uint16), ids, 0)
    assert np.array_equal(want.view(np.uint32), host(ro).view(np.uint32))


def test_pin_plain_row_norm(ref, orc, wz):
    """ple_group_multi (the reference's generic per-stream row RMSNorm) vs the no-add norm path."""
    r = np.random.default_rng(207)
    T, n, hc = 6, 2560, 4
    x = r.standard_normal((T * hc, n)).astype(np.float32)
    g = (1 + 0.02 * r.standard_normal((hc, n))).astype(np.float32)
    ry = torch.empty((T * hc, n), dtype=torch.float32, device=DEV)
    assert ref.ref_ple_group_multi(dev(x).data_ptr(), dev(g).data_ptr(), ry.data_ptr(), T, n, hc, 1e-6, sp()) == 0
    mine = torch.empty_like(ry)
    dx = dev(x)
    wz.gr_norm_f32(dx, dev(g), None, None, mine, T, n, hc)
    np.testing.assert_allclose(host(mine), host(ry), rtol=2e-6, atol=2e-6)
    assert np.array_equal(host(dx), x)
    # in place, as the reference calls it on ple_k (src/wzy_stage_v2.cuh:590), for every design
    for v in (wz.VARIANT_AUTO, wz.VARIANT_DIRECT, wz.VARIANT_ASYNC, wz.VARIANT_WIDE):
        wz.set_kernel_variant(wz.FAM_NORM, v)
        ip = dev(x)
        wz.gr_norm_f32(ip, dev(g), None, None, ip, T, n, hc)
        np.testing.assert_allclose(host(ip), host(ry), rtol=2e-6, atol=2e-6)
    wz.set_kernel_variant(wz.FAM_NORM, wz.VARIANT_AUTO)


def ctypes_dims(ref):
    import ctypes

    a, b = ctypes.c_int(), ctypes.c_int()
    ref.ref_dims(ctypes.byref(a), ctypes.byref(b))
    return a.value, b.value


def test_pin_q8_side_outputs(ref, orc, wz):
    """fused_gr_norm_multi's xq8/xs8 and silu_mul_quant32_multi at the reference's decode shapes."""
    r = np.random.default_rng(208)
    T, n, hc = 8, 2560, 4
    R = r.standard_normal((T * hc, n)).astype(np.float32)
    bo = r.standard_normal((T, n)).astype(np.float32)
    inj = r.standard_normal(T * hc).astype(np.float32)
    w = (1 + 0.02 * r.standard_normal((hc, n))).astype(np.float32)
    dR, dxn = dev(R), torch.empty((T * hc, n), dtype=torch.float32, device=DEV)
    dq = torch.empty((T * hc, n), dtype=torch.int8, device=DEV)
    ds = torch.empty((T * hc, n // 32), dtype=torch.float32, device=DEV)
    assert ref.ref_fused_gr_norm_multi_q8(dR.data_ptr(), dev(w).data_ptr(), dev(bo).data_ptr(), dev(inj).data_ptr(),
                                          dxn.data_ptr(), dq.data_ptr(), ds.data_ptr(), T, n, hc, 1e-6, sp()) == 0
    rq, rs = host(dq), host(ds)
    mq = torch.empty_like(dq)
    ms = torch.empty_like(ds)
    wz.gr_norm_q8_f32(dev(R), dev(w), dev(bo), dev(inj), torch.empty_like(dxn), mq, ms, T, n, hc)
    d = np.abs(host(mq).astype(np.int32) - rq.astype(np.int32))
    assert d.max() <= 1 and (d > 0).mean() < 1e-3
    np.testing.assert_allclose(host(ms), rs, rtol=4e-6)
    # SwiGLU + Q8: the same expression on the same inputs -> identical codes and scales
    nff = 640
    g = (2 * r.standard_normal(nff * T)).astype(np.float32)
    u = r.standard_normal(nff * T).astype(np.float32)
    # groups of tiny products: 127 / amax overflows (codes +-127 / 0), and amax / 127 rounds to 0
    for i, scale in enumerate([1e-38, 2e-37, 1e-42, 1e-44]):
        u[32 * i:32 * i + 32] *= np.float32(scale)
    q32 = torch.empty(nff * T, dtype=torch.int8, device=DEV)
    s32 = torch.empty(nff * T // 32, dtype=torch.float32, device=DEV)
    dg, du = dev(g), dev(u)
    assert ref.ref_silu_mul_quant32_multi(dg.data_ptr(), du.data_ptr(), q32.data_ptr(), s32.data_ptr(),
                                          nff * T // 32, sp()) == 0
    mq2, ms2 = torch.empty_like(q32), torch.empty_like(s32)
    wz.swiglu_q8_f32(dg, du, mq2, ms2)
    assert np.array_equal(host(mq2), host(q32))
    assert np.array_equal(host(ms2).view(np.uint32), host(s32).view(np.uint32))


def test_pin_hyper_connection_residual(ref, orc, wz):
    """gr_write_multi, pf_gr_up_mean_fp16, gr_up_gate_mean_pf_kernel and silu_div_hc_to_fp16_kernel at the
    reference's stream count (4) and width (2560)."""
    r = np.random.default_rng(209)
    T, n, hc = 64, 2560, 4
    # gated write: same gate expression, same fused multiply-add -> identical R
    R = r.standard_normal((T * hc, n)).astype(np.float32)
    blk = r.standard_normal((T, n)).astype(np.float32)
    inj = r.standard_normal(T * hc).astype(np.float32)
    dR, dblk, dinj = dev(R), dev(blk), dev(inj)
    assert ref.ref_gr_write_multi(dR.data_ptr(), dblk.data_ptr(), dinj.data_ptr(), T, n, hc, sp()) == 0
    ref_R = host(dR)
    np.testing.assert_allclose(orc.gr_write_f32(R, blk, inj, T, n, hc), ref_R, rtol=1e-6, atol=1e-6)
    mR = dev(R)
    wz.gr_write_f32(mR, dblk, dinj, T, n, hc)
    assert np.array_equal(host(mR), ref_R)
    # stream mixing, fp16 in
    xn = r.standard_normal((T, hc, n)).astype(np.float16)
    gg = (2 * r.standard_normal((T, hc, n))).astype(np.float16)
    dx, dg = dev(xn), dev(gg)
    m32 = torch.empty((T, n), dtype=torch.float32, device=DEV)
    m16 = torch.empty((T, n), dtype=torch.float16, device=DEV)
    assert ref.ref_pf_gr_up_mean_fp16(dx.data_ptr(), dg.data_ptr(), m32.data_ptr(), m16.data_ptr(), T, n, sp()) == 0
    r32, r16 = host(m32), host(m16)
    o32, o16 = orc.hc_mix(xn, gg, T, n, hc)
    np.testing.assert_allclose(o32, r32, rtol=2e-6, atol=2e-6)
    assert_f16_close(o16, r16, 1, "oracle vs reference pf_gr_up_mean_fp16")
    w32, w16 = torch.empty_like(m32), torch.empty_like(m16)
    wz.hc_mix(dx, dg, w32, w16, T, n, hc)
    np.testing.assert_allclose(host(w32), r32, rtol=2e-6, atol=2e-6)
    assert_f16_close(host(w16), r16, ULP_TOL, "CUDA vs reference pf_gr_up_mean_fp16")
    # stream mixing, fp32 in
    dx32, dg32 = dev(xn.astype(np.float32)), dev(gg.astype(np.float32))
    assert ref.ref_gr_up_gate_mean_pf(dx32.data_ptr(), dg32.data_ptr(), m32.data_ptr(), T, n, sp()) == 0
    f32 = torch.empty_like(m32)
    wz.hc_mix(dx32, dg32, f32, None, T, n, hc)
    np.testing.assert_allclose(host(f32), host(m32), rtol=2e-6, atol=2e-6)
    # scaled SiLU of the low-rank activations [T, 320] -> fp16
    lo = (4 * r.standard_normal(T * 320)).astype(np.float32)
    dlo = dev(lo)
    lo16 = torch.empty(T * 320, dtype=torch.float16, device=DEV)
    assert ref.ref_silu_div_hc_to_fp16(dlo.data_ptr(), lo16.data_ptr(), T * 320, 0.25, sp()) == 0
    r_lo = host(lo16)
    assert_f16_close(orc.silu_scale_f16(lo, 0.25), r_lo, 1, "oracle vs reference silu_div_hc")
    w_lo = torch.empty_like(lo16)
    wz.silu_scale_f16(dlo, w_lo, 0.25)
    assert_f16_close(host(w_lo), r_lo, ULP_TOL, "CUDA vs reference silu_div_hc")


def _kv_planes(ring_cap, max_ctx, kvd=512):
    z = lambda rows, cols, dt: torch.zeros((rows, cols), dtype=dt, device=DEV)  # noqa: E731
    return {"rkq": z(ring_cap, kvd, torch.int8), "rks": z(ring_cap, kvd // 64, torch.int16),
            "rvq": z(ring_cap, kvd, torch.int8), "rvs": z(ring_cap, kvd // 64, torch.int16),
            "fkq": z(max_ctx, kvd, torch.int8), "fks": z(max_ctx, kvd // 64, torch.int16),
            "fvq": z(max_ctx, kvd, torch.int8), "fvs": z(max_ctx, kvd // 64, torch.int16)}


def _ref_append(ref, k, v, p, dpos, T, cap, max_ctx):
    assert ref.ref_kv_append_int8_multi(k.data_ptr(), v.data_ptr(), *(p[n].data_ptr() for n in (
        "rkq", "rks", "rvq", "rvs", "fkq", "fks", "fvq", "fvs")), dpos.data_ptr(), T, cap, max_ctx, sp()) == 0


@pytest.mark.parametrize("T,base,cap,max_ctx", [(300, 4000, 8200, 9000), (40, 5, 16, 40), (4096, 0, 32768, 4096)])
def test_pin_kv_append_int8(ref, orc, wz, T, base, cap, max_ctx):
    """kv_append_int8_multi (KVD 512 = 2 heads x 256) with the ring's sink, window and wrap, and the
    full-context mirror: identical codes and fp16 scales."""
    r = np.random.default_rng(210 + T)
    k = r.standard_normal((T, 512)).astype(np.float32)
    v = (3 * r.standard_normal((T, 512))).astype(np.float32)
    dk, dv = dev(k), dev(v)
    dpos = torch.tensor([base], dtype=torch.int32, device=DEV)
    pr = _kv_planes(cap, max_ctx)
    _ref_append(ref, dk, dv, pr, dpos, T, cap, max_ctx)
    pm = _kv_planes(cap, max_ctx)
    cache = wz.kv_cache(pm["rkq"], pm["rks"], pm["rvq"], pm["rvs"], cap, max_ctx, pm["fkq"], pm["fks"], pm["fvq"],
                        pm["fvs"])
    wz.kv_append_int8_f32(dk, dv, T, 2, 256, cache, d_base_pos=dpos)
    oc = orc.KvCache(cap, max_ctx, 512, True)
    orc.kv_append_int8_f32(k, v, T, 512, base, oc)
    for nm in pr:
        got_ref = host(pr[nm])
        assert np.array_equal(host(pm[nm]), got_ref), f"CUDA vs reference {nm}"
        want = getattr(oc, nm)
        assert np.array_equal(got_ref.view(want.dtype), want), f"oracle vs reference {nm}"


def test_pin_k_rope_kv_append(ref, orc, wz):
    """The reference's k fused_head_norm_rope_multi + kv_append_int8_multi vs the one fused launch."""
    r = np.random.default_rng(211)
    T, base, cap, max_ctx = 64, 4090, 32768, 8192
    k = r.standard_normal((T, 512)).astype(np.float32)
    v = r.standard_normal((T, 512)).astype(np.float32)
    gam = (0.02 * r.standard_normal(256)).astype(np.float32)
    g32 = (np.float32(1.0) + gam).astype(np.float32)
    c, s = orc.ref_rope_table(base + T + 8, 1e7)
    dc, ds = dev(c), dev(s)
    dpos = torch.tensor([base], dtype=torch.int32, device=DEV)
    dk, dv = dev(k), dev(v)
    assert ref.ref_fused_head_norm_rope_multi(dk.data_ptr(), dev(g32).data_ptr(), dc.data_ptr(), ds.data_ptr(),
                                              dpos.data_ptr(), T, 2, 256, 256, 512, 1e-6, sp()) == 0
    pr = _kv_planes(cap, max_ctx)
    _ref_append(ref, dk, dv, pr, dpos, T, cap, max_ctx)
    mk = dev(k)
    pm = _kv_planes(cap, max_ctx)
    cache = wz.kv_cache(pm["rkq"], pm["rks"], pm["rvq"], pm["rvs"], cap, max_ctx, pm["fkq"], pm["fks"], pm["fvq"],
                        pm["fvs"])
    wz.k_rope_kv_append(mk, dev(gam), dv, dc, ds, T, 2, 256, cache, rot_dims=64, eps=1e-6, w_offset=1.0,
                        d_base_pos=dpos)
    np.testing.assert_allclose(host(mk), host(dk), rtol=1e-5, atol=2e-6)
    for nm in ("rvq", "rvs", "fvq", "fvs"):
        assert np.array_equal(host(pm[nm]), host(pr[nm])), nm
    for q, sc in (("rkq", "rks"), ("fkq", "fks")):
        d = np.abs(host(pm[q]).astype(np.int32) - host(pr[q]).astype(np.int32))
        assert d.max() <= 1 and (d > 0).mean() < 2e-3
        assert np.abs(host(pm[sc]).astype(np.int32) - host(pr[sc]).astype(np.int32)).max() <= 1


def test_pin_ple_gate_and_conv(ref, orc, wz):
    """ple_gate_gv_multi and ple_conv_multi at the reference's widths (n_embd 2560, 4 streams,
    HCD 10240), with a carried history and per-token snapshots."""
    r = np.random.default_rng(212)
    T, n, hc = 12, 2560, 4
    k = r.standard_normal((T * hc, n)).astype(np.float32)
    q = r.standard_normal((T * hc, n)).astype(np.float32)
    q[3] = -k[3]
    v = r.standard_normal((T, n)).astype(np.float32)
    dk, dq, dv = dev(k), dev(q), dev(v)
    rg = torch.empty((T * hc, n), dtype=torch.float32, device=DEV)
    assert ref.ref_ple_gate_gv_multi(dk.data_ptr(), dq.data_ptr(), dv.data_ptr(), rg.data_ptr(), T, hc, n, sp()) == 0
    ref_gv = host(rg)
    np.testing.assert_allclose(orc.ple_gate_f32(k, q, v, T, n, hc), ref_gv, rtol=2e-6, atol=1e-7)
    mg = torch.empty_like(rg)
    wz.ple_gate_f32(dk, dq, dv, mg, T, n, hc)
    np.testing.assert_allclose(host(mg), ref_gv, rtol=2e-6, atol=1e-7)
    hcd = hc * n
    norm = r.standard_normal((T, hcd)).astype(np.float32)
    cw = (0.5 * r.standard_normal((hcd, 4))).astype(np.float32)
    hist = r.standard_normal((hcd, 9)).astype(np.float32)
    gv = r.standard_normal((T, hcd)).astype(np.float32)
    R = r.standard_normal((T, hcd)).astype(np.float32)
    dn, dcw, dgv = dev(norm), dev(cw), dev(gv)
    rR, rh = dev(R), dev(hist)
    rs = torch.zeros((T, hcd, 9), dtype=torch.float32, device=DEV)
    assert ref.ref_ple_conv_multi(dn.data_ptr(), dcw.data_ptr(), rh.data_ptr(), dgv.data_ptr(), rR.data_ptr(), hcd, T,
                                  rs.data_ptr(), sp()) == 0
    mR, mh = dev(R), dev(hist)
    ms = torch.zeros_like(rs)
    wz.ple_conv_f32(dn, dcw, mh, dgv, mR, T, hcd, hist_snaps=ms)
    np.testing.assert_allclose(host(mR), host(rR), rtol=1e-6, atol=1e-6)
    assert np.array_equal(host(mh), host(rh))
    assert np.array_equal(host(ms), host(rs))
    oR, oh, osn = orc.ple_conv_f32(norm, cw, hist, gv, R, T, hcd, snaps=True)
    np.testing.assert_allclose(oR, host(rR), rtol=2e-6, atol=2e-6)
    assert np.array_equal(oh, host(rh)) and np.array_equal(osn, host(rs))


def _tiny_groups(r, x):
    """Row 0 of x: Q8 groups whose max is so small that 127 / max overflows to infinity while max / 127
    is still above 0 (codes then +-127 for nonzero values and 0 for zeros, as __float2int_rn(+-inf)
    and of NaN clamp), at the finite edge of 127 / max, subnormal maxima whose max / 127 rounds to 0
    or not, tiny groups holding a NaN or an infinity, and 16-element halves of different sizes."""
    def grp(n, top):
        g = (r.uniform(-1, 1, n) * top).astype(np.float32)
        g[r.integers(0, n)] = np.float32(top)
        return g
    specs = [(1e-38, None), (3.0e-37, None), (4.0e-37, None), (1e-43, None), (5e-44, None),
             (1e-38, np.nan), (1e-38, np.inf), (1e-40, None)]
    for i, (top, special) in enumerate(specs):
        g = grp(32, top)
        g[5] = 0.0
        if special is not None:
            g[11] = special
        x[0, 32 * i:32 * i + 32] = g
    x[0, 256:272], x[0, 272:288] = grp(16, 1e-39), grp(16, 1.0)


def test_pin_quant_act(ref, orc, wz):
    """quant_act_multi with both outputs (the src/wzy_stage_v2.cuh:697 launch) at n_embd 2560, with
    the edge groups of _tiny_groups in row 0."""
    r = np.random.default_rng(213)
    T, cols = 16, 2560
    x = (3 * r.standard_normal((T, cols))).astype(np.float32)
    _tiny_groups(r, x)
    dx = dev(x)
    n = T * cols
    rq32, rq16 = torch.empty(n, dtype=torch.int8, device=DEV), torch.empty(n, dtype=torch.int8, device=DEV)
    rs32, rs16 = torch.empty(n // 32, device=DEV), torch.empty(n // 16, device=DEV)
    assert ref.ref_quant_act_multi(dx.data_ptr(), rq32.data_ptr(), rs32.data_ptr(), rq16.data_ptr(), rs16.data_ptr(),
                                   cols, T, sp()) == 0
    mq32, mq16 = torch.empty_like(rq32), torch.empty_like(rq16)
    ms32, ms16 = torch.empty_like(rs32), torch.empty_like(rs16)
    wz.quant_act_f32(dx, mq32, ms32, mq16, ms16, T, cols)
    o32, os32, o16, os16 = orc.quant_act_f32(x)
    for got, want, oracle in ((mq32, rq32, o32), (mq16, rq16, o16), (ms32, rs32, os32), (ms16, rs16, os16)):
        g, w = host(got), host(want)
        assert np.array_equal(g.view(np.uint8), w.view(np.uint8))
        assert np.array_equal(oracle.view(np.uint8), w.view(np.uint8))


@pytest.mark.parametrize("fmt", ["mxfp8", "nvfp4"])
def test_pin_swiglu_block_formats(ref, orc, wz, fmt):
    """SwiGLU straight to MXFP8 / NVFP4 equals the oracle's quantiser applied to the reference's own
    silu_mul_multi output (the same fp32 expression)."""
    r = np.random.default_rng(214)
    n = 640 * 64
    g = (2 * r.standard_normal(n)).astype(np.float32)
    u = r.standard_normal(n).astype(np.float32)
    dg, du = dev(g), dev(u)
    act = torch.empty(n, dtype=torch.float32, device=DEV)
    assert ref.ref_silu_mul_multi(dg.data_ptr(), du.data_ptr(), act.data_ptr(), n, sp()) == 0
    a = host(act)
    want_q, want_s = orc.quant_mxfp8(a) if fmt == "mxfp8" else orc.quant_nvfp4(a, 2.5)
    q = torch.empty(n if fmt == "mxfp8" else n // 2, dtype=torch.uint8, device=DEV)
    s = torch.empty(n // (32 if fmt == "mxfp8" else 16), dtype=torch.uint8, device=DEV)
    wz.swiglu_block(dg, du, q, s, fmt=fmt, global_scale=2.5)
    assert np.array_equal(host(q), want_q) and np.array_equal(host(s), want_s)


def test_pin_ple_fp8_gather_against_plesrc(ref, orc, wz, tmp_path):
    """The CUDA fp8 PLE gather against the reference's own PleSrc decode of the same GGUF table (rows
    named by the reference hash's constants over a small synthetic table): bit-exact."""
    r = np.random.default_rng(89)
    vocab = [2003 + 6 * i for i in range(16)]
    hsh = orc.PleFp8Hash(vocab=vocab)
    table = r.integers(0, 256, (hsh.rows, 160)).astype(np.uint8)
    table[:, 5], table[:, 6] = 0x7F, 0xFF
    path = tmp_path / "ple-fp8.gguf"
    orc.write_ple_gguf(path, table, 1.375)
    T = 96
    ids = r.integers(0, 248320, T).astype(np.int32)
    ids[11], ids[40] = 248044, -1
    prev = (5, 6)
    seq = list(prev) + [int(v) for v in ids]
    rows = [orc.ple_fp8_row(seq[t + 2], seq[t + 1], seq[t], h, hsh) for t in range(T) for h in range(16)]
    ref_rows, scale, _, _ = orc.ref_ple_src_rows(path, rows)
    out = torch.empty((T, 16 * 160), dtype=torch.float32, device=DEV)
    wz.ple_gather_fp8_f32(dev(table), 160, scale, wz.ple_fp8_hash(vocab=vocab), dev(ids), out, prev_ids=prev)
    assert np.array_equal(host(out).reshape(T * 16, 160).view(np.uint32), ref_rows.view(np.uint32))
