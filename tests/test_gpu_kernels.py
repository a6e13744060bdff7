"""GPU parity: every CUDA entry point against the CPU oracle on the same seeded inputs.

Tolerances (north star): gathers bit-exact; norms / activation / RoPE within 2 fp16 ulp of the
oracle (max-abs and max-rel reported in the assertion message). fp32-output variants: within
2e-6 relative + 2e-6 absolute of the oracle (fp32 reduction order, rsqrtf and __expf differ from
libm by a few fp32 ulp).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import ULP_TOL, assert_f16_close, assert_f32_in_f16_out_close

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def rng(seed):
    return np.random.default_rng(seed)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def f16n(r, shape, std=1.0, mean=0.0):
    return (r.standard_normal(shape) * std + mean).astype(np.float16)


@pytest.fixture(autouse=True)
def _faults_clear(wz):
    torch.cuda.set_device(0)
    wz.read_faults(clear=True)
    yield
    torch.cuda.synchronize()
    for fam in (wz.FAM_NORM, wz.FAM_HEAD_ROPE, wz.FAM_GDN):
        wz.set_kernel_variant(fam, wz.VARIANT_AUTO)


# The norm families have several kernel designs (direct, cp.async, CTA-wide rows, pair; a family
# without one falls back to its default); parity must hold for each.
@pytest.fixture(params=["direct", "async", "wide", "pair"])
def variant(request, wz):
    v = {"direct": wz.VARIANT_DIRECT, "async": wz.VARIANT_ASYNC,
         "wide": wz.VARIANT_WIDE, "pair": wz.VARIANT_PAIR}[request.param]
    for fam in (wz.FAM_NORM, wz.FAM_HEAD_ROPE, wz.FAM_GDN):
        wz.set_kernel_variant(fam, v)
    return request.param


# ---------------------------------------------------------------------------------------------
# residual add + RMSNorm
# ---------------------------------------------------------------------------------------------
@pytest.mark.parametrize("T,n", [(1, 2048), (3, 2048), (17, 2048), (4096, 2048), (5, 2560), (9, 24),
                                 (7, 5120), (3, 16384), (300, 1000)])
def test_add_rmsnorm_f16(wz, orc, T, n, variant):
    r = rng(T * 7 + n)
    x, res = f16n(r, (T, n)), f16n(r, (T, n))
    w = f16n(r, (n,), 0.02)
    y_ref, res_ref = orc.add_rmsnorm_f16(x, res, w, 1e-6, 1.0)
    dx, dres, dw = dev(x), dev(res), dev(w)
    dy = torch.empty_like(dres)
    wz.add_rmsnorm_f16(dx, dres, dw, dy, 1e-6, 1.0)
    assert np.array_equal(host(dres), res_ref), "residual must be fp16(x + residual) exactly"
    assert_f16_close(host(dy), y_ref, ULP_TOL, f"add_rmsnorm T={T} n={n}")
    assert wz.read_faults() == 0


def test_rmsnorm_without_add(wz, orc, variant):
    r = rng(3)
    T, n = 33, 2048
    res, w = f16n(r, (T, n)), f16n(r, (n,), 0.02, 1.0)
    y_ref, _ = orc.add_rmsnorm_f16(None, res, w, 1e-6, 0.0)
    dres = dev(res)
    dy = torch.empty_like(dres)
    wz.add_rmsnorm_f16(None, dres, dev(w), dy, 1e-6, 0.0)
    assert np.array_equal(host(dres), res)
    assert_f16_close(host(dy), y_ref, ULP_TOL, "rmsnorm only")


@pytest.mark.parametrize("T,n", [(19, 2560), (19, 6144), (700, 2056), (700, 6144), (1000, 2560)])
@pytest.mark.parametrize("hc,with_inj,out16", [(1, False, False), (4, True, False), (4, True, True), (4, False, True)])
def test_gr_norm_f32_hyper_connection(wz, orc, T, n, hc, with_inj, out16, variant):
    """19 tokens take the row-per-CTA design, 700+ the token design with 4 streams (hc = 4); n 2056: a
    partly idle last warp; 6144: two vectors per thread; 1000 tokens: several tokens per CTA, so the
    parity-buffered partial sums are reused."""
    r = rng(11 + hc + n)
    R = r.standard_normal((T * hc, n)).astype(np.float32)
    bo = r.standard_normal((T, n)).astype(np.float32)
    inj = r.standard_normal((T * hc,)).astype(np.float32) if with_inj else None
    w = (1 + 0.02 * r.standard_normal((hc, n))).astype(np.float32)
    xn_ref, xh_ref, R_ref = orc.gr_norm_f32(R, w, bo, inj, T, n, hc)
    dR = dev(R)
    dxn = torch.empty((T * hc, n), dtype=torch.float16 if out16 else torch.float32, device=DEV)
    wz.gr_norm_f32(dR, dev(w), dev(bo), dev(inj) if inj is not None else None, dxn, T, n, hc)
    np.testing.assert_allclose(host(dR), R_ref, rtol=1e-6, atol=1e-6)
    if out16:
        assert_f32_in_f16_out_close(host(dxn), xn_ref, 2e-6, "gr_norm f16 out")
    else:
        np.testing.assert_allclose(host(dxn), xn_ref, rtol=2e-6, atol=2e-6)


# ---------------------------------------------------------------------------------------------
# per-head norm + RoPE
# ---------------------------------------------------------------------------------------------
def _rope_tab(orc, rows, rot, theta=1e7):
    c, s = orc.rope_table(rows, rot, theta)
    return c, s, dev(c), dev(s)


@pytest.mark.parametrize("T", [1, 5, 4096, 20000])
def test_qk_norm_rope_fused_baseline_shape(wz, orc, T, variant):
    """q [T,16,256], k [T,2,256], (1+w) gammas, rot 64, theta 1e7, positions 0..T-1.
    20,000 tokens reach the long-call shape of the default design (one 18-head item per token)."""
    r = rng(100 + T)
    hd, rot = 256, 64
    q, k = f16n(r, (T, 16, hd)), f16n(r, (T, 2, hd))
    gq, gk = f16n(r, (hd,), 0.02), f16n(r, (hd,), 0.02)
    c, s, dc, ds = _rope_tab(orc, T, rot)
    q_ref = orc.head_norm_rope(q.reshape(-1), gq, c, s, T, 16, hd, hd, 16 * hd, rot, 1e-6, 1.0, 0)
    k_ref = orc.head_norm_rope(k.reshape(-1), gk, c, s, T, 2, hd, hd, 2 * hd, rot, 1e-6, 1.0, 0)
    dq, dk = dev(q), dev(k)
    dgq, dgk = dev(gq), dev(gk)
    wz.qk_norm_rope_f16(wz.head_tensor(dq, dgq, 16, hd, 16 * hd), wz.head_tensor(dk, dgk, 2, hd, 2 * hd), dc, ds, T,
                        hd, rot, 1e-6, 1.0)
    assert_f16_close(host(dq).reshape(-1), q_ref, ULP_TOL, "q")
    assert_f16_close(host(dk).reshape(-1), k_ref, ULP_TOL, "k")
    assert wz.read_faults() == 0


@pytest.mark.parametrize("hd,rot", [(256, 0), (256, 16), (256, 128), (256, 256), (128, 64), (64, 32), (128, 48)])
def test_head_norm_rope_dims(wz, orc, hd, rot, variant):
    r = rng(hd * 1000 + rot)
    T, H = 13, 3
    x = f16n(r, (T, H, hd))
    g = f16n(r, (hd,), 0.02)
    rows = 64
    c, s, dc, ds = _rope_tab(orc, rows, max(rot, 2))
    want = orc.head_norm_rope(x.reshape(-1), g, c, s, T, H, hd, hd, H * hd, rot, 1e-6, 1.0, 40)
    d = dev(x)
    base = torch.tensor([30], dtype=torch.int32, device=DEV)
    wz.head_norm_rope(d, dev(g), dc, ds, T, H, hd, hd, H * hd, rot, 1e-6, 1.0, d_base_pos=base, pos_offset=10)
    assert_f16_close(host(d).reshape(-1), want, ULP_TOL, f"hd={hd} rot={rot}")


def test_head_norm_rope_strided_heads_f32(wz, orc, variant):
    """The reference's own q layout: heads interleaved with the gate (head_stride = 2*HD), fp32."""
    r = rng(77)
    T, H, hd, rot = 6, 24, 256, 64
    buf = r.standard_normal((T, H, 2 * hd)).astype(np.float32)
    g = (1 + 0.02 * r.standard_normal(hd)).astype(np.float32)
    c, s, dc, ds = _rope_tab(orc, 16, rot)
    want = orc.head_norm_rope(buf.reshape(-1), g, c, s, T, H, hd, 2 * hd, 2 * H * hd, rot, 1e-6, 0.0, 3)
    d = dev(buf)
    wz.head_norm_rope(d, dev(g), dc, ds, T, H, hd, 2 * hd, 2 * H * hd, rot, 1e-6, 0.0, pos_offset=3)
    got = host(d).reshape(-1)
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5)
    # the gate halves are untouched
    assert np.array_equal(got.reshape(T, H, 2 * hd)[..., hd:], buf[..., hd:])


def test_head_norm_rope_position_out_of_table(wz, orc, variant):
    """Positions past the table are flagged (fault bit), not read; those heads stay un-rotated."""
    r = rng(5)
    T, H, hd, rot = 8, 2, 128, 64
    x = f16n(r, (T, H, hd))
    g = f16n(r, (hd,), 0.02)
    c, s, dc, ds = _rope_tab(orc, 4, rot)
    want = orc.head_norm_rope(x.reshape(-1), g, c, s, T, H, hd, hd, H * hd, rot, 1e-6, 1.0, 0)
    d = dev(x)
    wz.head_norm_rope(d, dev(g), dc, ds, T, H, hd, hd, H * hd, rot, 1e-6, 1.0)
    assert_f16_close(host(d).reshape(-1), want, ULP_TOL, "pos range")
    assert wz.read_faults() & wz.FAULT_POS_RANGE


# ---------------------------------------------------------------------------------------------
# GDN gated norm
# ---------------------------------------------------------------------------------------------
@pytest.mark.parametrize("T,H,hd,mode", [(4096, 32, 128, 0), (7, 32, 128, 1), (3, 48, 128, 0), (5, 8, 64, 0),
                                         (5, 4, 256, 1), (2, 96, 128, 0), (3, 5, 128, 0)])
def test_gdn_gated_norm_f16(wz, orc, T, H, hd, mode, variant):
    r = rng(T + H + hd + mode)
    o, z = f16n(r, (T, H, hd)), f16n(r, (T, H, hd))
    gm = f16n(r, (hd,), 0.02, 1.0)
    want = orc.gdn_gated_norm(o, z, gm, T, H, hd, 1e-6, 0.0, mode)
    dy = torch.empty((T, H, hd), dtype=torch.float16, device=DEV)
    wz.gdn_gated_norm(dev(o), dev(z), dev(gm), dy, T, H, hd, 1e-6, 0.0, mode)
    assert_f16_close(host(dy), want, ULP_TOL, f"gdn T={T} H={H} hd={hd} mode={mode}")


def test_gdn_gated_norm_f32_in(wz, orc, variant):
    r = rng(9)
    T, H, hd = 21, 48, 128
    o = r.standard_normal((T, H, hd)).astype(np.float32)
    z = r.standard_normal((T, H, hd)).astype(np.float32)
    gm = (1 + 0.02 * r.standard_normal(hd)).astype(np.float32)
    want = orc.gdn_gated_norm(o, z, gm, T, H, hd, 1e-6, 0.0, 0).astype(np.float16)
    dy = torch.empty((T, H, hd), dtype=torch.float16, device=DEV)
    wz.gdn_gated_norm(dev(o), dev(z), dev(gm), dy, T, H, hd, 1e-6, 0.0, 0)
    assert_f16_close(host(dy), want, ULP_TOL, "gdn f32 in")


# ---------------------------------------------------------------------------------------------
# SwiGLU
# ---------------------------------------------------------------------------------------------
@pytest.mark.parametrize("rows,cols", [(4096 * 11, 512), (1, 8), (3, 640), (1001, 512)])
def test_swiglu_f16(wz, orc, rows, cols):
    r = rng(rows + cols)
    g, u = f16n(r, (rows, cols)), f16n(r, (rows, cols))
    want = orc.swiglu(g, u)
    dout = torch.empty((rows, cols), dtype=torch.float16, device=DEV)
    wz.swiglu(dev(g), dev(u), dout)
    assert_f16_close(host(dout), want, ULP_TOL, f"swiglu {rows}x{cols}")


def test_swiglu_f32_and_interleaved(wz, orc):
    r = rng(4)
    g = r.standard_normal(8 * 1234).astype(np.float32) * 4
    u = r.standard_normal(8 * 1234).astype(np.float32)
    out = torch.empty(g.size, dtype=torch.float32, device=DEV)
    wz.swiglu(dev(g), dev(u), out)
    np.testing.assert_allclose(host(out), orc.swiglu(g, u), rtol=2e-6, atol=2e-6)
    T, nff = 77, 640
    gu16 = f16n(r, (T, 2 * nff))
    o16 = torch.empty((T, nff), dtype=torch.float16, device=DEV)
    wz.swiglu_interleaved(dev(gu16), o16, T, nff)
    assert_f16_close(host(o16), orc.swiglu_interleaved(gu16, T, nff), ULP_TOL, "interleaved f16")
    gu32 = r.standard_normal((T, 2 * nff)).astype(np.float32)
    o16b = torch.empty((T, nff), dtype=torch.float16, device=DEV)
    wz.swiglu_interleaved(dev(gu32), o16b, T, nff)
    want = orc.swiglu_interleaved(gu32, T, nff).astype(np.float16)
    assert_f16_close(host(o16b), want, ULP_TOL, "interleaved f32->f16")


# ---------------------------------------------------------------------------------------------
# gathers (bit-exact)
# ---------------------------------------------------------------------------------------------
def test_embed_gather_baseline_shape(wz, orc):
    """fp16 table [151936, 2048] ~N(0,0.02), 4096 uniform ids."""
    gen = torch.Generator(device=DEV).manual_seed(31)
    table = (torch.randn((151936, 2048), generator=gen, device=DEV) * 0.02).half()
    ids = rng(32).integers(0, 151936, 4096).astype(np.int32)
    out = torch.empty((4096, 2048), dtype=torch.float16, device=DEV)
    cnt = torch.zeros(1, dtype=torch.int32, device=DEV)
    wz.embed_gather_f16(table, dev(ids), out, wz.OOB_CLAMP, cnt)
    want, bad = orc.embed_gather_rows(host(table), ids, 0)
    assert np.array_equal(host(out).view(np.uint16), want.view(np.uint16))
    assert int(host(cnt)[0]) == bad == 0


@pytest.mark.parametrize("policy", [0, 1])
def test_embed_gather_out_of_range(wz, orc, policy):
    r = rng(8)
    table = f16n(r, (1000, 72))
    ids = np.array([0, 999, -5, 1000, 123456, 17, -1], dtype=np.int32)
    out = torch.empty((ids.size, 72), dtype=torch.float16, device=DEV)
    cnt = torch.zeros(1, dtype=torch.int32, device=DEV)
    wz.embed_gather_f16(dev(table), dev(ids), out, policy, cnt)
    want, bad = orc.embed_gather_rows(table, ids, policy)
    assert np.array_equal(host(out).view(np.uint16), want.view(np.uint16))
    assert int(host(cnt)[0]) == bad == 4


def test_embed_gather_bf16_f32(wz, orc):
    r = rng(10)
    bits = r.integers(0, 65536, (5000, 2560), dtype=np.uint16)
    ids = r.integers(-10, 5010, 97).astype(np.int32)
    out = torch.empty((97, 2560), dtype=torch.float32, device=DEV)
    wz.embed_gather_bf16_f32(dev(bits.view(np.int16)), dev(ids), out, wz.OOB_CLAMP)
    want, _ = orc.embed_gather_bf16_f32(bits, ids, 0)
    assert np.array_equal(host(out).view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("row_bytes", [16, 48, 160, 4112])
@pytest.mark.parametrize("policy", [0, 1])
def test_embed_gather_rows_any_width(wz, orc, row_bytes, policy):
    """The generic byte-row gather at several row widths (one 16-byte chunk to 257), with out-of-range
    ids under both policies and the device counter of out-of-range ids."""
    r = rng(row_bytes + policy)
    vocab = 3001
    table = r.integers(0, 256, (vocab, row_bytes)).astype(np.uint8)
    ids = r.integers(0, vocab, 517).astype(np.int32)
    ids[[0, 100, 516]] = [-7, vocab, 1 << 30]
    want, bad = orc.embed_gather_rows(table, ids, policy)
    out = torch.empty((ids.size, row_bytes), dtype=torch.uint8, device=DEV)
    cnt = torch.zeros(1, dtype=torch.int32, device=DEV)
    wz.embed_gather_rows(dev(table), dev(ids), out, oob_policy=policy, oob_count=cnt)
    assert np.array_equal(host(out), want)
    assert int(host(cnt)[0]) == bad == 3


@pytest.mark.parametrize("variant", [0, 1])
def test_ple_gather_baseline_shape(wz, orc, variant):
    """configs[3] PLE: 16 fp16 tables [2^20, 128] ~N(0,0.02), 4096 uniform ids -> [4096, 2048]."""
    gen = torch.Generator(device=DEV).manual_seed(41)
    tables = [(torch.randn((1 << 20, 128), generator=gen, device=DEV) * 0.02).half() for _ in range(16)]
    ids = rng(42).integers(0, 151936, 4096).astype(np.int32)
    out = torch.empty((4096, 2048), dtype=torch.float16, device=DEV)
    wz.ple_gather_f16(tables, dev(ids), out, prev_ids=None, hash_variant=variant)
    want = orc.ple_gather_f16([host(t) for t in tables], ids, None, 248044, variant)
    assert np.array_equal(host(out).view(np.uint16), want.view(np.uint16))


def test_ple_gather_history_and_eos(wz, orc):
    r = rng(12)
    tables = [f16n(r, (4099, 64)) for _ in range(5)]  # rows not a power of two
    ids = np.array([5, 248044, 7, 8, -1, 9, 10, 11], dtype=np.int32)
    for prev in [None, (1, 2), (248044, 3), (4, -1)]:
        out = torch.empty((ids.size, 5 * 64), dtype=torch.float16, device=DEV)
        wz.ple_gather_f16([dev(t) for t in tables], dev(ids), out, prev_ids=prev)
        want = orc.ple_gather_f16(tables, ids, prev, 248044, 0)
        assert np.array_equal(host(out).view(np.uint16), want.view(np.uint16)), prev


# ---------------------------------------------------------------------------------------------
# run-to-run determinism and shard equivalence (no collective: shards are independent)
# ---------------------------------------------------------------------------------------------
def test_bitwise_deterministic(wz):
    r = rng(13)
    T, n = 1024, 2048
    x, res, w = f16n(r, (T, n)), f16n(r, (T, n)), f16n(r, (n,), 0.02)
    outs = []
    for _ in range(2):
        dres, dy = dev(res), torch.empty((T, n), dtype=torch.float16, device=DEV)
        wz.add_rmsnorm_f16(dev(x), dres, dev(w), dy)
        outs.append(host(dy).view(np.uint16).copy())
    assert np.array_equal(outs[0], outs[1])


def test_layer_bundles_match_oracle(wz, orc):
    """The executor's bundle entry points (wzyb_attn_prep_f16: add+RMSNorm then q/k norm+RoPE;
    wzyb_act_f16: SwiGLU over the expert rows then the GDN gated norm) -- the calls the end-to-end
    measurement makes -- at the configs' shapes, against the oracle."""
    import ctypes

    r = rng(91)
    T, n, hd, rot, off = 300, 2048, 256, 64, 17
    x, res = f16n(r, (T, n)), f16n(r, (T, n))
    w = f16n(r, (n,), 0.02)
    q, k = f16n(r, (T, 16, hd)), f16n(r, (T, 2, hd))
    gq, gk = f16n(r, (hd,), 0.02), f16n(r, (hd,), 0.02)
    c, s, dc, ds = _rope_tab(orc, T + off, rot)
    dx, dres, dw, dy = dev(x), dev(res), dev(w), torch.empty((T, n), dtype=torch.float16, device=DEV)
    dq, dk, dgq, dgk = dev(q), dev(k), dev(gq), dev(gk)
    a = wz.AttnPrepArgs()
    a.x, a.residual, a.norm_weight, a.normed, a.hidden = dx.data_ptr(), dres.data_ptr(), dw.data_ptr(), dy.data_ptr(), n
    a.q = wz.head_tensor(dq, dgq, 16, hd, 16 * hd)
    a.k = wz.head_tensor(dk, dgk, 2, hd, 2 * hd)
    a.head_dim, a.rot_dims = hd, rot
    a.cos_tab, a.sin_tab, a.table_rows = dc.data_ptr(), ds.data_ptr(), T + off
    a.d_base_pos, a.pos_offset, a.eps, a.w_offset = None, off, 1e-6, 1.0
    wz.call("wzyb_attn_prep_f16", ctypes.byref(a), T, wz._stream())
    y_ref, res_ref = orc.add_rmsnorm_f16(x, res, w, 1e-6, 1.0)
    assert np.array_equal(host(dres), res_ref)
    assert_f16_close(host(dy), y_ref, ULP_TOL, "bundle add+rmsnorm")
    q_ref = orc.head_norm_rope(q.reshape(-1), gq, c, s, T, 16, hd, hd, 16 * hd, rot, 1e-6, 1.0, off)
    k_ref = orc.head_norm_rope(k.reshape(-1), gk, c, s, T, 2, hd, hd, 2 * hd, rot, 1e-6, 1.0, off)
    assert_f16_close(host(dq).reshape(-1), q_ref, ULP_TOL, "bundle q")
    assert_f16_close(host(dk).reshape(-1), k_ref, ULP_TOL, "bundle k")

    rows, ffn, H, ghd = 11 * T, 512, 32, 128
    g, u = f16n(r, (rows, ffn), 2.0), f16n(r, (rows, ffn))
    o, z = f16n(r, (T, H, ghd)), f16n(r, (T, H, ghd))
    gm = f16n(r, (ghd,), 0.02, 1.0)
    dg, du, dact = dev(g), dev(u), torch.empty((rows, ffn), dtype=torch.float16, device=DEV)
    do, dz, dgm, dgy = dev(o), dev(z), dev(gm), torch.empty((T, H, ghd), dtype=torch.float16, device=DEV)
    b = wz.ActArgs()
    b.gate, b.up, b.act, b.act_rows, b.ffn = dg.data_ptr(), du.data_ptr(), dact.data_ptr(), rows, ffn
    b.o, b.z, b.gdn_gamma, b.gdn_out = do.data_ptr(), dz.data_ptr(), dgm.data_ptr(), dgy.data_ptr()
    b.gdn_heads, b.gdn_head_dim, b.eps, b.gdn_w_offset, b.gate_mode = H, ghd, 1e-6, 0.0, wz.GATE_SIGMOID
    wz.call("wzyb_act_f16", ctypes.byref(b), T, wz._stream())
    assert_f16_close(host(dact), orc.swiglu(g, u), ULP_TOL, "bundle swiglu")
    assert_f16_close(host(dgy), orc.gdn_gated_norm(o, z, gm, T, H, ghd, 1e-6, 0.0, 0), ULP_TOL, "bundle gdn")
    assert wz.read_faults() == 0


@pytest.mark.parametrize("shards", [2, 8])
def test_sharded_equals_unsharded(wz, orc, shards):
    """Each shard gets its row slice, a RoPE pos_offset = its first row, and a 2-id PLE halo."""
    r = rng(14)
    T, hd = 600, 256
    q = f16n(r, (T, 4, hd))
    gq = f16n(r, (hd,), 0.02)
    c, s, dc, ds = _rope_tab(orc, T, 64)
    full = dev(q)
    wz.head_norm_rope(full, dev(gq), dc, ds, T, 4, hd, hd, 4 * hd, 64, 1e-6, 1.0)
    tables = [dev(f16n(r, (1 << 12, 128))) for _ in range(16)]
    ids = r.integers(0, 151936, T).astype(np.int32)
    ple_full = torch.empty((T, 2048), dtype=torch.float16, device=DEV)
    wz.ple_gather_f16(tables, dev(ids), ple_full, prev_ids=(11, 12))
    parts, ple_parts = [], []
    for k in range(shards):
        r0, n = wz.shard_rows(T, shards, k)
        part = dev(q[r0:r0 + n])
        wz.head_norm_rope(part, dev(gq), dc, ds, n, 4, hd, hd, 4 * hd, 64, 1e-6, 1.0, pos_offset=r0)
        parts.append(host(part))
        halo = wz.ple_halo(ids, r0, (11, 12))
        po = torch.empty((n, 2048), dtype=torch.float16, device=DEV)
        wz.ple_gather_f16(tables, dev(ids[r0:r0 + n]), po, prev_ids=halo)
        ple_parts.append(host(po))
    assert np.array_equal(np.concatenate(parts).view(np.uint16), host(full).view(np.uint16))
    assert np.array_equal(np.concatenate(ple_parts).view(np.uint16), host(ple_full).view(np.uint16))


def test_device_rope_table_close_to_host(wz, orc):
    rows = 262144
    c, s = orc.rope_table(rows, 64, 1e7)
    dc = torch.empty((rows, 32), dtype=torch.float32, device=DEV)
    ds = torch.empty_like(dc)
    wz.rope_table(dc, ds, rows, 64, 1e7)
    gc, gs = host(dc), host(ds)
    # CUDA's fp64 pow/cos/sin vs libm, both rounded to fp32: the angles agree to ~1e-16 relative, so
    # the values agree to ~1e-10 absolute (near a zero crossing that is many fp32 ulp of a tiny value)
    assert np.abs(gc - c).max() <= 1.2e-7 and np.abs(gs - s).max() <= 1.2e-7  # <= 2 fp32 ulp at 1.0
    assert (gc == c).mean() > 0.999 and (gs == s).mean() > 0.999


# ---------------------------------------------------------------------------------------------
# Q8_0 side outputs (decode path)
# ---------------------------------------------------------------------------------------------
def _q8_close(q_got, s_got, q_want, s_want, what):
    dq = np.abs(q_got.astype(np.int32) - q_want.astype(np.int32))
    # fp32 inputs to the rounding differ by a few ulp (reduction order, exp): a code may sit on the
    # other side of a .5 boundary, never further
    assert dq.max() <= 1 and (dq > 0).mean() < 1e-3, f"{what}: max {dq.max()} frac {(dq > 0).mean()}"
    np.testing.assert_allclose(s_got, s_want, rtol=4e-6, atol=0)


@pytest.mark.parametrize("T,n,hc", [(1, 2560, 4), (8, 2560, 4), (5, 2048, 1), (3, 96, 2), (7, 2080, 4), (3, 6144, 4),
                                    (700, 2560, 4), (650, 2080, 4), (600, 6144, 4)])
def test_gr_norm_q8_f32(wz, orc, T, n, hc):
    r = rng(T * n + hc)
    R = r.standard_normal((T * hc, n)).astype(np.float32)
    bo = r.standard_normal((T, n)).astype(np.float32)
    inj = r.standard_normal(T * hc).astype(np.float32)
    w = (1 + 0.02 * r.standard_normal((hc, n))).astype(np.float32)
    xn_ref, q_ref, s_ref, R_ref = orc.gr_norm_q8_f32(R, w, bo, inj, T, n, hc)
    dR, dxn = dev(R), torch.empty((T * hc, n), dtype=torch.float32, device=DEV)
    dq = torch.empty((T * hc, n), dtype=torch.int8, device=DEV)
    ds = torch.empty((T * hc, n // 32), dtype=torch.float32, device=DEV)
    wz.gr_norm_q8_f32(dR, dev(w), dev(bo), dev(inj), dxn, dq, ds, T, n, hc)
    np.testing.assert_allclose(host(dR), R_ref, rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(host(dxn), xn_ref, rtol=2e-6, atol=2e-6)
    _q8_close(host(dq), host(ds), q_ref, s_ref, "gr_norm q8")


@pytest.mark.parametrize("n", [32, 640 * 8, 45056 * 512])
def test_swiglu_q8_f32(wz, orc, n):
    r = rng(n % 1000)
    g = (2 * r.standard_normal(n)).astype(np.float32)
    u = r.standard_normal(n).astype(np.float32)
    q_ref, s_ref = orc.swiglu_q8_f32(g, u)
    dq = torch.empty(n, dtype=torch.int8, device=DEV)
    ds = torch.empty(n // 32, dtype=torch.float32, device=DEV)
    wz.swiglu_q8_f32(dev(g), dev(u), dq, ds)
    _q8_close(host(dq), host(ds), q_ref, s_ref, "swiglu q8")


# ---------------------------------------------------------------------------------------------
# multi-stream residual: gated write, stream mixing, scaled SiLU
# ---------------------------------------------------------------------------------------------
@pytest.mark.parametrize("T,n,hc,with_inj", [(1, 2560, 4, True), (37, 2560, 4, True), (5, 2048, 1, False),
                                             (3, 24, 3, True), (4096, 2048, 1, False)])
def test_gr_write_f32(wz, orc, T, n, hc, with_inj):
    r = rng(T + n + hc)
    R = r.standard_normal((T * hc, n)).astype(np.float32)
    blk = r.standard_normal((T, n)).astype(np.float32)
    inj = r.standard_normal(T * hc).astype(np.float32) if with_inj else None
    want = orc.gr_write_f32(R, blk, inj, T, n, hc)
    dR = dev(R)
    wz.gr_write_f32(dR, dev(blk), dev(inj) if inj is not None else None, T, n, hc)
    got = host(dR)
    if with_inj:  # __expf in the gate: a few fp32 ulp
        np.testing.assert_allclose(got, want, rtol=1e-6, atol=1e-6)
    else:  # gate 1.0: fma(b, 1, R) is the exact sum
        assert np.array_equal(got, want)


@pytest.mark.parametrize("T,n,hc", [(1, 2560, 4), (19, 2560, 4), (4096, 2048, 4), (7, 64, 3), (5, 128, 1)])
def test_hc_mix(wz, orc, T, n, hc):
    r = rng(T * 3 + n + hc)
    xn = f16n(r, (T, hc, n))
    gg = f16n(r, (T, hc, n), 2.0)
    m32_ref, m16_ref = orc.hc_mix(xn, gg, T, n, hc)
    d32 = torch.empty((T, n), dtype=torch.float32, device=DEV)
    d16 = torch.empty((T, n), dtype=torch.float16, device=DEV)
    dx, dg = dev(xn), dev(gg)
    wz.hc_mix(dx, dg, d32, d16, T, n, hc)
    np.testing.assert_allclose(host(d32), m32_ref, rtol=2e-6, atol=2e-6)
    assert_f16_close(host(d16), m16_ref, ULP_TOL, "hc_mix fp16 out")
    # either output alone
    e16 = torch.empty_like(d16)
    wz.hc_mix(dx, dg, None, e16, T, n, hc)
    assert np.array_equal(host(e16), host(d16))
    # fp32 inputs (the fp32 twin)
    x32, g32 = xn.astype(np.float32), gg.astype(np.float32)
    f32 = torch.empty((T, n), dtype=torch.float32, device=DEV)
    wz.hc_mix(dev(x32), dev(g32), f32, None, T, n, hc)
    np.testing.assert_allclose(host(f32), orc.hc_mix(x32, g32, T, n, hc), rtol=2e-6, atol=2e-6)


@pytest.mark.parametrize("n", [8, 4096 * 320, 262144 * 320])
def test_silu_scale_f16(wz, orc, n):
    r = rng(n % 977)
    lo = (4 * r.standard_normal(n)).astype(np.float32)
    want = orc.silu_scale_f16(lo, 0.25)
    out = torch.empty(n, dtype=torch.float16, device=DEV)
    wz.silu_scale_f16(dev(lo), out, 0.25)
    assert_f16_close(host(out), want, ULP_TOL, "silu_scale")


# ---------------------------------------------------------------------------------------------
# INT8 KV append (alone, and fused after k's norm + RoPE)
# ---------------------------------------------------------------------------------------------
_KV_PLANES = ["rkq", "rks", "rvq", "rvs", "fkq", "fks", "fvq", "fvs"]


def _kv_seeded(orc, r, cap, max_ctx, kvd, full):
    """Oracle cache pre-filled with random bytes (untouched cells must keep them) + its device copy."""
    c = orc.KvCache(cap, max_ctx, kvd, full)
    for nm in _KV_PLANES[: 8 if full else 4]:
        a = getattr(c, nm)
        a[...] = r.integers(0, 256 if a.dtype == np.int8 else 65536, a.shape).astype(a.dtype)
    d = {nm: dev(getattr(c, nm).view(np.int16) if nm.endswith("s") else getattr(c, nm))
         for nm in _KV_PLANES[: 8 if full else 4]}
    return c, d


def _kv_desc(wz, d, cap, max_ctx, full):
    return wz.kv_cache(d["rkq"], d["rks"], d["rvq"], d["rvs"], cap, max_ctx, *(
        (d["fkq"], d["fks"], d["fvq"], d["fvs"]) if full else ()))


def _kv_host(d, nm):
    a = host(d[nm])
    return a.view(np.uint16) if nm.endswith("s") else a


@pytest.mark.parametrize("T,heads,hd,base,cap,max_ctx,full", [
    (7, 2, 256, 100, 64, 200, True), (300, 2, 256, 4000, 8200, 9000, True), (50, 4, 128, -5, 16, 40, False),
    (4096, 2, 256, 0, 32768, 8192, True), (9, 3, 64, 1, 16, 64, True), (1, 2, 256, 8191, 32768, 8192, True)])
def test_kv_append_int8_f32(wz, orc, T, heads, hd, base, cap, max_ctx, full):
    r = rng(T + heads + cap)
    kvd = heads * hd
    k = r.standard_normal((T, kvd)).astype(np.float32)
    v = (3 * r.standard_normal((T, kvd))).astype(np.float32)
    v[0, :64] = 0.0
    c, d = _kv_seeded(orc, r, cap, max_ctx, kvd, full)
    orc.kv_append_int8_f32(k, v, T, kvd, base, c)
    bp = torch.tensor([base - 3], dtype=torch.int32, device=DEV)  # device base + pos_offset 3
    wz.kv_append_int8_f32(dev(k), dev(v), T, heads, hd, _kv_desc(wz, d, cap, max_ctx, full), d_base_pos=bp,
                          pos_offset=3)
    for nm in _KV_PLANES[: 8 if full else 4]:
        assert np.array_equal(_kv_host(d, nm), getattr(c, nm)), nm


def test_kv_append_codes_at_rounding_boundaries(wz, orc):
    """The INT8 codes are rint(x / d) of the correctly rounded quotient. Values are placed on and one or
    two fp32 ulps either side of every half-integer multiple (n + 0.5) * d of their group's scale, and
    on the integers, where a quotient off by one ulp would change the code; bit-exact against the
    oracle's IEEE division."""
    r = rng(4242)
    T, heads, hd = 2048, 2, 256
    kvd = heads * hd
    groups = T * kvd // 64
    amax = (np.exp(r.uniform(-12, 6, groups)) * np.where(r.random(groups) < 0.5, -1, 1)).astype(np.float32)
    d = (np.abs(amax) / np.float32(127)).astype(np.float32).astype(np.float16).astype(np.float32)
    n = r.integers(-127, 127, (groups, 63)).astype(np.float64)
    half = r.random((groups, 63)) < 0.8
    x = ((n + np.where(half, 0.5, 0.0)) * d[:, None].astype(np.float64)).astype(np.float32)
    step = r.integers(-2, 3, (groups, 63))
    x = np.where(step > 0, np.nextafter(x, np.float32(np.inf)), np.where(step < 0, np.nextafter(x, np.float32(-np.inf)), x))
    x = np.where(np.abs(step) == 2, np.where(step > 0, np.nextafter(x, np.float32(np.inf)),
                                             np.nextafter(x, np.float32(-np.inf))), x).astype(np.float32)
    grp = np.concatenate([amax[:, None], x], axis=1)
    idx = np.argsort(r.random((groups, 64)), axis=1)
    grp = np.take_along_axis(grp, idx, axis=1)
    k = grp.reshape(T, kvd).astype(np.float32)
    v = np.ascontiguousarray(k[::-1])
    c, dd = _kv_seeded(orc, r, T, T, kvd, True)
    orc.kv_append_int8_f32(k, v, T, kvd, 0, c)
    wz.kv_append_int8_f32(dev(k), dev(v), T, heads, hd, _kv_desc(wz, dd, T, T, True))
    for nm in _KV_PLANES:
        assert np.array_equal(_kv_host(dd, nm), getattr(c, nm)), nm


def test_kv_append_scales_at_fp16_ties(wz, orc):
    """The fp16 scale is fp16(max / 127) of the correctly rounded fp32 quotient (the kernel computes it
    without a divide). Group maxima on and one fp32 ulp either side of 127 times every tie point
    between adjacent positive fp16 values, subnormal scales included, with the group's other values
    spread below the max: scales and codes bit-exact against the oracle's IEEE division."""
    r = rng(4545)
    vals = np.arange(0, 0x7C00, dtype=np.uint16).view(np.float16).astype(np.float64)
    ties = (vals[:-1] + vals[1:]) / 2
    top = (127.0 * ties).astype(np.float32)
    top = np.concatenate([np.nextafter(top, np.float32(0)), top, np.nextafter(top, np.float32(np.inf))])
    heads, hd = 2, 256
    kvd = heads * hd
    T = -(-top.size * 64 // kvd)
    groups = T * kvd // 64
    top = np.concatenate([top, r.choice(top, groups - top.size)])
    grp = (r.uniform(-1, 1, (groups, 64)) * top[:, None]).astype(np.float32)
    grp[np.arange(groups), r.integers(0, 64, groups)] = np.where(r.random(groups) < 0.5, -top, top)
    k = grp.reshape(T, kvd)
    v = np.ascontiguousarray(k[::-1])
    c, dd = _kv_seeded(orc, r, T, T, kvd, True)
    orc.kv_append_int8_f32(k, v, T, kvd, 0, c)
    wz.kv_append_int8_f32(dev(k), dev(v), T, heads, hd, _kv_desc(wz, dd, T, T, True))
    for nm in _KV_PLANES:
        assert np.array_equal(_kv_host(dd, nm), getattr(c, nm)), nm


def test_kv_append_codes_non_finite(wz, orc):
    """Groups holding NaN or an infinity take the scalar conversion: NaN codes are 0 (as
    __float2int_rn), an infinite group max gives an infinite scale whose codes are 0, and the other
    lanes of such groups keep their own codes; bit-exact against the oracle."""
    r = rng(4343)
    T, heads, hd = 64, 2, 256
    kvd = heads * hd
    k = r.standard_normal((T, kvd)).astype(np.float32)
    v = (3 * r.standard_normal((T, kvd))).astype(np.float32)
    k[1, 5], k[2, 70], k[3, 130] = np.nan, np.inf, -np.inf
    v[4, 0], v[5, 63], v[6, 64] = np.nan, np.inf, np.nan
    k[7, 200:210] = np.nan
    # finite groups whose scale max/127 is at fp16's largest value, at the tie that rounds it to
    # infinity, and past it (fp32 inputs only): an infinite scale's codes are all 0
    for (row, g0), top in zip([(8, 64), (9, 128), (10, 192), (11, 256), (12, 0)],
                              [127.0 * 65504.0, 127.0 * 65520.0, 1e7, 3e38, 127.0 * 65519.0]):
        grp = r.standard_normal(64).astype(np.float32)
        grp *= np.float32(top / 4.0 / np.abs(grp).max())
        grp[7] = np.float32(-top)
        (v if row % 2 == 0 else k)[row, g0:g0 + 64] = grp
    c, dd = _kv_seeded(orc, r, T, T, kvd, True)
    orc.kv_append_int8_f32(k, v, T, kvd, 0, c)
    wz.kv_append_int8_f32(dev(k), dev(v), T, heads, hd, _kv_desc(wz, dd, T, T, True))
    for nm in _KV_PLANES:
        assert np.array_equal(_kv_host(dd, nm), getattr(c, nm)), nm


@pytest.mark.parametrize("dtype", [np.float16, np.float32])
@pytest.mark.parametrize("T,heads,hd,base", [(5, 2, 256, 17), (4096, 2, 256, 0), (33, 1, 128, 3)])
def test_k_rope_kv_append_fused(wz, orc, dtype, T, heads, hd, base):
    r = rng(T * 5 + heads + hd)
    kvd, rot, cap, max_ctx = heads * hd, 64, 32768, 8192
    k = r.standard_normal((T, kvd)).astype(dtype)
    v = r.standard_normal((T, kvd)).astype(dtype)
    gam = (0.02 * r.standard_normal(hd)).astype(dtype)
    c_, s_, dc, ds = _rope_tab(orc, base + T + 8, rot)
    cache, d = _kv_seeded(orc, r, cap, max_ctx, kvd, True)
    k_ref = orc.k_rope_kv_append(k, gam, v, c_, s_, T, heads, hd, rot, 1e-6, 1.0, base, cache)
    dk = dev(k)
    wz.k_rope_kv_append(dk, dev(gam), dev(v), dc, ds, T, heads, hd, _kv_desc(wz, d, cap, max_ctx, True), rot_dims=rot,
                        eps=1e-6, w_offset=1.0, pos_offset=base)
    if dtype == np.float16:
        assert_f16_close(host(dk).reshape(-1), k_ref.reshape(-1), ULP_TOL, "k")
    else:
        np.testing.assert_allclose(host(dk), k_ref.reshape(T, kvd), rtol=1e-5, atol=1e-5)
    # v is quantised from the same values on both sides: identical
    for nm in ["rvq", "rvs", "fvq", "fvs"]:
        assert np.array_equal(_kv_host(d, nm), getattr(cache, nm)), nm
    # k is quantised after the rotation, whose fp32 results differ by a few ulp: a code may sit on the
    # other side of a rounding boundary, a scale one fp16 ulp away
    for q, s in (("rkq", "rks"), ("fkq", "fks")):
        dq = np.abs(_kv_host(d, q).astype(np.int32) - getattr(cache, q).astype(np.int32))
        assert dq.max() <= 1 and (dq > 0).mean() < 2e-3, (q, dq.max(), (dq > 0).mean())
        ds_ = np.abs(_kv_host(d, s).astype(np.int32) - getattr(cache, s).astype(np.int32))
        assert ds_.max() <= 1, s
    assert wz.read_faults() == 0


@pytest.mark.parametrize("dtype", [np.float16, np.float32])
@pytest.mark.parametrize("T,base", [(1, 700), (8, 0), (4096, 3)])
def test_qk_rope_kv_append_one_launch(wz, orc, dtype, T, base):
    """q norm + RoPE (the reference's q layout: 24 heads interleaved with their gates, head_stride =
    2*hd) in the same launch as the k norm + RoPE + INT8 KV append: q against the oracle, the gate halves
    untouched, and k and the cache bit-identical to the k-only entry point's."""
    r = rng(T * 7 + base)
    heads, hd, qh, rot, cap, max_ctx = 2, 256, 24, 64, 32768, 8192
    kvd = heads * hd
    k = r.standard_normal((T, kvd)).astype(dtype)
    v = r.standard_normal((T, kvd)).astype(dtype)
    kg = (0.02 * r.standard_normal(hd)).astype(dtype)
    qbuf = r.standard_normal((T, qh, 2 * hd)).astype(dtype)
    qg = (0.02 * r.standard_normal(hd)).astype(dtype)
    c_, s_, dc, ds = _rope_tab(orc, base + T + 8, rot)
    # k-only launch
    cache1, d1 = _kv_seeded(orc, rng(5), cap, max_ctx, kvd, True)
    dk1 = dev(k)
    wz.k_rope_kv_append(dk1, dev(kg), dev(v), dc, ds, T, heads, hd, _kv_desc(wz, d1, cap, max_ctx, True),
                        rot_dims=rot, eps=1e-6, w_offset=1.0, pos_offset=base)
    # q + k + append in one launch
    cache2, d2 = _kv_seeded(orc, rng(5), cap, max_ctx, kvd, True)
    dk2, dq, dqg = dev(k), dev(qbuf), dev(qg)
    wz.k_rope_kv_append(dk2, dev(kg), dev(v), dc, ds, T, heads, hd, _kv_desc(wz, d2, cap, max_ctx, True),
                        rot_dims=rot, eps=1e-6, w_offset=1.0, pos_offset=base,
                        q=wz.head_tensor(dq, dqg, qh, 2 * hd, 2 * qh * hd))
    assert np.array_equal(host(dk2), host(dk1))
    for nm in ["rkq", "rks", "rvq", "rvs", "fkq", "fks", "fvq", "fvs"]:
        assert np.array_equal(_kv_host(d2, nm), _kv_host(d1, nm)), nm
    want = orc.head_norm_rope(qbuf.reshape(-1), qg, c_, s_, T, qh, hd, 2 * hd, 2 * qh * hd, rot, 1e-6, 1.0,
                              base).reshape(T, qh, 2 * hd)
    got = host(dq)
    assert np.array_equal(got[..., hd:], qbuf[..., hd:])  # gates untouched
    if dtype == np.float16:
        assert_f16_close(got[..., :hd].reshape(-1), want[..., :hd].reshape(-1), ULP_TOL, "q")
    else:
        np.testing.assert_allclose(got[..., :hd], want[..., :hd], rtol=1e-5, atol=1e-5)
    assert wz.read_faults() == 0


@pytest.mark.parametrize("hd,kv_heads,qh,T,rot,dpos", [(64, 2, 5, 8, 64, False), (128, 2, 7, 512, 64, True),
                                                       (128, 1, 7, 33, 0, False), (64, 4, 5, 100, 64, True),
                                                       (256, 2, 3, 512, 256, False), (64, 1, 9, 1, 32, True)])
def test_qk_rope_kv_append_one_launch_shapes(wz, orc, hd, kv_heads, qh, T, rot, dpos):
    """The one-launch q + k + append at head_dim 64 and 128 (4 or 2 heads per warp, q head counts that do
    not fill the last warp round), rot_dims 0 and == head_dim, positions from a device base position, and
    T = 512 (the k-only call takes one head round per warp item, the fused call two): k and the cache
    bit-identical to the k-only entry point's, q within 2 fp16 ulp of the oracle."""
    r = rng(hd * 31 + qh * 7 + T)
    cap, max_ctx = 1024, 1024
    kvd = kv_heads * hd
    k = r.standard_normal((T, kvd)).astype(np.float16)
    v = r.standard_normal((T, kvd)).astype(np.float16)
    kg = (0.02 * r.standard_normal(hd)).astype(np.float16)
    qbuf = r.standard_normal((T, qh, 2 * hd)).astype(np.float16)
    qg = (0.02 * r.standard_normal(hd)).astype(np.float16)
    base_dev, off = (37, 5) if dpos else (0, 11)
    rot_t = rot if rot > 0 else 16
    c_, s_, dc, ds = _rope_tab(orc, base_dev + off + T + 8, rot_t)
    d_base = torch.tensor([base_dev], dtype=torch.int32, device=DEV) if dpos else None
    kw = dict(rot_dims=rot, eps=1e-6, w_offset=1.0, pos_offset=off, d_base_pos=d_base)
    cache1, d1 = _kv_seeded(orc, rng(5), cap, max_ctx, kvd, True)
    dk1 = dev(k)
    wz.k_rope_kv_append(dk1, dev(kg), dev(v), dc, ds, T, kv_heads, hd, _kv_desc(wz, d1, cap, max_ctx, True), **kw)
    cache2, d2 = _kv_seeded(orc, rng(5), cap, max_ctx, kvd, True)
    dk2, dq, dqg = dev(k), dev(qbuf), dev(qg)
    wz.k_rope_kv_append(dk2, dev(kg), dev(v), dc, ds, T, kv_heads, hd, _kv_desc(wz, d2, cap, max_ctx, True),
                        q=wz.head_tensor(dq, dqg, qh, 2 * hd, 2 * qh * hd), **kw)
    assert np.array_equal(host(dk2), host(dk1))
    for nm in ["rkq", "rks", "rvq", "rvs", "fkq", "fks", "fvq", "fvs"]:
        assert np.array_equal(_kv_host(d2, nm), _kv_host(d1, nm)), nm
    want = orc.head_norm_rope(qbuf.reshape(-1), qg, c_, s_, T, qh, hd, 2 * hd, 2 * qh * hd, rot, 1e-6, 1.0,
                              base_dev + off).reshape(T, qh, 2 * hd)
    got = host(dq)
    assert np.array_equal(got[..., hd:], qbuf[..., hd:])  # gates untouched
    assert_f16_close(got[..., :hd].reshape(-1), want[..., :hd].reshape(-1), ULP_TOL, "q")
    assert wz.read_faults() == 0


# ---------------------------------------------------------------------------------------------
# the reference model's PLE: fp8 rows by the n-gram hash, gate, causal conv
# ---------------------------------------------------------------------------------------------
_SMALL_PLE_VOCAB = [1009, 1013, 1019, 1021, 1031, 1033, 1039, 1049, 1051, 1061, 1063, 1069, 1087, 1091, 1093, 1097]


@pytest.mark.parametrize("rb,prev", [(160, (1, 2)), (160, None), (32, (248044, 7)), (48, (-1, 5))])
def test_ple_gather_fp8(wz, orc, rb, prev):
    r = rng(rb)
    hsh_o = orc.PleFp8Hash(vocab=_SMALL_PLE_VOCAB)
    table = r.integers(0, 256, (hsh_o.rows, rb)).astype(np.uint8)
    table[:, 0] = 0x7F  # NaN codes in every row
    table[:, 1] = 0xFF
    T = 300
    ids = r.integers(-2, 248320, T).astype(np.int32)
    ids[5], ids[9] = 248044, -1
    want = orc.ple_gather_fp8_f32(table, rb, 0.61, hsh_o, ids, prev_ids=prev)
    out = torch.empty((T, 16 * rb), dtype=torch.float32, device=DEV)
    wz.ple_gather_fp8_f32(dev(table), rb, 0.61, wz.ple_fp8_hash(vocab=_SMALL_PLE_VOCAB), dev(ids), out,
                          prev_ids=prev)
    assert np.array_equal(host(out).view(np.uint32), want.view(np.uint32))


def test_ple_gather_fp8_full_reference_table(wz, orc):
    """The reference's hash over its full 320,001,446-row x 160-byte table (51.2 GB in HBM)."""
    hsh_o = orc.PleFp8Hash()
    rb, T = 160, 64
    gen = torch.Generator(device=DEV).manual_seed(9)
    table = torch.randint(0, 256, (hsh_o.rows, rb), generator=gen, device=DEV, dtype=torch.uint8)
    ids_np = rng(77).integers(0, 248320, T).astype(np.int32)
    out = torch.empty((T, 16 * rb), dtype=torch.float32, device=DEV)
    wz.ple_gather_fp8_f32(table, rb, 0.5, wz.ple_fp8_hash(), dev(ids_np), out, prev_ids=(100, 200))
    seq = [100, 200] + [int(v) for v in ids_np]
    rows = [orc.ple_fp8_row(seq[t + 2], seq[t + 1], seq[t], h, hsh_o) for t in range(T) for h in range(16)]
    assert max(rows) < hsh_o.rows and min(rows) >= 0
    sub = table[torch.tensor(rows, device=DEV, dtype=torch.int64)].cpu()  # [T*16, rb]
    # the rows the oracle's hash names, decoded on the host (e4m3 as torch reads it, NaN codes -> 0)
    dec = sub.view(torch.float8_e4m3fn).float().numpy()
    raw = sub.numpy()
    dec = np.where((raw & 0x7F) == 0x7F, np.where(raw & 0x80, -0.0, 0.0), dec).astype(np.float32) * np.float32(0.5)
    got = host(out).reshape(T * 16, rb)
    del table
    torch.cuda.empty_cache()
    assert np.array_equal(got.view(np.uint32), dec.view(np.uint32))


@pytest.mark.parametrize("T,n,hc", [(1, 2560, 4), (8, 2560, 4), (4096, 2560, 4), (3, 96, 2), (5, 16384, 1)])
def test_ple_gate_f32(wz, orc, T, n, hc):
    r = rng(T + n + hc)
    k = r.standard_normal((T * hc, n)).astype(np.float32)
    q = r.standard_normal((T * hc, n)).astype(np.float32)
    q[0] = -k[0]
    v = r.standard_normal((T, n)).astype(np.float32)
    want = orc.ple_gate_f32(k, q, v, T, n, hc)
    gv = torch.empty((T * hc, n), dtype=torch.float32, device=DEV)
    wz.ple_gate_f32(dev(k), dev(q), dev(v), gv, T, n, hc)
    got = host(gv)
    # The gate is sigmoid(sqrt|d|) of an n-term fp32 dot product d: where d cancels towards 0 the
    # rounding of the sum (reduction order differs) is amplified by 1/sqrt|d|, so a few rows may sit
    # several fp32 ulp away; nearly every element is within 2e-6.
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-7)
    close = np.isclose(got, want, rtol=2e-6, atol=1e-7)
    assert close.mean() > 0.999


@pytest.mark.parametrize("T,hcd,snaps", [(1, 10240, False), (5, 12, True), (9, 40, True), (40, 12, True),
                                         (4096, 10240, False), (77, 10240, True)])
def test_ple_conv_f32(wz, orc, T, hcd, snaps):
    r = rng(T * 3 + hcd)
    norm = r.standard_normal((T, hcd)).astype(np.float32)
    cw = (0.5 * r.standard_normal((hcd, 4))).astype(np.float32)
    hist = r.standard_normal((hcd, 9)).astype(np.float32)
    gv = r.standard_normal((T, hcd)).astype(np.float32)
    R = r.standard_normal((T, hcd)).astype(np.float32)
    R_ref, h_ref, s_ref = orc.ple_conv_f32(norm, cw, hist, gv, R, T, hcd, snaps=snaps)
    dR, dh = dev(R), dev(hist)
    ds = torch.empty((T, hcd, 9), dtype=torch.float32, device=DEV) if snaps else None
    wz.ple_conv_f32(dev(norm), dev(cw), dh, dev(gv), dR, T, hcd, hist_snaps=ds)
    np.testing.assert_allclose(host(dR), R_ref, rtol=2e-6, atol=2e-6)
    assert np.array_equal(host(dh), h_ref)
    if snaps:
        assert np.array_equal(host(ds), s_ref)


@pytest.mark.parametrize("T,cols,q32,q16", [(8, 2560, True, True), (4096, 2560, True, True), (1, 320, True, False),
                                             (3, 48, False, True), (77, 2560, False, True)])
def test_quant_act_f32(wz, orc, T, cols, q32, q16):
    r = rng(T + cols)
    x = (3 * r.standard_normal((T, cols))).astype(np.float32)
    x[0, :32] = 0.0  # an all-zero group
    if cols >= 96:
        # non-finite inputs (NaN dropped from the group max, code 0) and exact .5 ties (amax 127: t = x)
        x[-1, 3], x[-1, 70], x[-1, 75] = np.nan, np.inf, -np.inf
        x[-1, 32:40] = [127.0, 2.5, 3.5, -2.5, -0.5, 0.5, 126.5, -126.5]
    w32, ws32, w16, ws16 = orc.quant_act_f32(x, q32, q16)
    n = T * cols
    d32 = torch.empty(n, dtype=torch.int8, device=DEV) if q32 else None
    s32 = torch.empty(n // 32, dtype=torch.float32, device=DEV) if q32 else None
    d16 = torch.empty(n, dtype=torch.int8, device=DEV) if q16 else None
    s16 = torch.empty(n // 16, dtype=torch.float32, device=DEV) if q16 else None
    wz.quant_act_f32(dev(x), d32, s32, d16, s16, T, cols)
    # the same expression on the same fp32 values: identical codes and scales
    if q32:
        assert np.array_equal(host(d32), w32) and np.array_equal(host(s32).view(np.uint32), ws32.view(np.uint32))
    if q16:
        assert np.array_equal(host(d16), w16) and np.array_equal(host(s16).view(np.uint32), ws16.view(np.uint32))


# ---------------------------------------------------------------------------------------------
# block-scaled GEMM inputs: MXFP8 and NVFP4
# ---------------------------------------------------------------------------------------------
def _block_inputs(r, T, cols):
    # rows of very different magnitudes (and an all-zero group) exercise the per-block scales
    x = (r.standard_normal((T, cols)) * 10.0 ** r.uniform(-3, 3, (T, 1))).astype(np.float32)
    x[0, :32] = 0.0
    return x


def _dev_block_out(n, fmt):
    q = torch.empty(n if fmt == "mxfp8" else n // 2, dtype=torch.uint8, device=DEV)
    s = torch.empty(n // (32 if fmt == "mxfp8" else 16), dtype=torch.uint8, device=DEV)
    return q, s


def _oracle_block(orc, x, fmt, gs):
    return orc.quant_mxfp8(x) if fmt == "mxfp8" else orc.quant_nvfp4(x, gs)


@pytest.mark.parametrize("fmt,gs", [("mxfp8", 1.0), ("nvfp4", 1.0), ("nvfp4", 448.0 * 6.0 / 37.0)])
@pytest.mark.parametrize("T,cols", [(8, 2560), (4096, 2560), (3, 32)])
def test_quant_act_block_formats(wz, orc, fmt, gs, T, cols):
    x = _block_inputs(rng(T + cols), T, cols)
    want_q, want_s = _oracle_block(orc, x, fmt, gs)
    q, s = _dev_block_out(T * cols, fmt)
    wz.quant_act_block(dev(x), q, s, T, cols, fmt=fmt, global_scale=gs)
    assert np.array_equal(host(q), want_q) and np.array_equal(host(s), want_s)


@pytest.mark.parametrize("T", [9, 700])
@pytest.mark.parametrize("fmt", ["mxfp8", "nvfp4"])
def test_gr_norm_block_formats(wz, orc, fmt, T):
    """The norm's fp32 output and, from exactly those values, its block-format codes (9 tokens: a CTA
    per row; 700: a CTA per token)."""
    r = rng(61)
    n, hc = 2560, 4
    R = r.standard_normal((T * hc, n)).astype(np.float32)
    bo = r.standard_normal((T, n)).astype(np.float32)
    inj = r.standard_normal(T * hc).astype(np.float32)
    w = (1 + 0.02 * r.standard_normal((hc, n))).astype(np.float32)
    xn_ref, _, R_ref = orc.gr_norm_f32(R, w, bo, inj, T, n, hc)
    dR, dxn = dev(R), torch.empty((T * hc, n), dtype=torch.float32, device=DEV)
    q, s = _dev_block_out(T * hc * n, fmt)
    wz.gr_norm_block(dR, dev(w), dev(bo), dev(inj), dxn, q, s, T, n, hc, fmt=fmt, global_scale=3.0)
    xn = host(dxn)
    np.testing.assert_allclose(xn, xn_ref, rtol=2e-6, atol=2e-6)
    np.testing.assert_allclose(host(dR), R_ref, rtol=1e-6, atol=1e-6)
    want_q, want_s = _oracle_block(orc, xn, fmt, 3.0)
    assert np.array_equal(host(q), want_q) and np.array_equal(host(s), want_s)


def _to_blocked(sc, pad=0xAB):
    """Row-major [rows, scols] scale bytes -> the tiled 128x4 layout, built by reshapes: 128 x 4 tiles,
    the tiles of a 128-row band consecutive, and within a tile the (r // 32, r % 32, c) order swapped to
    (r % 32, r // 32, c). Padding rows / columns hold `pad`."""
    rows, scols = sc.shape
    rb, cb = -(-rows // 128), -(-scols // 4)
    p = np.full((rb * 128, cb * 4), pad, dtype=np.uint8)
    p[:rows, :scols] = sc
    t = p.reshape(rb, 128, cb, 4).transpose(0, 2, 1, 3)  # (band, tile, r, c)
    t = t.reshape(rb, cb, 4, 32, 4).transpose(0, 1, 3, 2, 4)  # (band, tile, r % 32, r // 32, c)
    return np.ascontiguousarray(t).reshape(-1)


@pytest.mark.parametrize("fmt", ["mxfp8", "nvfp4"])
@pytest.mark.parametrize("T,cols", [(200, 96), (129, 2560), (8, 32)])
def test_block_scales_tiled_layout(wz, fmt, T, cols):
    """The tiled scale layout holds exactly the row-major scales, relaid by reshapes; codes are the
    same; padding bytes are not written."""
    x = _block_inputs(rng(T * 7 + cols), T, cols)
    q0, s0 = _dev_block_out(T * cols, fmt)
    wz.quant_act_block(dev(x), q0, s0, T, cols, fmt=fmt, global_scale=2.0)
    q1 = torch.empty_like(q0)
    s1 = torch.full((wz.sf_tiled_bytes(T, cols, fmt),), 0xAB, dtype=torch.uint8, device=DEV)
    wz.quant_act_block(dev(x), q1, s1, T, cols, fmt=fmt, global_scale=2.0, sf_layout=wz.SF_TILED_128X4)
    g = 32 if fmt == "mxfp8" else 16
    assert np.array_equal(host(q1), host(q0))
    assert np.array_equal(host(s1), _to_blocked(host(s0).reshape(T, cols // g)))


@pytest.mark.parametrize("T", [9, 700])
def test_gr_norm_block_tiled_layout(wz, T):
    r = rng(63)
    n, hc = 2560, 4
    R = r.standard_normal((T * hc, n)).astype(np.float32)
    bo = r.standard_normal((T, n)).astype(np.float32)
    inj = r.standard_normal(T * hc).astype(np.float32)
    w = (1 + 0.02 * r.standard_normal((hc, n))).astype(np.float32)
    for fmt in ("mxfp8", "nvfp4"):
        outs = []
        for layout in (None, wz.SF_TILED_128X4):
            dxn = torch.empty((T * hc, n), dtype=torch.float32, device=DEV)
            q, s = _dev_block_out(T * hc * n, fmt)
            if layout is not None:
                s = torch.full((wz.sf_tiled_bytes(T * hc, n, fmt),), 0xAB, dtype=torch.uint8, device=DEV)
            wz.gr_norm_block(dev(R), dev(w), dev(bo), dev(inj), dxn, q, s, T, n, hc, fmt=fmt, global_scale=3.0,
                             sf_layout=layout)
            outs.append((host(dxn), host(q), host(s)))
        g = 32 if fmt == "mxfp8" else 16
        assert np.array_equal(outs[0][0], outs[1][0]) and np.array_equal(outs[0][1], outs[1][1])
        assert np.array_equal(outs[1][2], _to_blocked(outs[0][2].reshape(T * hc, n // g)))


@pytest.mark.parametrize("fmt", ["mxfp8", "nvfp4"])
def test_swiglu_block_tiled_layout(wz, fmt):
    r = rng(65)
    rows, cols = 77, 512
    g = (2 * r.standard_normal((rows, cols))).astype(np.float32)
    u = r.standard_normal((rows, cols)).astype(np.float32)
    q0, s0 = _dev_block_out(rows * cols, fmt)
    wz.swiglu_block(dev(g), dev(u), q0, s0, fmt=fmt, global_scale=2.0)
    q1 = torch.empty_like(q0)
    s1 = torch.full((wz.sf_tiled_bytes(rows, cols, fmt),), 0xAB, dtype=torch.uint8, device=DEV)
    wz.swiglu_block(dev(g), dev(u), q1, s1, fmt=fmt, global_scale=2.0, sf_layout=wz.SF_TILED_128X4, cols=cols)
    gsz = 32 if fmt == "mxfp8" else 16
    assert np.array_equal(host(q1), host(q0))
    assert np.array_equal(host(s1), _to_blocked(host(s0).reshape(rows, cols // gsz)))


def test_nvfp4_tiled_scales_feed_a_block_scaled_gemm(wz):
    """As the MXFP8 case, for NVFP4 (e2m1 pairs, e4m3 scale per 16; global scale 1) through torch's FP4
    block-scaled GEMM, where this torch build has one."""
    if not hasattr(torch, "float4_e2m1fn_x2"):
        pytest.skip("torch has no float4_e2m1fn_x2")
    M, N, K = 256, 256, 512
    r = rng(66)
    a = r.standard_normal((M, K)).astype(np.float32)
    b = r.standard_normal((N, K)).astype(np.float32)
    qa, qb = torch.empty(M * K // 2, dtype=torch.uint8, device=DEV), torch.empty(N * K // 2, dtype=torch.uint8, device=DEV)
    sa = torch.empty(wz.sf_tiled_bytes(M, K, "nvfp4"), dtype=torch.uint8, device=DEV)
    sb = torch.empty(wz.sf_tiled_bytes(N, K, "nvfp4"), dtype=torch.uint8, device=DEV)
    wz.quant_act_block(dev(a), qa, sa, M, K, fmt="nvfp4", sf_layout=wz.SF_TILED_128X4)
    wz.quant_act_block(dev(b), qb, sb, N, K, fmt="nvfp4", sf_layout=wz.SF_TILED_128X4)
    A = qa.view(torch.float4_e2m1fn_x2).view(M, K // 2)
    B = qb.view(torch.float4_e2m1fn_x2).view(N, K // 2)
    try:
        out = torch._scaled_mm(A, B.t(), scale_a=sa.view(torch.float8_e4m3fn), scale_b=sb.view(torch.float8_e4m3fn),
                               out_dtype=torch.bfloat16)
    except (RuntimeError, TypeError, ValueError, NotImplementedError) as e:
        pytest.skip(f"no NVFP4 block-scaled GEMM in this torch build: {str(e)[:120]}")
    lut = torch.tensor([0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6], device=DEV)

    def deq(q, rows, x):
        rs = torch.empty(rows * K // 16, dtype=torch.uint8, device=DEV)
        qq = torch.empty_like(q)
        wz.quant_act_block(dev(x), qq, rs, rows, K, fmt="nvfp4")
        v = torch.stack([lut[(qq & 0xF).long()], lut[(qq >> 4).long()]], dim=-1).view(rows, K)
        return v * rs.view(torch.float8_e4m3fn).float().view(rows, K // 16).repeat_interleave(16, dim=1)

    want = deq(qa, M, a).double() @ deq(qb, N, b).double().t()
    err = (out.double() - want).abs().max().item() / want.abs().max().item()
    assert err < 1e-2, f"NVFP4 block-scaled GEMM vs dequantised product: {err}"


def test_mxfp8_tiled_scales_feed_a_block_scaled_gemm(wz):
    """End to end: A [M, K] and B [N, K] quantised to MXFP8 with tiled scales go straight into the block-
    scaled tensor-core GEMM of this torch build (torch._scaled_mm, cuBLASLt); the product matches the
    fp32 product of the dequantised operands."""
    if not hasattr(torch, "float8_e8m0fnu"):
        pytest.skip("torch has no float8_e8m0fnu")
    M, N, K = 256, 384, 512
    r = rng(64)
    a = (r.standard_normal((M, K)) * np.exp(r.uniform(-3, 3, (M, 1)))).astype(np.float32)
    b = r.standard_normal((N, K)).astype(np.float32)
    qa, qb = torch.empty(M * K, dtype=torch.uint8, device=DEV), torch.empty(N * K, dtype=torch.uint8, device=DEV)
    sa = torch.empty(wz.sf_tiled_bytes(M, K), dtype=torch.uint8, device=DEV)
    sb = torch.empty(wz.sf_tiled_bytes(N, K), dtype=torch.uint8, device=DEV)
    wz.quant_act_block(dev(a), qa, sa, M, K, sf_layout=wz.SF_TILED_128X4)
    wz.quant_act_block(dev(b), qb, sb, N, K, sf_layout=wz.SF_TILED_128X4)
    A = qa.view(torch.float8_e4m3fn).view(M, K)
    B = qb.view(torch.float8_e4m3fn).view(N, K)
    try:
        out = torch._scaled_mm(A, B.t(), scale_a=sa.view(torch.float8_e8m0fnu), scale_b=sb.view(torch.float8_e8m0fnu),
                               out_dtype=torch.bfloat16)
    except (RuntimeError, TypeError, ValueError) as e:
        pytest.skip(f"no MXFP8 block-scaled GEMM in this torch build: {str(e)[:120]}")
    # dequantise from the row-major scales of the same data
    ra, rs = torch.empty_like(qa), torch.empty(M * K // 32, dtype=torch.uint8, device=DEV)
    rb_, rbs = torch.empty_like(qb), torch.empty(N * K // 32, dtype=torch.uint8, device=DEV)
    wz.quant_act_block(dev(a), ra, rs, M, K)
    wz.quant_act_block(dev(b), rb_, rbs, N, K)
    da = A.float() * torch.exp2(rs.float() - 127).view(M, K // 32).repeat_interleave(32, dim=1)
    db = B.float() * torch.exp2(rbs.float() - 127).view(N, K // 32).repeat_interleave(32, dim=1)
    want = da.double() @ db.double().t()
    err = (out.double() - want).abs().max().item() / want.abs().max().item()
    assert err < 1e-2, f"block-scaled GEMM vs dequantised product: {err}"


@pytest.mark.parametrize("fmt", ["mxfp8", "nvfp4"])
def test_swiglu_block_formats(wz, orc, fmt):
    r = rng(62)
    n = 640 * 512
    g = (2 * r.standard_normal(n)).astype(np.float32)
    u = r.standard_normal(n).astype(np.float32)
    act = orc.swiglu(g, u)  # libm expf: the kernel's __expf can move a value across a rounding boundary
    want_q, want_s = _oracle_block(orc, act, fmt, 1.0)
    q, s = _dev_block_out(n, fmt)
    wz.swiglu_block(dev(g), dev(u), q, s, fmt=fmt)
    gq, gs_ = host(q), host(s)
    assert (gs_ != want_s).mean() < 1e-3
    assert (gq != want_q).mean() < 1e-3


def test_graph_capture_replays_bit_identical(wz, orc):
    """Every entry point is capture-safe (no sync, allocation or host read of device memory): a window of
    launches recorded into a CUDA graph and replayed gives the eager results bit for bit."""
    r = rng(91)
    T, n = 8, 2048
    x, res0 = f16n(r, (T, n)), f16n(r, (T, n))
    w = f16n(r, (n,), 0.02)
    q0, k0 = f16n(r, (T, 16, 256)), f16n(r, (T, 2, 256))
    gq = f16n(r, (256,), 0.02)
    c, s, dc, ds = _rope_tab(orc, 64, 64)
    g, u = f16n(r, (T * 11, 512)), f16n(r, (T * 11, 512))
    R0 = r.standard_normal((T * 4, 2560)).astype(np.float32)
    bo = r.standard_normal((T, 2560)).astype(np.float32)
    wn = (1 + 0.02 * r.standard_normal((4, 2560))).astype(np.float32)

    def window(bufs):
        dres, dy, dq, dk, act, dR, xn, q8, s8 = bufs
        wz.add_rmsnorm_f16(dx, dres, dw, dy, 1e-6, 1.0)
        wz.qk_norm_rope_f16(wz.head_tensor(dq, dgq, 16, 256, 4096), wz.head_tensor(dk, dgq, 2, 256, 512), dc, ds, T,
                            256, 64, 1e-6, 1.0, pos_offset=3)
        wz.swiglu(dg, du, act)
        wz.gr_norm_q8_f32(dR, dwn, dbo, None, xn, q8, s8, T, 2560, 4)

    dx, dw, dgq, dg, du, dbo, dwn = dev(x), dev(w), dev(gq), dev(g), dev(u), dev(bo), dev(wn)

    def fresh():
        return [dev(res0), torch.empty((T, n), dtype=torch.float16, device=DEV), dev(q0), dev(k0),
                torch.empty((T * 11, 512), dtype=torch.float16, device=DEV), dev(R0),
                torch.empty((T * 4, 2560), device=DEV), torch.empty((T * 4, 2560), dtype=torch.int8, device=DEV),
                torch.empty((T * 4, 80), device=DEV)]

    eager = fresh()
    window(eager)
    torch.cuda.synchronize()
    graphed = fresh()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        window(graphed)
    # capture records without running: restore the in-place inputs, then replay once
    for i, src in ((0, res0), (2, q0), (3, k0), (5, R0)):
        graphed[i].copy_(torch.from_numpy(np.ascontiguousarray(src)).to(DEV))
    graph.replay()
    torch.cuda.synchronize()
    for a, b in zip(eager, graphed):
        assert torch.equal(a, b)
    del graph
