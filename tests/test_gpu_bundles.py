"""GPU parity of the one-launch layer bundles (wzyb_attn_prep_f16, wzyb_act_f16, wzyb_embed_ple_f16).

Each bundle up to its measured one-launch size runs its two ops in one persistent grid (larger ones as the ops' own
launches). Checked here:
  - against the oracle on the same seeded inputs (norms, RoPE, gate, SwiGLU within 2 fp16 ulp; the
    gathers and the residual bit-exact), at the configs' shapes (4096 tokens), a long call (20,000)
    and ragged short calls where some roles get a single CTA;
  - bit for bit against the same ops issued as separate launches (WZYB_VARIANT_SPLIT), since the one-
    launch kernels run the per-op device code;
  - every grid schedule (split grid, one item per warp, both ops on every CTA) bit for bit against the
    separate launches, at sizes where the ops get one item per warp, several, and uneven counts;
  - that tensors shared between the two ops make the entry point fall back to the ordered launches.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import ULP_TOL, assert_f16_close

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
def _reset(wz):
    torch.cuda.set_device(0)
    wz.read_faults(clear=True)
    yield
    torch.cuda.synchronize()
    wz.set_kernel_variant(wz.FAM_BUNDLE, wz.VARIANT_AUTO)
    wz.set_launch_tuning(wz.FAM_BUNDLE, 1, 0)


def _bits(t):
    return host(t).view(np.uint16).copy()


def _attn_inputs(r, T, n, qh, kh, hd):
    return dict(x=f16n(r, (T, n)), res=f16n(r, (T, n)), w=f16n(r, (n,), 0.02), q=f16n(r, (T, qh, hd)),
                k=f16n(r, (T, kh, hd)), gq=f16n(r, (hd,), 0.02), gk=f16n(r, (hd,), 0.02))


def _run_attn(wz, inp, c, s, T, n, qh, kh, hd, rot, off, variant):
    wz.set_kernel_variant(wz.FAM_BUNDLE, variant)
    d = {k: dev(v) for k, v in inp.items()}
    dy = torch.empty((T, n), dtype=torch.float16, device=DEV)
    a = wz.AttnPrepArgs()
    a.x, a.residual, a.norm_weight, a.normed, a.hidden = (d["x"].data_ptr(), d["res"].data_ptr(), d["w"].data_ptr(),
                                                          dy.data_ptr(), n)
    a.q = wz.head_tensor(d["q"], d["gq"], qh, hd, qh * hd)
    a.k = wz.head_tensor(d["k"], d["gk"], kh, hd, kh * hd)
    a.head_dim, a.rot_dims = hd, rot
    a.cos_tab, a.sin_tab, a.table_rows = c.data_ptr(), s.data_ptr(), c.shape[0]
    a.d_base_pos, a.pos_offset, a.eps, a.w_offset = None, off, 1e-6, 1.0
    wz.call("wzyb_attn_prep_f16", ctypes.byref(a), T, wz._stream())
    return {"y": _bits(dy), "res": _bits(d["res"]), "q": _bits(d["q"]), "k": _bits(d["k"])}


@pytest.mark.parametrize("T,n,qh,kh,hd", [(1, 2048, 16, 2, 256), (7, 2048, 16, 2, 256), (300, 2048, 16, 2, 256),
                                          (4096, 2048, 16, 2, 256), (20000, 2048, 16, 2, 256),
                                          (513, 1024, 8, 1, 128), (97, 2560, 5, 3, 64), (33, 24, 16, 2, 256)])
def test_attn_prep_bundle(wz, orc, T, n, qh, kh, hd):
    """residual add + RMSNorm [T, 2048] and q/k norm + partial RoPE (16 + 2 heads of 256) in
    one launch; other hidden sizes and head sizes exercise each instantiation (hidden 24: a row shorter
    than a warp's first vector round)."""
    r = rng(T * 3 + n + hd)
    rot, off = 64, 11
    inp = _attn_inputs(r, T, n, qh, kh, hd)
    c_h, s_h = orc.rope_table(T + off, rot, 1e7)
    c, s = dev(c_h), dev(s_h)
    one = _run_attn(wz, inp, c, s, T, n, qh, kh, hd, rot, off, wz.VARIANT_AUTO)
    split = _run_attn(wz, inp, c, s, T, n, qh, kh, hd, rot, off, wz.VARIANT_SPLIT)
    for key in one:
        assert np.array_equal(one[key], split[key]), f"one launch vs separate launches differ in {key}"
    y_ref, res_ref = orc.add_rmsnorm_f16(inp["x"], inp["res"], inp["w"], 1e-6, 1.0)
    assert np.array_equal(one["res"], res_ref.view(np.uint16))
    assert_f16_close(one["y"].view(np.float16), y_ref, ULP_TOL, f"attn bundle norm T={T}")
    q_ref = orc.head_norm_rope(inp["q"].reshape(-1), inp["gq"], c_h, s_h, T, qh, hd, hd, qh * hd, rot, 1e-6, 1.0, off)
    k_ref = orc.head_norm_rope(inp["k"].reshape(-1), inp["gk"], c_h, s_h, T, kh, hd, hd, kh * hd, rot, 1e-6, 1.0, off)
    assert_f16_close(one["q"].view(np.float16).reshape(-1), q_ref, ULP_TOL, f"attn bundle q T={T}")
    assert_f16_close(one["k"].view(np.float16).reshape(-1), k_ref, ULP_TOL, f"attn bundle k T={T}")
    assert wz.read_faults() == 0


def _run_act(wz, inp, T, rows, ffn, H, ghd, gate_mode, variant):
    wz.set_kernel_variant(wz.FAM_BUNDLE, variant)
    d = {k: dev(v) for k, v in inp.items()}
    dact = torch.empty((rows, ffn), dtype=torch.float16, device=DEV)
    dgy = torch.empty((T, H, ghd), dtype=torch.float16, device=DEV)
    b = wz.ActArgs()
    b.gate, b.up, b.act, b.act_rows, b.ffn = d["g"].data_ptr(), d["u"].data_ptr(), dact.data_ptr(), rows, ffn
    b.o, b.z, b.gdn_gamma, b.gdn_out = d["o"].data_ptr(), d["z"].data_ptr(), d["gm"].data_ptr(), dgy.data_ptr()
    b.gdn_heads, b.gdn_head_dim, b.eps, b.gdn_w_offset, b.gate_mode = H, ghd, 1e-6, 0.0, gate_mode
    wz.call("wzyb_act_f16", ctypes.byref(b), T, wz._stream())
    return {"act": _bits(dact), "gy": _bits(dgy)}


@pytest.mark.parametrize("T,H,ghd,gate_mode", [(1, 32, 128, 0), (5, 32, 128, 0), (300, 32, 128, 1),
                                               (4096, 32, 128, 0), (20000, 32, 128, 0), (77, 6, 256, 0),
                                               (129, 3, 64, 1)])
def test_act_bundle(wz, orc, T, H, ghd, gate_mode):
    """SwiGLU over 11 expert rows x 512 per token and the GDN gated norm [T, 32, 128] in one
    launch (gate sigmoid as the reference, or z*sigmoid(z))."""
    r = rng(T * 5 + H + ghd)
    rows, ffn = 11 * T, 512
    inp = dict(g=f16n(r, (rows, ffn), 2.0), u=f16n(r, (rows, ffn)), o=f16n(r, (T, H, ghd)), z=f16n(r, (T, H, ghd)),
               gm=f16n(r, (ghd,), 0.02, 1.0))
    one = _run_act(wz, inp, T, rows, ffn, H, ghd, gate_mode, wz.VARIANT_AUTO)
    split = _run_act(wz, inp, T, rows, ffn, H, ghd, gate_mode, wz.VARIANT_SPLIT)
    for key in one:
        assert np.array_equal(one[key], split[key]), f"one launch vs separate launches differ in {key}"
    assert_f16_close(one["act"].view(np.float16), orc.swiglu(inp["g"], inp["u"]), ULP_TOL, f"act bundle swiglu T={T}")
    want = orc.gdn_gated_norm(inp["o"], inp["z"], inp["gm"], T, H, ghd, 1e-6, 0.0, gate_mode)
    assert_f16_close(one["gy"].view(np.float16), want, ULP_TOL, f"act bundle gdn T={T}")


def _run_embed_ple(wz, table, tabs, ids, T, hidden, heads, hd, prev, variant, policy=0):
    wz.set_kernel_variant(wz.FAM_BUNDLE, variant)
    emb = torch.empty((T, hidden), dtype=torch.float16, device=DEV)
    ple = torch.empty((T, heads * hd), dtype=torch.float16, device=DEV)
    cnt = torch.zeros(1, dtype=torch.int32, device=DEV)
    args = wz.embed_ple_args(table, tabs, ids, emb, ple, prev_ids=prev, oob_policy=policy, oob_count=cnt)
    wz.embed_ple_f16(args, T)
    return _bits(emb), _bits(ple), int(host(cnt)[0])


@pytest.mark.parametrize("T,vocab,hidden,heads,rows,hd", [(1, 5000, 2048, 16, 4096, 128), (2, 5000, 2048, 16, 4096, 128),
                                                          (300, 7001, 2048, 16, 4099, 128),
                                                          (20000, 9000, 2048, 16, 1 << 12, 128),
                                                          (257, 3000, 72, 5, 4099, 64), (64, 3000, 1024, 4, 777, 256)])
def test_embed_ple_bundle(wz, orc, T, vocab, hidden, heads, rows, hd):
    """configs[3] layout (token rows and 16 PLE rows of the same ids) in one launch, with out-of-range ids
    (counted), EOS ids and a 2-id history from a previous chunk; bit-exact."""
    r = rng(T + vocab + hd)
    table = f16n(r, (vocab, hidden), 0.02)
    tabs = [f16n(r, (rows, hd), 0.02) for _ in range(heads)]
    ids = r.integers(0, vocab, T).astype(np.int32)
    if T > 8:
        ids[[1, T // 2, T - 1]] = [-3, vocab + 5, 248044]
    prev = (17, 248044) if T % 2 else (9, 4)
    dt, dtabs, dids = dev(table), [dev(t) for t in tabs], dev(ids)
    e1, p1, c1 = _run_embed_ple(wz, dt, dtabs, dids, T, hidden, heads, hd, prev, wz.VARIANT_AUTO)
    e2, p2, c2 = _run_embed_ple(wz, dt, dtabs, dids, T, hidden, heads, hd, prev, wz.VARIANT_SPLIT)
    assert np.array_equal(e1, e2) and np.array_equal(p1, p2) and c1 == c2
    want_e, bad = orc.embed_gather_rows(table, ids, 0)
    assert np.array_equal(e1, want_e.view(np.uint16))
    assert c1 == bad
    want_p = orc.ple_gather_f16(tabs, ids, prev, 248044, 0)
    assert np.array_equal(p1, want_p.view(np.uint16))


def test_embed_ple_bundle_baseline_shape(wz, orc):
    """configs[3] exactly: fp16 token table [151936, 2048] ~N(0,0.02), 16 PLE tables [2^20, 128], 4096
    uniform ids, one launch; bit-exact."""
    T = 4096
    gen = torch.Generator(device=DEV).manual_seed(51)
    table = (torch.randn((151936, 2048), generator=gen, device=DEV) * 0.02).half()
    tabs = [(torch.randn((1 << 20, 128), generator=gen, device=DEV) * 0.02).half() for _ in range(16)]
    ids = rng(52).integers(0, 151936, T).astype(np.int32)
    e, p, c = _run_embed_ple(wz, table, tabs, dev(ids), T, 2048, 16, 128, None, wz.VARIANT_AUTO)
    want_e, bad = orc.embed_gather_rows(host(table), ids, 0)
    assert np.array_equal(e, want_e.view(np.uint16)) and c == bad == 0
    want_p = orc.ple_gather_f16([host(t) for t in tabs], ids, None, 248044, 0)
    assert np.array_equal(p, want_p.view(np.uint16))


def test_bundle_with_shared_tensor_keeps_launch_order(wz, orc):
    """When one op's output is the other op's input (here the GDN norm reads the SwiGLU output as o),
    the bundle must keep the reference's order: SwiGLU first, then the norm of its result."""
    r = rng(77)
    T, H, ghd, ffn = 64, 4, 128, 512
    rows = T  # SwiGLU output [T, 512] == o [T, 4, 128]
    g, u, z = f16n(r, (rows, ffn)), f16n(r, (rows, ffn)), f16n(r, (T, H, ghd))
    gm = f16n(r, (ghd,), 0.02, 1.0)
    dg, du, dz, dgm = dev(g), dev(u), dev(z), dev(gm)
    dact = torch.empty((rows, ffn), dtype=torch.float16, device=DEV)
    dgy = torch.empty((T, H, ghd), dtype=torch.float16, device=DEV)
    b = wz.ActArgs()
    b.gate, b.up, b.act, b.act_rows, b.ffn = dg.data_ptr(), du.data_ptr(), dact.data_ptr(), rows, ffn
    b.o, b.z, b.gdn_gamma, b.gdn_out = dact.data_ptr(), dz.data_ptr(), dgm.data_ptr(), dgy.data_ptr()
    b.gdn_heads, b.gdn_head_dim, b.eps, b.gdn_w_offset, b.gate_mode = H, ghd, 1e-6, 0.0, 0
    wz.call("wzyb_act_f16", ctypes.byref(b), T, wz._stream())
    act_ref = orc.swiglu(g, u)
    assert_f16_close(host(dact), act_ref, ULP_TOL, "swiglu")
    # the norm must have read the SwiGLU output that this library wrote
    want = orc.gdn_gated_norm(host(dact).reshape(T, H, ghd), z, gm, T, H, ghd, 1e-6, 0.0, 0)
    assert_f16_close(host(dgy), want, ULP_TOL, "gdn of the swiglu output")


@pytest.mark.parametrize("sched", [1, 2, 3])
@pytest.mark.parametrize("T", [3, 700, 4096, 9001])
def test_bundle_schedules_bit_identical(wz, orc, sched, T):
    """Each schedule of the one-launch grid (wzyb_set_launch_tuning(WZYB_FAM_BUNDLE, 1, sched): 1 split
    grid, 2 one item per warp, 3 both ops on every CTA) against the ops' own launches, for all three
    bundles, bit for bit (the schedules only move work between warps)."""
    r = rng(1000 * sched + T)
    wz.set_launch_tuning(wz.FAM_BUNDLE, 1, sched)
    n, qh, kh, hd, rot, off = 2048, 16, 2, 256, 64, 5
    inp = _attn_inputs(r, T, n, qh, kh, hd)
    c_h, s_h = orc.rope_table(T + off, rot, 1e7)
    c, s = dev(c_h), dev(s_h)
    one = _run_attn(wz, inp, c, s, T, n, qh, kh, hd, rot, off, wz.VARIANT_AUTO)
    split = _run_attn(wz, inp, c, s, T, n, qh, kh, hd, rot, off, wz.VARIANT_SPLIT)
    for key in one:
        assert np.array_equal(one[key], split[key]), f"attn sched {sched}: {key} differs"
    rows, ffn, H, ghd = 11 * T, 512, 32, 128
    ainp = dict(g=f16n(r, (rows, ffn), 2.0), u=f16n(r, (rows, ffn)), o=f16n(r, (T, H, ghd)),
                z=f16n(r, (T, H, ghd)), gm=f16n(r, (ghd,), 0.02, 1.0))
    one = _run_act(wz, ainp, T, rows, ffn, H, ghd, 0, wz.VARIANT_AUTO)
    split = _run_act(wz, ainp, T, rows, ffn, H, ghd, 0, wz.VARIANT_SPLIT)
    for key in one:
        assert np.array_equal(one[key], split[key]), f"act sched {sched}: {key} differs"
    vocab, hidden, heads, prow, phd = 6000, 2048, 16, 4099, 128
    table = f16n(r, (vocab, hidden), 0.02)
    tabs = [f16n(r, (prow, phd), 0.02) for _ in range(heads)]
    ids = r.integers(-2, vocab + 2, T).astype(np.int32)
    dt, dtabs, dids = dev(table), [dev(t) for t in tabs], dev(ids)
    e1, p1, c1 = _run_embed_ple(wz, dt, dtabs, dids, T, hidden, heads, phd, (3, 4), wz.VARIANT_AUTO)
    e2, p2, c2 = _run_embed_ple(wz, dt, dtabs, dids, T, hidden, heads, phd, (3, 4), wz.VARIANT_SPLIT)
    assert np.array_equal(e1, e2) and np.array_equal(p1, p2) and c1 == c2, f"embed_ple sched {sched} differs"
    want_e, bad = orc.embed_gather_rows(table, ids, 0)
    assert np.array_equal(e1, want_e.view(np.uint16)) and c1 == bad
    assert wz.read_faults() == 0
