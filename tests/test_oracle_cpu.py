"""CPU checks of the oracle itself: fp16 conversion, an independent numpy restatement of each op,
the reference's own host RoPE table, and the PLE hash against a pure-Python restatement."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_f16_close, f16_ulp_distance

RNG = np.random.default_rng(1234)


def test_f16_roundtrip_matches_numpy(orc):
    # every fp16 bit pattern widens exactly
    bits = np.arange(65536, dtype=np.uint16)
    want = bits.view(np.float16).astype(np.float32)
    got = np.empty(65536, dtype=np.float32)
    orc.lib().or_h2f_array(bits.ctypes.data, got.ctypes.data, 65536)
    finite = np.isfinite(want)
    assert np.array_equal(got[finite].view(np.uint32), want[finite].view(np.uint32))
    assert np.all(np.isnan(got[~finite & np.isnan(want)]))
    # float -> fp16 rounding (RN-even) matches numpy on a wide sample incl. subnormals, ties, overflow
    x = np.concatenate([
        RNG.standard_normal(200000).astype(np.float32) * np.float32(10.0) ** RNG.integers(-9, 6, 200000),
        (np.arange(-4096, 4096, dtype=np.float32) + 0.5) * np.float32(2.0 ** -24),  # ties in the subnormal range
        np.array([65504, 65519.99, 65520, 70000, -65520, 6.1035156e-05, 5.96e-08, 2.98e-08, 0.0, -0.0],
                 dtype=np.float32),
    ]).astype(np.float32)
    got = np.empty(x.size, dtype=np.uint16)
    orc.lib().or_f2h_array(x.ctypes.data, got.ctypes.data, x.size)
    with np.errstate(over="ignore"):
        want16 = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, want16)


def _ref64_rmsnorm(v, g, eps):
    v = v.astype(np.float64)
    return v / np.sqrt((v * v).mean(axis=-1, keepdims=True) + eps) * g


def test_add_rmsnorm_against_float64(orc):
    T, n = 37, 2048
    x = RNG.standard_normal((T, n)).astype(np.float16)
    r = RNG.standard_normal((T, n)).astype(np.float16)
    w = (RNG.standard_normal(n) * 0.02).astype(np.float16)
    y, r2 = orc.add_rmsnorm_f16(x, r, w, 1e-6, 1.0)
    v = x.astype(np.float32) + r.astype(np.float32)
    assert np.array_equal(r2, v.astype(np.float16))
    want = _ref64_rmsnorm(v, 1.0 + w.astype(np.float64), 1e-6).astype(np.float16)
    assert_f16_close(y, want, 1, "add_rmsnorm vs f64")
    # x = None: plain norm, residual untouched
    y2, r3 = orc.add_rmsnorm_f16(None, r, w, 1e-6, 0.0)
    assert np.array_equal(r3, r)
    assert_f16_close(y2, _ref64_rmsnorm(r.astype(np.float32), w.astype(np.float64), 1e-6).astype(np.float16), 1)


def test_gr_norm_hyper_connection_against_float64(orc):
    T, n, hc = 5, 256, 4
    R = RNG.standard_normal((T * hc, n)).astype(np.float32)
    bo = RNG.standard_normal((T, n)).astype(np.float32)
    inj = RNG.standard_normal((T * hc,)).astype(np.float32)
    w = (1 + 0.02 * RNG.standard_normal((hc, n))).astype(np.float32)
    xn, xh, R2 = orc.gr_norm_f32(R, w, bo, inj, T, n, hc)
    gw = 2.0 / (1.0 + np.exp(-inj.astype(np.float64) / hc))
    v = R.astype(np.float64) + np.repeat(bo, hc, axis=0) * gw[:, None]
    np.testing.assert_allclose(R2, v, rtol=1e-6, atol=1e-6)
    want = _ref64_rmsnorm(v, np.tile(w, (T, 1)), 1e-6)
    np.testing.assert_allclose(xn, want, rtol=2e-6, atol=2e-6)


def test_rope_table_matches_reference_host_builder(orc):
    """The oracle's table equals the reference's own build_rope_cos_sin_host bit for bit."""
    if not orc.ref_available():
        pytest.skip("reference kernels library not built (needs the reference sources)")
    rows = 5000
    c, s = orc.rope_table(rows, 64, 1e7)
    rc, rs = orc.ref_rope_table(rows, 1e7)
    assert np.array_equal(c.view(np.uint32), rc.view(np.uint32))
    assert np.array_equal(s.view(np.uint32), rs.view(np.uint32))


def test_head_norm_rope_against_float64(orc):
    T, H, hd, rot = 9, 3, 256, 64
    data = RNG.standard_normal((T, H, hd)).astype(np.float16)
    gam = (0.02 * RNG.standard_normal(hd)).astype(np.float16)
    c, s = orc.rope_table(64, rot, 1e7)
    got = orc.head_norm_rope(data.reshape(-1), gam, c, s, T, H, hd, hd, H * hd, rot, 1e-6, 1.0, base_pos=7)
    p = _ref64_rmsnorm(data.astype(np.float32), 1.0 + gam.astype(np.float64), 1e-6)
    half = rot // 2
    pos = 7 + np.arange(T)
    cs = c[pos][:, None, :].astype(np.float64)
    sn = s[pos][:, None, :].astype(np.float64)
    a, d = p[..., :half].copy(), p[..., half:rot].copy()
    p[..., :half] = a * cs - d * sn
    p[..., half:rot] = a * sn + d * cs
    assert_f16_close(got.reshape(T, H, hd), p.astype(np.float16), 1, "head_norm_rope vs f64")


def test_gdn_and_swiglu_against_float64(orc):
    T, H, hd = 11, 4, 128
    o = RNG.standard_normal((T, H, hd)).astype(np.float16)
    z = RNG.standard_normal((T, H, hd)).astype(np.float16)
    gm = (1 + 0.02 * RNG.standard_normal(hd)).astype(np.float16)
    y = orc.gdn_gated_norm(o, z, gm, T, H, hd, 1e-6, 0.0, 0)
    want = _ref64_rmsnorm(o.astype(np.float32), gm.astype(np.float64), 1e-6) / (1 + np.exp(-z.astype(np.float64)))
    assert_f16_close(y, want.astype(np.float16), 1, "gdn sigmoid")
    y2 = orc.gdn_gated_norm(o, z, gm, T, H, hd, 1e-6, 0.0, 1)
    want2 = want * z.astype(np.float64)
    assert_f16_close(y2, want2.astype(np.float16), 1, "gdn silu")
    g = RNG.standard_normal(4096).astype(np.float16)
    u = RNG.standard_normal(4096).astype(np.float16)
    out = orc.swiglu(g, u)
    g64 = g.astype(np.float64)
    assert_f16_close(out, (g64 / (1 + np.exp(-g64)) * u).astype(np.float16), 1, "swiglu")
    gu = np.concatenate([g.reshape(8, 512), u.reshape(8, 512)], axis=1)
    out2 = orc.swiglu_interleaved(gu, 8, 512)
    assert np.array_equal(out2.reshape(-1), out)


def _py_ple_row(t0, t1, t2, head, rows, eos, variant):
    cut = t1 < 0 or t1 == eos
    c1 = eos if cut else t1
    cut = cut or t2 < 0 or t2 == eos
    c2 = eos if cut else t2
    m = 0xFFFFFFFF
    a = (t0 * 0x9E3779B1) & m
    b = (c1 * 0x85EBCA77) & m
    c = (c2 * 0xC2B2AE3D) & m
    h = ((a ^ b ^ c) + head) & m if variant == 1 else (a ^ b ^ ((c + head) & m))
    return h % rows


@pytest.mark.parametrize("variant", [0, 1])
def test_ple_row_matches_python(orc, variant):
    rows = 1 << 20
    cases = [(5, 7, 9), (0, -1, -1), (123, 248044, 55), (123, 55, 248044), (-3, 4, 5), (151935, 151934, 151933)]
    cases += [tuple(int(v) for v in RNG.integers(-2, 151936, 3)) for _ in range(200)]
    for t0, t1, t2 in cases:
        for h in (0, 1, 15):
            assert orc.ple_row(t0, t1, t2, h, rows, 248044, variant) == _py_ple_row(t0, t1, t2, h, rows, 248044,
                                                                                     variant)
    # the two readings of the formula differ (so the choice is observable)
    assert any(orc.ple_row(t0, t1, t2, 3, rows, 248044, 0) != orc.ple_row(t0, t1, t2, 3, rows, 248044, 1)
               for t0, t1, t2 in cases)


def test_ple_gather_boundary_and_cut(orc):
    heads, rows, hd = 4, 64, 16
    tables = [RNG.standard_normal((rows, hd)).astype(np.float16) for _ in range(heads)]
    ids = np.array([3, 248044, 9, 10, 11], dtype=np.int32)
    out = orc.ple_gather_f16(tables, ids, prev_ids=(1, 2), eos=248044, variant=0)
    seq = [1, 2] + [int(v) for v in ids]  # prev_ids = (id[-2], id[-1])
    for t in range(ids.size):
        t0, t1, t2 = seq[t + 2], seq[t + 1], seq[t]
        for h in range(heads):
            r = _py_ple_row(t0, t1, t2, h, rows, 248044, 0)
            assert np.array_equal(out[t, h * hd:(h + 1) * hd], tables[h][r])
    # no history = (-1, -1): both history slots become EOS
    out2 = orc.ple_gather_f16(tables, ids[:1], prev_ids=None)
    r = _py_ple_row(3, 248044, 248044, 0, rows, 248044, 0)
    assert np.array_equal(out2[0, :hd], tables[0][r])


def test_embed_gather_policies(orc):
    table = RNG.standard_normal((100, 64)).astype(np.float16)
    ids = np.array([0, 5, 99, -1, 100, 7], dtype=np.int32)
    out, bad = orc.embed_gather_rows(table, ids, 0)
    assert bad == 2
    assert np.array_equal(out, table[[0, 5, 99, 0, 99, 7]])
    out, bad = orc.embed_gather_rows(table, ids, 1)
    assert np.array_equal(out, table[[0, 5, 99, 0, 0, 7]])
    bits = RNG.integers(0, 65536, (10, 16), dtype=np.uint16)
    f, _ = orc.embed_gather_bf16_f32(bits, np.array([1, 3], dtype=np.int32))
    assert np.array_equal(f.view(np.uint32), bits[[1, 3]].astype(np.uint32) << 16)


def test_ulp_helper():
    a = np.array([1.0, -0.0, 0.0, 65504], dtype=np.float16)
    b = np.array([1.0009765625, 0.0, 5.96e-08, 65504], dtype=np.float16)
    assert list(f16_ulp_distance(a, b)) == [1, 0, 1, 0]


def _np_q8(v, group=32):
    """Q8_0 per group restated in numpy (round half to even, clamp to +-127); the group max drops NaNs
    (fmaxf) and a NaN product (NaN or infinite input) gives code 0 (__float2int_rn)."""
    g = v.reshape(-1, group).astype(np.float32)
    with np.errstate(invalid="ignore", divide="ignore", over="ignore"):
        am = np.nanmax(np.where(np.isnan(g), 0, np.abs(g)), axis=1).astype(np.float32)
        d = (am / np.float32(127.0)).astype(np.float32)
        inv = np.where(d > 0, np.float32(127.0) / np.where(am > 0, am, 1), 0).astype(np.float32)
        t = (g * inv[:, None]).astype(np.float32)
        q = np.clip(np.rint(np.where(np.isnan(t), 0, t)), -127, 127).astype(np.int8)
    return q.reshape(v.shape), d


def test_q8_paths_against_numpy(orc):
    r = np.random.default_rng(31)
    T, n, hc = 3, 256, 4
    R = r.standard_normal((T * hc, n)).astype(np.float32)
    bo = r.standard_normal((T, n)).astype(np.float32)
    inj = r.standard_normal(T * hc).astype(np.float32)
    w = (1 + 0.02 * r.standard_normal((hc, n))).astype(np.float32)
    xn, q8, s8, _ = orc.gr_norm_q8_f32(R, w, bo, inj, T, n, hc)
    q_np, d_np = _np_q8(xn)
    assert np.array_equal(q8, q_np) and np.array_equal(s8.reshape(-1), d_np)
    g = (3 * r.standard_normal(32 * 50)).astype(np.float32)
    u = r.standard_normal(32 * 50).astype(np.float32)
    g[:32] = 0.0  # an all-zero group: scale 0, codes 0
    q, s = orc.swiglu_q8_f32(g, u)
    q_np, d_np = _np_q8(orc.swiglu(g, u))
    assert np.array_equal(q, q_np) and np.array_equal(s, d_np)
    assert s[0] == 0 and not q[:32].any()


def _np_kv_q8(x):
    """64-element groups: fp16 scale of max/127, codes rint(x / scale) clamped to +-127."""
    g = x.reshape(-1, 64).astype(np.float32)
    sh = (np.abs(g).max(axis=1) / np.float32(127.0)).astype(np.float32).astype(np.float16)
    d = sh.astype(np.float32)
    safe = np.where(d > 0, d, np.float32(1.0))
    q = np.where(d[:, None] > 0, np.clip(np.rint(g / safe[:, None]), -127, 127), 0).astype(np.int8)
    return q.reshape(x.shape), sh.view(np.uint16).reshape(x.shape[:-1] + (x.shape[-1] // 64,))


def _np_ring_cell(p, end, cap):
    if cap <= 8192:
        return (p % cap) if p >= max(0, end - cap) else None
    if p < 4096:
        return p
    return 4096 + (p - 4096) % (cap - 4096) if p >= max(4096, end - (cap - 4096)) else None


@pytest.mark.parametrize("T,base,cap,max_ctx,full", [(40, 5, 16, 40, True), (10, 4090, 8200, 9000, True),
                                                     (5000, 20000, 8200, 30000, False), (6, -3, 64, 100, True)])
def test_kv_append_against_numpy(orc, T, base, cap, max_ctx, full):
    r = np.random.default_rng(T + cap)
    kvd = 128
    k = r.standard_normal((T, kvd)).astype(np.float32)
    v = (3 * r.standard_normal((T, kvd))).astype(np.float32)
    v[0, :64] = 0.0  # an all-zero group: scale 0, codes 0
    c = orc.KvCache(cap, max_ctx, kvd, full)
    orc.kv_append_int8_f32(k, v, T, kvd, base, c)
    w = orc.KvCache(cap, max_ctx, kvd, full)
    kq, ks = _np_kv_q8(k)
    vq, vs = _np_kv_q8(v)
    for t in range(T):
        p = base + t
        if p < 0 or p >= max_ctx:
            continue
        cell = _np_ring_cell(p, base + T, cap)
        if cell is not None:
            w.rkq[cell], w.rks[cell], w.rvq[cell], w.rvs[cell] = kq[t], ks[t], vq[t], vs[t]
        if full:
            w.fkq[p], w.fks[p], w.fvq[p], w.fvs[p] = kq[t], ks[t], vq[t], vs[t]
    names = ["rkq", "rks", "rvq", "rvs"] + (["fkq", "fks", "fvq", "fvs"] if full else [])
    for nm in names:
        assert np.array_equal(getattr(c, nm), getattr(w, nm)), nm
    # past the sink, only the last (ring_cap - 4096) positions of the call land in the ring, and the
    # pinned sink cells stay untouched
    if cap > 8192 and base >= 4096:
        assert not c.rks[:4096].any()
        assert np.count_nonzero(c.rks[4096:, 0]) == min(T, cap - 4096)


def test_hyper_connection_residual_against_float64(orc):
    r = np.random.default_rng(41)
    T, n, hc = 6, 80, 4
    R = r.standard_normal((T * hc, n)).astype(np.float32)
    blk = r.standard_normal((T, n)).astype(np.float32)
    inj = r.standard_normal(T * hc).astype(np.float32)
    gw = 2.0 / (1.0 + np.exp(-inj.astype(np.float64) / hc))
    want = R.astype(np.float64) + np.repeat(blk, hc, axis=0) * gw[:, None]
    np.testing.assert_allclose(orc.gr_write_f32(R, blk, inj, T, n, hc), want, rtol=1e-6, atol=1e-6)
    assert np.array_equal(orc.gr_write_f32(R, blk, None, T, n, hc), R + np.repeat(blk, hc, axis=0))
    xn = r.standard_normal((T, hc, n)).astype(np.float16)
    gg = (2 * r.standard_normal((T, hc, n))).astype(np.float16)
    m32, m16 = orc.hc_mix(xn, gg, T, n, hc)
    w = (xn.astype(np.float64) / (1 + np.exp(-gg.astype(np.float64)))).mean(axis=1)
    np.testing.assert_allclose(m32, w, rtol=1e-5, atol=1e-6)
    assert np.array_equal(m16, m32.astype(np.float16))
    np.testing.assert_array_equal(orc.hc_mix(xn.astype(np.float32), gg.astype(np.float32), T, n, hc), m32)
    lo = (4 * r.standard_normal(1000)).astype(np.float32)
    v = lo.astype(np.float64) * 0.25
    assert_f16_close(orc.silu_scale_f16(lo, 0.25), (v / (1 + np.exp(-v))).astype(np.float16), 1, "silu_scale")


def _py_ple_fp8_row(cur, p1, p0, h, mult, vocab, off, eos=248044):
    m64 = (1 << 64) - 1
    c1 = eos if (p1 < 0 or p1 == eos) else p1
    cut = p1 < 0 or p1 == eos or p0 < 0 or p0 == eos
    c2 = eos if cut else p0
    mixed = ((cur & m64) * mult[0] & m64) ^ (c1 * mult[1] & m64)
    if h >= 8:
        mixed ^= c2 * mult[2] & m64
    return (mixed % vocab[h] + off[h]) & 0xFFFFFFFF


def test_ple_fp8_hash_matches_python(orc):
    hsh = orc.PleFp8Hash()
    assert hsh.rows == 320001446
    mult, vocab, off = ([int(x) for x in a] for a in (hsh.mult, hsh.vocab, hsh.off))
    r = np.random.default_rng(51)
    cases = [(5, 7, 9), (0, -1, -1), (123, 248044, 55), (123, 55, 248044), (-3, 4, 5), (248044, 1, 2),
             (151935, 151934, 151933), (2 ** 31 - 1, 2 ** 31 - 1, 2 ** 31 - 1)]
    cases += [tuple(int(v) for v in r.integers(-2, 248320, 3)) for _ in range(300)]
    for cur, p1, p0 in cases:
        for h in range(16):
            assert orc.ple_fp8_row(cur, p1, p0, h, hsh) == _py_ple_fp8_row(cur, p1, p0, h, mult, vocab, off)


def test_ple_fp8_gather_decode_and_context(orc):
    """Every e4m3 code decodes as torch's float8_e4m3fn times the scale (the NaN codes as signed zero),
    and each token reads the rows its (id, id[-1], id[-2]) context hashes to."""
    import torch

    hsh = orc.PleFp8Hash(vocab=[13, 17, 19, 23, 29, 31, 37, 41, 43, 47, 53, 59, 61, 67, 71, 73])
    rb, scale = 32, 0.37
    table = np.arange(hsh.rows * rb, dtype=np.int64).astype(np.uint8).reshape(hsh.rows, rb)  # every code
    ids = np.array([3, 248044, 9, -1, 11, 12], dtype=np.int32)
    out = orc.ple_gather_fp8_f32(table, rb, scale, hsh, ids, prev_ids=(1, 2))
    dec = torch.from_numpy(table.reshape(-1).copy()).view(torch.float8_e4m3fn).float().numpy()
    dec = np.where((table.reshape(-1) & 0x7F) == 0x7F, np.where(table.reshape(-1) & 0x80, -0.0, 0.0), dec)
    dec = (dec.astype(np.float32) * np.float32(scale)).reshape(hsh.rows, rb)
    seq = [1, 2] + [int(v) for v in ids]
    for t in range(ids.size):
        for h in range(16):
            row = orc.ple_fp8_row(seq[t + 2], seq[t + 1], seq[t], h, hsh)
            got = out[t, h * rb:(h + 1) * rb]
            assert np.array_equal(got.view(np.uint32), dec[row].view(np.uint32)), (t, h)


def test_ple_fp8_decode_matches_reference_plesrc(orc, tmp_path):
    """The oracle's fp8 PLE rows against the reference's own PleSrc (src/wzy_stage_v2.cuh:215-324),
    built from its header into oracle/_ref: the table is written as a GGUF file that PleSrc::open parses
    (scale key, tensor offset), and PleSrc::row decodes the rows the hash names. Bit-exact, including
    the NaN codes (read as signed zero) and subnormals."""
    if not orc.ref_available():
        pytest.skip("oracle/_ref/libwzyref.so not built (needs the reference sources at build time)")
    r = np.random.default_rng(88)
    hsh = orc.PleFp8Hash(vocab=[1009 + 4 * i for i in range(16)])
    table = r.integers(0, 256, (hsh.rows, 160)).astype(np.uint8)
    table[:, 0], table[:, 1], table[:, 2] = 0x7F, 0xFF, 0x03  # NaN codes, a subnormal
    path = tmp_path / "ple-fp8.gguf"
    orc.write_ple_gguf(path, table, 0.6172)
    T = 40
    ids = r.integers(-1, 248320, T).astype(np.int32)
    ids[7] = 248044
    prev = (17, 248044)
    seq = list(prev) + [int(v) for v in ids]
    rows = [orc.ple_fp8_row(seq[t + 2], seq[t + 1], seq[t], h, hsh) for t in range(T) for h in range(16)]
    ref_rows, scale, rb, nrows = orc.ref_ple_src_rows(path, rows)
    assert rb == 160 and nrows == hsh.rows and scale == np.float32(0.6172)
    got = orc.ple_gather_fp8_f32(table, 160, scale, hsh, ids, prev_ids=prev)
    assert np.array_equal(got.reshape(T * 16, 160).view(np.uint32), ref_rows.view(np.uint32))


def test_ple_gate_and_conv_against_numpy(orc):
    r = np.random.default_rng(52)
    T, n, hc = 5, 96, 4
    k = r.standard_normal((T * hc, n)).astype(np.float32)
    q = r.standard_normal((T * hc, n)).astype(np.float32)
    q[1] = -k[1]  # a negative dot product
    v = r.standard_normal((T, n)).astype(np.float32)
    gv = orc.ple_gate_f32(k, q, v, T, n, hc)
    d = (k.astype(np.float64) * q).sum(axis=1) / np.sqrt(n)
    g = 1 / (1 + np.exp(-np.sign(np.where(d == 0, 1, d)) * np.sqrt(np.maximum(np.abs(d), 1e-6))))
    np.testing.assert_allclose(gv, np.repeat(v, hc, axis=0) * g[:, None], rtol=2e-6, atol=1e-7)
    # conv: the sequential restatement equals the time-parallel form, history carried across calls
    hcd = 12
    cw = r.standard_normal((hcd, 4)).astype(np.float32)
    hist = r.standard_normal((hcd, 9)).astype(np.float32)
    for T in (3, 20):
        norm = r.standard_normal((T, hcd)).astype(np.float32)
        gvc = r.standard_normal((T, hcd)).astype(np.float32)
        R = r.standard_normal((T, hcd)).astype(np.float32)
        R2, h2, sn = orc.ple_conv_f32(norm, cw, hist, gvc, R, T, hcd, snaps=True)
        x = np.concatenate([hist.T, norm], axis=0).astype(np.float64)  # x[s + 9]
        acc = sum(cw[:, j] * x[3 * j:3 * j + T] for j in range(4))
        want = R + gvc + acc / (1 + np.exp(-acc))
        np.testing.assert_allclose(R2, want, rtol=1e-5, atol=1e-6)
        assert np.array_equal(h2, x[T:T + 9].T.astype(np.float32))
        for t in range(T):
            assert np.array_equal(sn[t], x[t + 1:t + 10].T.astype(np.float32))
        hist = h2


def test_quant_act_against_numpy(orc):
    r = np.random.default_rng(53)
    x = (3 * r.standard_normal(32 * 40)).astype(np.float32)
    x[64:96] = 0.0
    x[100], x[140], x[200] = np.nan, np.inf, -np.inf  # non-finite inputs: NaN dropped from the max, code 0
    x[256:288] = 127.0 * np.sign(r.standard_normal(32))  # amax 127: t = x exactly, so .5 ties below
    x[257:263] = [2.5, 3.5, -2.5, -0.5, 0.5, 126.5]
    q32, s32, q16, s16 = orc.quant_act_f32(x)
    w32, d32 = _np_q8(x)
    assert np.array_equal(q32, w32) and np.array_equal(s32.view(np.uint32), d32.view(np.uint32))
    assert list(q32[257:263]) == [2, 4, -2, 0, 0, 126]  # round half to even
    w16, d16 = _np_q8(x, 16)
    assert np.array_equal(q16, w16) and np.array_equal(s16.view(np.uint32), d16.view(np.uint32))


def _e2m1_exact(v):
    """Round-to-nearest-even onto {0, .5, 1, 1.5, 2, 3, 4, 6} (saturating), as a code with sign bit 8."""
    from fractions import Fraction

    grid = [Fraction(0), Fraction(1, 2), Fraction(1), Fraction(3, 2), Fraction(2), Fraction(3), Fraction(4),
            Fraction(6)]
    a = abs(Fraction(float(v)))
    if a >= 6:
        code = 7
    else:
        best = min(range(8), key=lambda c: (abs(grid[c] - a), c & 1))  # tie -> even code (mantissa 0)
        code = best
    return code | (8 if np.signbit(v) else 0)


def test_block_format_codecs(orc):
    import torch

    L = orc.lib()
    r = np.random.default_rng(54)
    # e4m3 encode == torch's float8_e4m3fn below the saturation point, including exact ties and subnormals
    steps = np.concatenate([np.arange(0, 16) * 2.0 ** -9, *(np.arange(8, 16) * 2.0 ** (e - 3) for e in range(-6, 9))])
    ties = (steps[:-1] + steps[1:]) / 2
    x = np.concatenate([steps, ties, r.standard_normal(4000) * 10.0 ** r.integers(-4, 3, 4000)]).astype(np.float32)
    x = x[np.abs(x) < 448]
    x = np.concatenate([x, -x])
    got = np.array([L.or_f2e4m3(float(v)) for v in x], dtype=np.uint8)
    want = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(got, want)
    assert L.or_f2e4m3(448.0) == 0x7E and L.or_f2e4m3(1e9) == 0x7E and L.or_f2e4m3(-500.0) == 0xFE
    # e4m3 decode of every non-NaN code == torch
    codes = np.array([c for c in range(256) if (c & 0x7F) != 0x7F], dtype=np.uint8)
    dec = np.array([L.or_e4m32f(int(c)) for c in codes], dtype=np.float32)
    assert np.array_equal(dec, torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy())
    # e2m1 encode == the exact rational rounding, on a dense grid with every tie
    y = np.concatenate([np.arange(-8, 8, 1 / 64), r.uniform(-7, 7, 2000)]).astype(np.float32)
    assert [L.or_f2e2m1(float(v)) for v in y] == [_e2m1_exact(v) for v in y]


def test_block_quantisers_against_numpy(orc):
    L = orc.lib()
    r = np.random.default_rng(55)
    x = (r.standard_normal(32 * 24) * np.repeat(10.0 ** r.uniform(-3, 3, 24), 32)).astype(np.float32)
    x[:32] = 0.0
    q, s = orc.quant_mxfp8(x)
    g = x.reshape(-1, 32)
    am = np.abs(g).max(axis=1)
    # the smallest power-of-two scale X with amax / X <= 448, as an E8M0 byte
    e8 = np.array([0 if a == 0 else 127 + int(np.ceil(np.log2(np.float64(np.float32(a / np.float32(448.0))))))
                   for a in am], dtype=np.uint32)
    inv = ((254 - e8) << 23).astype(np.uint32).view(np.float32)
    want_q = np.array([L.or_f2e4m3(float(v)) for v in (g * inv[:, None]).reshape(-1)], dtype=np.uint8)
    assert np.array_equal(s, e8.astype(np.uint8)) and np.array_equal(q, want_q)
    # nothing saturates: every element decodes within half an e4m3 step (2^-4 relative for normals,
    # 2^-10 of the scale in the subnormal range)
    dec = np.array([L.or_e4m32f(int(c)) for c in q], dtype=np.float64).reshape(-1, 32) / inv[:, None]
    assert np.all(np.abs(dec - g) <= np.maximum(np.abs(g) * 2.0 ** -4, 2.0 ** -10 / inv[:, None]))
    # NVFP4 with a per-tensor scale
    gs = np.float32(37.0)
    q4, s4 = orc.quant_nvfp4(x, gs)
    g16 = x.reshape(-1, 16)
    sc = np.array([L.or_f2e4m3(float(np.float32(np.float32(a * gs) / np.float32(6.0)))) for a in np.abs(g16).max(1)],
                  dtype=np.uint8)
    sf = np.array([L.or_e4m32f(int(c)) for c in sc], dtype=np.float32)
    rr = np.where(sf > 0, gs / np.where(sf > 0, sf, 1), 0).astype(np.float32)
    codes = np.array([L.or_f2e2m1(float(v)) for v in (g16 * rr[:, None]).astype(np.float32).reshape(-1)], np.uint8)
    assert np.array_equal(s4, sc) and np.array_equal(q4, codes[0::2] | (codes[1::2] << 4))


@pytest.mark.parametrize("rows,scols", [(1, 1), (200, 3), (129, 80), (256, 160), (77, 33)])
def test_tiled_scale_layout_helper(rows, scols):
    """The GPU tests' relayout of row-major scales into the 128x4-tiled MMA operand layout (built from
    reshapes) equals the layout's byte formula: tile (row // 128, col // 4) at ((row // 128) *
    ceil(scols / 4) + col // 4) * 512, and (r % 32) * 16 + (r % 128 // 32) * 4 + col % 4 inside it."""
    from test_gpu_kernels import _to_blocked

    sc = (np.arange(rows * scols) % 251).astype(np.uint8).reshape(rows, scols)
    blk = _to_blocked(sc)
    ncb = -(-scols // 4)
    assert blk.size == -(-rows // 128) * 128 * ncb * 4
    r, c = np.meshgrid(np.arange(rows), np.arange(scols), indexing="ij")
    off = ((r // 128) * ncb + c // 4) * 512 + (r % 32) * 16 + (r % 128 // 32) * 4 + c % 4
    assert np.array_equal(blk[off], sc)
    pad = np.ones(blk.size, bool)
    pad[off.reshape(-1)] = False
    assert (blk[pad] == 0xAB).all()
