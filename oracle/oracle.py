"""TEST INFRASTRUCTURE ONLY: numpy/ctypes binding of the CPU oracle (liboracle.so) and of the
reference's own kernels built from its sources (_ref/libwzyref.so).

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg only -- as the checker,
never as the measured or shipped path.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_double, c_float, c_int, c_int32, c_int64, c_uint16, c_uint32, c_void_p

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_PATH = os.path.join(HERE, "liboracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libwzyref.so")

P = c_void_p
_SIGS = {
    "or_h2f": (c_float, [c_uint16]),
    "or_f2h": (c_uint16, [c_float]),
    "or_h2f_array": (None, [P, P, c_int64]),
    "or_f2h_array": (None, [P, P, c_int64]),
    "or_set_threads": (None, [c_int]),
    "or_get_threads": (c_int, []),
    "or_add_rmsnorm_f16": (None, [P, P, P, P, c_int64, c_int, c_float, c_float]),
    "or_time_add_rmsnorm_f16": (None, [P, P, P, P, c_int64, c_int, c_float, c_float, c_int, P]),
    "or_gr_norm_f32": (None, [P, P, P, P, P, P, c_int64, c_int, c_int, c_float]),
    "or_gr_norm_q8_f32": (None, [P, P, P, P, P, P, P, c_int64, c_int, c_int, c_float]),
    "or_swiglu_q8_f32": (None, [P, P, P, P, c_int64]),
    "or_quant_act_f32": (None, [P, P, P, P, P, c_int64]),
    "or_f2e4m3": (ctypes.c_uint8, [c_float]),
    "or_e4m32f": (c_float, [ctypes.c_uint8]),
    "or_f2e2m1": (ctypes.c_uint8, [c_float]),
    "or_quant_mxfp8": (None, [P, P, P, c_int64]),
    "or_quant_nvfp4": (None, [P, P, P, c_float, c_int64]),
    "or_gr_write_f32": (None, [P, P, P, c_int64, c_int, c_int]),
    "or_hc_mix_f16": (None, [P, P, P, P, c_int64, c_int, c_int]),
    "or_hc_mix_f32": (None, [P, P, P, c_int64, c_int, c_int]),
    "or_silu_scale_f16": (None, [P, P, c_int64, c_float]),
    "or_kv_append_int8_f32": (None, [P, P, c_int64, c_int, c_int64, P, P, P, P, P, P, P, P, c_int64, c_int64]),
    "or_ple_fp8_row": (c_uint32, [c_int32, c_int32, c_int32, c_int, P, P, P, c_int32]),
    "or_ple_gather_fp8_f32": (None, [P, c_int, c_float, P, P, P, P, c_int64, POINTER(c_int32), c_int32, P]),
    "or_ple_gate_f32": (None, [P, P, P, P, c_int64, c_int, c_int]),
    "or_ple_conv_f32": (None, [P, P, P, P, P, c_int64, c_int, P]),
    "or_k_rope_kv_append_f16": (
        None, [P, P, P, P, P, c_int64, c_int64, c_int64, c_int, c_int, c_int, c_float, c_float,
               P, P, P, P, P, P, P, P, c_int64, c_int64]),
    "or_head_norm_rope_f16": (
        None, [P, P, P, P, c_int64, c_int64, c_int64, c_int, c_int, c_int64, c_int64, c_int, c_float, c_float]),
    "or_head_norm_rope_f32": (
        None, [P, P, P, P, c_int64, c_int64, c_int64, c_int, c_int, c_int64, c_int64, c_int, c_float, c_float]),
    "or_rope_table": (None, [P, P, c_int64, c_int, c_double]),
    "or_gdn_gated_norm_f16": (None, [P, P, P, P, c_int64, c_int, c_int, c_float, c_float, c_int]),
    "or_gdn_gated_norm_f32": (None, [P, P, P, P, c_int64, c_int, c_int, c_float, c_float, c_int]),
    "or_swiglu_f16": (None, [P, P, P, c_int64]),
    "or_swiglu_f32": (None, [P, P, P, c_int64]),
    "or_swiglu_interleaved_f16": (None, [P, P, c_int64, c_int]),
    "or_swiglu_interleaved_f32": (None, [P, P, c_int64, c_int]),
    "or_embed_gather_rows": (c_uint32, [P, c_int64, c_int64, P, c_int64, P, c_int]),
    "or_embed_gather_bf16_f32": (c_uint32, [P, c_int64, c_int, P, c_int64, P, c_int]),
    "or_ple_row": (c_uint32, [c_int32, c_int32, c_int32, c_int, c_int64, c_int32, c_int]),
    "or_ple_gather_f16": (None, [POINTER(c_void_p), c_int, c_int64, c_int, P, c_int64, POINTER(c_int32), c_int32,
                                 c_int, P]),
}

_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_PATH):
            raise OSError(f"{ORACLE_PATH} is missing: build it with `make -C oracle`")
        L = ctypes.CDLL(ORACLE_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a):
    return a.ctypes.data_as(c_void_p) if a is not None else None


def set_threads(n: int) -> None:
    lib().or_set_threads(n)


def get_threads() -> int:
    return lib().or_get_threads()


# ---- numpy wrappers; fp16 tensors are np.float16 arrays (bit patterns passed as uint16) --------
def add_rmsnorm_f16(x, res, w, eps=1e-6, w_offset=1.0):
    """Returns (y, res_out); inputs are not modified."""
    res_out = np.array(res, dtype=np.float16, copy=True)
    y = np.empty_like(res_out)
    T, n = res_out.shape
    xx = np.ascontiguousarray(x, dtype=np.float16) if x is not None else None
    lib().or_add_rmsnorm_f16(_p(xx), _p(res_out), _p(np.ascontiguousarray(w, dtype=np.float16)), _p(y), T, n, eps,
                             w_offset)
    return y, res_out


def time_add_rmsnorm_f16(x, res, w, reps, eps=1e-6, w_offset=1.0):
    """Per-call wall times (ns) of `reps` scalar add + RMSNorm calls on the calling thread (res is updated
    in place every call, as the decode step does)."""
    T, n = res.shape
    samples = np.empty(reps, dtype=np.float64)
    lib().or_time_add_rmsnorm_f16(_p(np.ascontiguousarray(x, np.float16)), _p(res),
                                  _p(np.ascontiguousarray(w, np.float16)), _p(np.empty_like(res)), T, n, eps,
                                  w_offset, reps, _p(samples))
    return samples


def gr_norm_f32(R, w, bo, inj, T, n, hc, eps=1e-6):
    """fp32 hyper-connection norm; returns (xn_f32, xn_f16, R_out)."""
    R_out = np.array(R, dtype=np.float32, copy=True)
    xn = np.empty((T * hc, n), dtype=np.float32)
    xh = np.empty((T * hc, n), dtype=np.float16)
    lib().or_gr_norm_f32(_p(R_out), _p(np.ascontiguousarray(w, np.float32)),
                         _p(np.ascontiguousarray(bo, np.float32)) if bo is not None else None,
                         _p(np.ascontiguousarray(inj, np.float32)) if inj is not None else None,
                         _p(xn), _p(xh), T, n, hc, eps)
    return xn, xh, R_out


def gr_norm_q8_f32(R, w, bo, inj, T, n, hc, eps=1e-6):
    """fp32 hyper-connection norm with the Q8_0 side output; returns (xn, q8, s8, R_out)."""
    R_out = np.array(R, dtype=np.float32, copy=True)
    xn = np.empty((T * hc, n), dtype=np.float32)
    q8 = np.empty((T * hc, n), dtype=np.int8)
    s8 = np.empty((T * hc, n // 32), dtype=np.float32)
    lib().or_gr_norm_q8_f32(_p(R_out), _p(np.ascontiguousarray(w, np.float32)),
                            _p(np.ascontiguousarray(bo, np.float32)) if bo is not None else None,
                            _p(np.ascontiguousarray(inj, np.float32)) if inj is not None else None,
                            _p(xn), _p(q8), _p(s8), T, n, hc, eps)
    return xn, q8, s8, R_out


def swiglu_q8_f32(g, u):
    g = np.ascontiguousarray(g, np.float32)
    u = np.ascontiguousarray(u, np.float32)
    q = np.empty(g.size, dtype=np.int8)
    s = np.empty(g.size // 32, dtype=np.float32)
    lib().or_swiglu_q8_f32(_p(g), _p(u), _p(q), _p(s), g.size)
    return q, s


def quant_act_f32(x, q32=True, q16=True):
    """(q32, s32, q16, s16) of the flat fp32 array x (None where not asked for)."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    a = (np.empty(x.size, np.int8), np.empty(x.size // 32, np.float32)) if q32 else (None, None)
    b = (np.empty(x.size, np.int8), np.empty(x.size // 16, np.float32)) if q16 else (None, None)
    lib().or_quant_act_f32(_p(x), _p(a[0]) if q32 else None, _p(a[1]) if q32 else None, _p(b[0]) if q16 else None,
                           _p(b[1]) if q16 else None, x.size)
    return a[0], a[1], b[0], b[1]


def quant_mxfp8(x):
    """MXFP8 of the flat fp32 array x: (e4m3 code bytes [n], E8M0 scale bytes [n/32])."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    q, sc = np.empty(x.size, np.uint8), np.empty(x.size // 32, np.uint8)
    lib().or_quant_mxfp8(_p(x), _p(q), _p(sc), x.size)
    return q, sc


def quant_nvfp4(x, gs=1.0):
    """NVFP4 of the flat fp32 array x: (e2m1 pairs [n/2], e4m3 scale bytes [n/16])."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    q, sc = np.empty(x.size // 2, np.uint8), np.empty(x.size // 16, np.uint8)
    lib().or_quant_nvfp4(_p(x), _p(q), _p(sc), gs, x.size)
    return q, sc


def gr_write_f32(R, blk, inj, T, n, hc):
    """R [T*hc, n] + blk[t] * 2*sigmoid(inj/hc) (gate 1.0 with inj None); returns the new R."""
    out = np.array(R, dtype=np.float32, copy=True)
    lib().or_gr_write_f32(_p(out), _p(np.ascontiguousarray(blk, np.float32)),
                          _p(np.ascontiguousarray(inj, np.float32)) if inj is not None else None, T, n, hc)
    return out


def hc_mix(xn, gg, T, n, hc):
    """Stream mixing; fp16 inputs give (mixed fp32, mixed fp16), fp32 inputs give mixed fp32."""
    mixed = np.empty((T, n), dtype=np.float32)
    if xn.dtype == np.float16:
        m16 = np.empty((T, n), dtype=np.float16)
        lib().or_hc_mix_f16(_p(np.ascontiguousarray(xn)), _p(np.ascontiguousarray(gg)), _p(mixed), _p(m16), T, n, hc)
        return mixed, m16
    lib().or_hc_mix_f32(_p(np.ascontiguousarray(xn, np.float32)), _p(np.ascontiguousarray(gg, np.float32)),
                        _p(mixed), T, n, hc)
    return mixed


def silu_scale_f16(lo, scale):
    lo = np.ascontiguousarray(lo, np.float32)
    out = np.empty(lo.shape, dtype=np.float16)
    lib().or_silu_scale_f16(_p(lo), _p(out), lo.size, scale)
    return out


def rope_table(rows, rot=64, theta=1e7):
    half = rot // 2
    c = np.empty((rows, half), dtype=np.float32)
    s = np.empty((rows, half), dtype=np.float32)
    lib().or_rope_table(_p(c), _p(s), rows, rot, theta)
    return c, s


def head_norm_rope(data, gamma, cos_tab, sin_tab, T, heads, hd, head_stride, row_stride, rot=64, eps=1e-6,
                   w_offset=0.0, base_pos=0):
    """In-place op on a copy of `data` (fp16 or fp32 flat array); returns the copy."""
    out = np.array(data, copy=True)
    rows = cos_tab.shape[0] if cos_tab is not None else 0
    fn = lib().or_head_norm_rope_f16 if out.dtype == np.float16 else lib().or_head_norm_rope_f32
    fn(_p(out), _p(np.ascontiguousarray(gamma, out.dtype)), _p(cos_tab), _p(sin_tab), rows, base_pos, T, heads, hd,
       head_stride, row_stride, rot, eps, w_offset)
    return out


class KvCache:
    """Host INT8 KV cache: ring [ring_cap, kvd] codes + [ring_cap, kvd/64] fp16 scale bits, and an
    optional full-context mirror [max_ctx, ...]. Cells start zeroed."""

    def __init__(self, ring_cap, max_ctx, kvd, full=True):
        self.ring_cap, self.max_ctx, self.kvd = ring_cap, max_ctx, kvd
        self.rkq = np.zeros((ring_cap, kvd), np.int8)
        self.rvq = np.zeros((ring_cap, kvd), np.int8)
        self.rks = np.zeros((ring_cap, kvd // 64), np.uint16)
        self.rvs = np.zeros((ring_cap, kvd // 64), np.uint16)
        self.full = full
        if full:
            self.fkq = np.zeros((max_ctx, kvd), np.int8)
            self.fvq = np.zeros((max_ctx, kvd), np.int8)
            self.fks = np.zeros((max_ctx, kvd // 64), np.uint16)
            self.fvs = np.zeros((max_ctx, kvd // 64), np.uint16)

    def args(self):
        f = (lambda a: _p(a)) if self.full else (lambda a: None)
        return [_p(self.rkq), _p(self.rks), _p(self.rvq), _p(self.rvs),
                f(getattr(self, "fkq", None)), f(getattr(self, "fks", None)), f(getattr(self, "fvq", None)),
                f(getattr(self, "fvs", None)), self.ring_cap, self.max_ctx]


def kv_append_int8_f32(k, v, T, kvd, base_pos, cache: KvCache):
    lib().or_kv_append_int8_f32(_p(np.ascontiguousarray(k, np.float32)), _p(np.ascontiguousarray(v, np.float32)), T,
                                kvd, base_pos, *cache.args())


def k_rope_kv_append(k, gamma, v, cos_tab, sin_tab, T, kv_heads, hd, rot, eps, w_offset, base_pos, cache: KvCache):
    """k normalised + rotated (returned as a new array) and k, v appended to `cache`."""
    kvd = kv_heads * hd
    rows = cos_tab.shape[0] if cos_tab is not None else 0
    if k.dtype == np.float16:
        out = np.array(k, copy=True)
        lib().or_k_rope_kv_append_f16(_p(out), _p(np.ascontiguousarray(gamma, np.float16)),
                                      _p(np.ascontiguousarray(v, np.float16)), _p(cos_tab), _p(sin_tab), rows, base_pos,
                                      T, kv_heads, hd, rot, eps, w_offset, *cache.args())
        return out
    out = head_norm_rope(np.ascontiguousarray(k, np.float32).reshape(-1), gamma, cos_tab, sin_tab, T, kv_heads, hd, hd,
                         kvd, rot, eps, w_offset, base_pos)
    kv_append_int8_f32(out, v, T, kvd, base_pos, cache)
    return out.reshape(k.shape)


def gdn_gated_norm(o, z, gamma, T, heads, hd=128, eps=1e-6, w_offset=0.0, gate_mode=0):
    if o.dtype == np.float16:
        y = np.empty(o.shape, dtype=np.float16)
        lib().or_gdn_gated_norm_f16(_p(o), _p(z), _p(np.ascontiguousarray(gamma, np.float16)), _p(y), T, heads, hd,
                                    eps, w_offset, gate_mode)
    else:
        y = np.empty(o.shape, dtype=np.float32)
        lib().or_gdn_gated_norm_f32(_p(o), _p(z), _p(np.ascontiguousarray(gamma, np.float32)), _p(y), T, heads, hd,
                                    eps, w_offset, gate_mode)
    return y


def swiglu(g, u):
    out = np.empty(g.shape, dtype=g.dtype)
    fn = lib().or_swiglu_f16 if g.dtype == np.float16 else lib().or_swiglu_f32
    fn(_p(np.ascontiguousarray(g)), _p(np.ascontiguousarray(u)), _p(out), g.size)
    return out


def swiglu_interleaved(gu, T, nff):
    out = np.empty((T, nff), dtype=gu.dtype)
    fn = lib().or_swiglu_interleaved_f16 if gu.dtype == np.float16 else lib().or_swiglu_interleaved_f32
    fn(_p(np.ascontiguousarray(gu)), _p(out), T, nff)
    return out


def embed_gather_rows(table, ids, oob_policy=0):
    vocab = table.shape[0]
    row_bytes = table[0].nbytes
    out = np.empty((ids.size,) + table.shape[1:], dtype=table.dtype)
    bad = lib().or_embed_gather_rows(_p(np.ascontiguousarray(table)), vocab, row_bytes,
                                     _p(np.ascontiguousarray(ids, np.int32)), ids.size, _p(out), oob_policy)
    return out, int(bad)


def embed_gather_bf16_f32(table_bits, ids, oob_policy=0):
    vocab, hidden = table_bits.shape
    out = np.empty((ids.size, hidden), dtype=np.float32)
    bad = lib().or_embed_gather_bf16_f32(_p(np.ascontiguousarray(table_bits, np.uint16)), vocab, hidden,
                                         _p(np.ascontiguousarray(ids, np.int32)), ids.size, _p(out), oob_policy)
    return out, int(bad)


def ple_row(t0, t1, t2, head, rows, eos=248044, variant=0) -> int:
    return int(lib().or_ple_row(t0, t1, t2, head, rows, eos, variant))


def ple_gather_f16(tables, ids, prev_ids=None, eos=248044, variant=0):
    heads = len(tables)
    rows, hd = tables[0].shape
    arr = (c_void_p * heads)(*[t.ctypes.data for t in tables])
    prev = (c_int32 * 2)(*prev_ids) if prev_ids is not None else None
    ids = np.ascontiguousarray(ids, np.int32)
    out = np.empty((ids.size, heads * hd), dtype=np.float16)
    lib().or_ple_gather_f16(arr, heads, rows, hd, _p(ids), ids.size, prev, eos, variant, _p(out))
    return out


class PleFp8Hash:
    """mult[3], vocab[16], off[16] as uint64 arrays (the reference's by default)."""

    REF_VOCAB = [20000003, 20000023, 20000033, 20000047, 20000059, 20000063, 20000069, 20000077,
                 20000081, 20000093, 20000107, 20000147, 20000153, 20000159, 20000161, 20000171]
    REF_MULT = [23703573157769, 20109073645365, 8052911324071]

    def __init__(self, vocab=None, mult=None):
        self.vocab = np.array(vocab if vocab is not None else self.REF_VOCAB, dtype=np.uint64)
        self.mult = np.array(mult if mult is not None else self.REF_MULT, dtype=np.uint64)
        self.off = np.concatenate([[0], np.cumsum(self.vocab)[:-1]]).astype(np.uint64)

    @property
    def rows(self):
        return int(self.off[-1] + self.vocab[-1])


def ple_fp8_row(cur, p1, p0, h, hsh: PleFp8Hash, eos=248044):
    return lib().or_ple_fp8_row(cur, p1, p0, h, _p(hsh.mult), _p(hsh.vocab), _p(hsh.off), eos)


def ple_gather_fp8_f32(table, row_bytes, scale, hsh: PleFp8Hash, ids, prev_ids=None, eos=248044):
    ids = np.ascontiguousarray(ids, np.int32)
    prev = (c_int32 * 2)(*prev_ids) if prev_ids is not None else None
    out = np.empty((ids.size, 16 * row_bytes), dtype=np.float32)
    lib().or_ple_gather_fp8_f32(_p(np.ascontiguousarray(table, np.uint8)), row_bytes, scale, _p(hsh.mult),
                                _p(hsh.vocab), _p(hsh.off), _p(ids), ids.size, prev, eos, _p(out))
    return out


def ple_gate_f32(key, query, value, T, n, hc):
    gv = np.empty((T * hc, n), dtype=np.float32)
    lib().or_ple_gate_f32(_p(np.ascontiguousarray(key, np.float32)), _p(np.ascontiguousarray(query, np.float32)),
                          _p(np.ascontiguousarray(value, np.float32)), _p(gv), T, n, hc)
    return gv


def ple_conv_f32(norm, cw, hist, gv, R, T, hcd, snaps=False):
    """Returns (R', hist', snaps or None); inputs are not modified."""
    R2 = np.array(R, dtype=np.float32, copy=True)
    h2 = np.array(hist, dtype=np.float32, copy=True)
    sn = np.zeros((T, hcd, 9), dtype=np.float32) if snaps else None
    lib().or_ple_conv_f32(_p(np.ascontiguousarray(norm, np.float32)), _p(np.ascontiguousarray(cw, np.float32)),
                          _p(h2), _p(np.ascontiguousarray(gv, np.float32)), _p(R2), T, hcd,
                          _p(sn) if snaps else None)
    return R2, h2, sn


# ---- the reference's own kernels (GPU) and host table builder --------------------------------
_ref = None


def ref_available() -> bool:
    return os.path.exists(REF_PATH)


def ref_lib() -> ctypes.CDLL:
    global _ref
    if _ref is None:
        L = ctypes.CDLL(REF_PATH)
        I = c_int
        F = c_float
        sigs = {
            "ref_fused_gr_norm_multi": [P, P, P, P, P, I, I, I, F, P],
            "ref_fused_gr_norm_multi_q8": [P, P, P, P, P, P, P, I, I, I, F, P],
            "ref_silu_mul_quant32_multi": [P, P, P, P, I, P],
            "ref_pf_gr_norm_fp16": [P, P, P, P, P, I, I, I, F, P],
            "ref_gr_write_multi": [P, P, P, I, I, I, P],
            "ref_pf_gr_up_mean_fp16": [P, P, P, P, I, I, P],
            "ref_quant_act_multi": [P, P, P, P, P, I, I, P],
            "ref_kv_append_int8_multi": [P, P, P, P, P, P, P, P, P, P, P, I, I, I, P],
            "ref_ple_gate_gv_multi": [P, P, P, P, I, I, I, P],
            "ref_ple_conv_multi": [P, P, P, P, P, I, I, P, P],
            "ref_gr_up_gate_mean_pf": [P, P, P, I, I, P],
            "ref_silu_div_hc_to_fp16": [P, P, I, F, P],
            "ref_fused_head_norm_rope_multi": [P, P, P, P, P, I, I, I, I, I, F, P],
            "ref_pf_gdn_rmsnorm_gate_parallel": [P, P, P, P, I, I, F, P],
            "ref_silu_mul_multi": [P, P, P, I, P],
            "ref_pf_silu_mul_interleaved_to_fp16": [P, P, I, I, P],
            "ref_mtp_gather_bf16_emb": [P, P, P, I, P],
            "ref_ple_group_multi": [P, P, P, I, I, I, F, P],
        }
        for name, args in sigs.items():
            fn = getattr(L, name)
            fn.restype = c_int
            fn.argtypes = args
        L.ref_build_rope_cos_sin_host.restype = None
        L.ref_build_rope_cos_sin_host.argtypes = [I, F, P, P]
        L.ref_ple_src_rows.restype = c_int
        L.ref_ple_src_rows.argtypes = [ctypes.c_char_p, P, I, P, POINTER(c_float), POINTER(c_int),
                                       POINTER(ctypes.c_uint64)]
        L.ref_dims.restype = c_int
        L.ref_dims.argtypes = [POINTER(c_int), POINTER(c_int)]
        _ref = L
    return _ref


def write_ple_gguf(path, table, scale):
    """A minimal GGUF file as the reference's PleSrc::open reads it (src/wzy_stage_v2.cuh:228-283):
    magic, version, one key "strata.ple.scale" (float32), one tensor "per_layer_token_embd.weight" of
    dims [row_bytes, rows] at offset 0, data aligned to 32 bytes."""
    import struct

    table = np.ascontiguousarray(table, np.uint8)
    rows, rb = table.shape

    def gstr(x):
        b = x.encode()
        return struct.pack("<Q", len(b)) + b

    head = b"GGUF" + struct.pack("<I", 3) + struct.pack("<QQ", 1, 1)
    head += gstr("strata.ple.scale") + struct.pack("<I", 6) + struct.pack("<f", scale)
    head += gstr("per_layer_token_embd.weight") + struct.pack("<I", 2) + struct.pack("<QQ", rb, rows)
    head += struct.pack("<I", 0) + struct.pack("<Q", 0)
    pad = (-len(head)) % 32
    with open(path, "wb") as f:
        f.write(head + b"\0" * pad)
        f.write(table.tobytes())


def ref_ple_src_rows(path, rows_idx):
    """The reference's PleSrc decode of the given rows: (floats [n, row_bytes], scale, row_bytes, rows)."""
    idx = np.ascontiguousarray(rows_idx, np.uint64)
    out = np.empty((idx.size, 160), dtype=np.float32)
    sc, rb, nr = c_float(), c_int(), ctypes.c_uint64()
    rc = ref_lib().ref_ple_src_rows(str(path).encode(), _p(idx), idx.size, _p(out), ctypes.byref(sc),
                                    ctypes.byref(rb), ctypes.byref(nr))
    assert rc == 0, "PleSrc::open rejected the file"
    return out, sc.value, rb.value, nr.value


def ref_rope_table(rows, theta=1e7):
    """The reference's own host builder (32 pairs = rot 64)."""
    c = np.empty((rows, 32), dtype=np.float32)
    s = np.empty((rows, 32), dtype=np.float32)
    ref_lib().ref_build_rope_cos_sin_host(rows, theta, _p(c), _p(s))
    return c, s
