"""ctypes binding of libwzyb200.so, the C ABI declared in include/wzyb200.h.

The kernels, their launchers and the host-side executor are native (CUDA/C++ in csrc/). This module
only loads the shared library, declares the entry points, and offers thin wrappers that take torch
tensors (torch is used for device memory and streams) and raise on a non-zero status.

There is no fallback: if the library is missing or the device is not an sm_100 GPU the calls raise.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_double, c_float, c_int, c_int32, c_int64, c_uint32, c_void_p

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libwzyb200.so")
HEADER_PATH = os.path.join(os.path.dirname(HERE), "include", "wzyb200.h")

OK = 0
ERR_NULL, ERR_ALIGN, ERR_SHAPE, ERR_DEVICE, ERR_VALUE = -1, -2, -3, -4, -5
FAULT_WAIT_TIMEOUT, FAULT_POS_RANGE = 0x1, 0x2
GATE_SIGMOID, GATE_SILU = 0, 1
OOB_CLAMP, OOB_ZERO_ID = 0, 1
PLE_HASH_C_PRECEDENCE, PLE_HASH_XOR_THEN_ADD = 0, 1
PLE_EOS_DEFAULT = 248044
FAM_NORM, FAM_HEAD_ROPE, FAM_GDN, FAM_SWIGLU, FAM_GATHER, FAM_BUNDLE, FAM_KV = 0, 1, 2, 3, 4, 5, 6
VARIANT_AUTO, VARIANT_RING, VARIANT_DIRECT, VARIANT_ASYNC, VARIANT_WIDE, VARIANT_PAIR = 0, 1, 2, 3, 4, 5
VARIANT_SPLIT = 6


class WzybError(RuntimeError):
    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} returned {code}: {msg}")
        self.code = code


class KvCache(ctypes.Structure):
    """wzyb_kv_cache: INT8 ring (and optional full-context mirror) codes and fp16 scale bits."""
    _fields_ = [
        ("ring_k_q", c_void_p),
        ("ring_k_s", c_void_p),
        ("ring_v_q", c_void_p),
        ("ring_v_s", c_void_p),
        ("full_k_q", c_void_p),
        ("full_k_s", c_void_p),
        ("full_v_q", c_void_p),
        ("full_v_s", c_void_p),
        ("ring_cap", c_int64),
        ("max_ctx", c_int64),
    ]


class PleFp8Hash(ctypes.Structure):
    """wzyb_ple_fp8_hash: n-gram multipliers and the 16 heads' sub-table sizes and offsets."""
    _fields_ = [("mult", ctypes.c_uint64 * 3), ("vocab", ctypes.c_uint64 * 16), ("off", ctypes.c_uint64 * 16)]


class HeadTensor(ctypes.Structure):
    _fields_ = [
        ("data", c_void_p),
        ("gamma", c_void_p),
        ("heads", c_int),
        ("head_stride", c_int64),
        ("row_stride", c_int64),
    ]


class AttnPrepArgs(ctypes.Structure):
    _fields_ = [
        ("x", c_void_p),
        ("residual", c_void_p),
        ("norm_weight", c_void_p),
        ("normed", c_void_p),
        ("hidden", c_int),
        ("q", HeadTensor),
        ("k", HeadTensor),
        ("head_dim", c_int),
        ("rot_dims", c_int),
        ("cos_tab", c_void_p),
        ("sin_tab", c_void_p),
        ("table_rows", c_int64),
        ("d_base_pos", c_void_p),
        ("pos_offset", c_int64),
        ("eps", c_float),
        ("w_offset", c_float),
    ]


class ActArgs(ctypes.Structure):
    _fields_ = [
        ("gate", c_void_p),
        ("up", c_void_p),
        ("act", c_void_p),
        ("act_rows", c_int64),
        ("ffn", c_int),
        ("o", c_void_p),
        ("z", c_void_p),
        ("gdn_gamma", c_void_p),
        ("gdn_out", c_void_p),
        ("gdn_heads", c_int),
        ("gdn_head_dim", c_int),
        ("eps", c_float),
        ("gdn_w_offset", c_float),
        ("gate_mode", c_int),
    ]


class EmbedPleArgs(ctypes.Structure):
    _fields_ = [
        ("ids", c_void_p),
        ("table", c_void_p),
        ("vocab", c_int64),
        ("hidden", c_int),
        ("oob_policy", c_int),
        ("d_oob_count", c_void_p),
        ("emb_out", c_void_p),
        ("ple_tables", POINTER(c_void_p)),
        ("ple_heads", c_int),
        ("ple_rows", c_int64),
        ("ple_head_dim", c_int),
        ("prev_ids", POINTER(c_int32)),
        ("eos_id", c_int32),
        ("hash_variant", c_int),
        ("ple_out", c_void_p),
    ]


P = c_void_p
S = c_void_p  # cudaStream_t
_SIGS = {
    "wzyb_add_rmsnorm_f16": (c_int, [P, P, P, P, c_int64, c_int, c_float, c_float, S]),
    "wzyb_gr_norm_f32": (c_int, [P, P, P, P, P, c_int64, c_int, c_int, c_float, S]),
    "wzyb_gr_norm_f32_f16": (c_int, [P, P, P, P, P, c_int64, c_int, c_int, c_float, S]),
    "wzyb_gr_norm_q8_f32": (c_int, [P, P, P, P, P, P, P, c_int64, c_int, c_int, c_float, S]),
    "wzyb_swiglu_q8_f32": (c_int, [P, P, P, P, c_int64, S]),
    "wzyb_quant_act_f32": (c_int, [P, P, P, P, P, c_int64, c_int, S]),
    "wzyb_quant_act_mxfp8_f32": (c_int, [P, P, P, c_int64, c_int, S]),
    "wzyb_quant_act_block_f32": (c_int, [P, P, P, c_int, c_int, c_float, c_int64, c_int, S]),
    "wzyb_swiglu_block_f32": (c_int, [P, P, P, P, c_int, c_int, c_float, c_int64, c_int, S]),
    "wzyb_gr_norm_block_f32": (c_int, [P, P, P, P, P, P, P, c_int, c_int, c_float, c_int64, c_int, c_int, c_float, S]),
    "wzyb_quant_act_nvfp4_f32": (c_int, [P, P, P, c_float, c_int64, c_int, S]),
    "wzyb_swiglu_mxfp8_f32": (c_int, [P, P, P, P, c_int64, S]),
    "wzyb_swiglu_nvfp4_f32": (c_int, [P, P, P, P, c_float, c_int64, S]),
    "wzyb_gr_norm_mxfp8_f32": (c_int, [P, P, P, P, P, P, P, c_int64, c_int, c_int, c_float, S]),
    "wzyb_gr_norm_nvfp4_f32": (c_int, [P, P, P, P, P, P, P, c_float, c_int64, c_int, c_int, c_float, S]),
    "wzyb_gr_write_f32": (c_int, [P, P, P, c_int64, c_int, c_int, S]),
    "wzyb_hc_mix_f16": (c_int, [P, P, P, P, c_int64, c_int, c_int, S]),
    "wzyb_hc_mix_f32": (c_int, [P, P, P, c_int64, c_int, c_int, S]),
    "wzyb_silu_scale_f16": (c_int, [P, P, c_int64, c_float, S]),
    "wzyb_kv_append_int8_f32": (c_int, [P, P, c_int64, c_int, c_int, P, c_int64, POINTER(KvCache), S]),
    "wzyb_ple_fp8_reference_hash": (c_int, [POINTER(PleFp8Hash)]),
    "wzyb_ple_gather_fp8_f32": (
        c_int, [P, c_int64, c_int, c_float, POINTER(PleFp8Hash), P, c_int64, POINTER(c_int32), c_int32, P, S]),
    "wzyb_ple_gate_f32": (c_int, [P, P, P, P, c_int64, c_int, c_int, S]),
    "wzyb_ple_conv_f32": (c_int, [P, P, P, P, P, c_int64, c_int, P, S]),
    "wzyb_k_rope_kv_append_f32": (
        c_int,
        [P, P, P, P, P, c_int64, P, c_int64, c_int64, c_int, c_int, c_int, c_float, c_float, POINTER(KvCache), S],
    ),
    "wzyb_k_rope_kv_append_f16": (
        c_int,
        [P, P, P, P, P, c_int64, P, c_int64, c_int64, c_int, c_int, c_int, c_float, c_float, POINTER(KvCache), S],
    ),
    "wzyb_qk_rope_kv_append_f32": (
        c_int,
        [POINTER(HeadTensor), P, P, P, P, P, c_int64, P, c_int64, c_int64, c_int, c_int, c_int, c_float, c_float,
         POINTER(KvCache), S],
    ),
    "wzyb_qk_rope_kv_append_f16": (
        c_int,
        [POINTER(HeadTensor), P, P, P, P, P, c_int64, P, c_int64, c_int64, c_int, c_int, c_int, c_float, c_float,
         POINTER(KvCache), S],
    ),
    "wzyb_head_norm_rope_f16": (
        c_int,
        [P, P, P, P, c_int64, P, c_int64, c_int64, c_int, c_int, c_int64, c_int64, c_int, c_float, c_float, S],
    ),
    "wzyb_head_norm_rope_f32": (
        c_int,
        [P, P, P, P, c_int64, P, c_int64, c_int64, c_int, c_int, c_int64, c_int64, c_int, c_float, c_float, S],
    ),
    "wzyb_qk_norm_rope_f16": (
        c_int,
        [POINTER(HeadTensor), POINTER(HeadTensor), P, P, c_int64, P, c_int64, c_int64, c_int, c_int, c_float,
         c_float, S],
    ),
    "wzyb_rope_table_host_f32": (c_int, [P, P, c_int64, c_int, c_double]),
    "wzyb_rope_table_f32": (c_int, [P, P, c_int64, c_int, c_double, S]),
    "wzyb_gdn_gated_norm_f16": (c_int, [P, P, P, P, c_int64, c_int, c_int, c_float, c_float, c_int, S]),
    "wzyb_gdn_gated_norm_f32_f16": (c_int, [P, P, P, P, c_int64, c_int, c_int, c_float, c_float, c_int, S]),
    "wzyb_swiglu_f16": (c_int, [P, P, P, c_int64, S]),
    "wzyb_swiglu_f32": (c_int, [P, P, P, c_int64, S]),
    "wzyb_swiglu_interleaved_f16": (c_int, [P, P, c_int64, c_int, S]),
    "wzyb_swiglu_interleaved_f32_f16": (c_int, [P, P, c_int64, c_int, S]),
    "wzyb_embed_gather_rows": (c_int, [P, c_int64, c_int64, P, c_int64, P, c_int, P, S]),
    "wzyb_embed_gather_f16": (c_int, [P, c_int64, c_int, P, c_int64, P, c_int, P, S]),
    "wzyb_embed_gather_bf16_f32": (c_int, [P, c_int64, c_int, P, c_int64, P, c_int, P, S]),
    "wzyb_ple_gather_f16": (
        c_int,
        [POINTER(c_void_p), c_int, c_int64, c_int, P, c_int64, POINTER(c_int32), c_int32, c_int, P, S],
    ),
    "wzyb_ple_row_index": (c_uint32, [c_int32, c_int32, c_int32, c_int, c_int64, c_int32, c_int]),
    "wzyb_attn_prep_f16": (c_int, [POINTER(AttnPrepArgs), c_int64, S]),
    "wzyb_act_f16": (c_int, [POINTER(ActArgs), c_int64, S]),
    "wzyb_embed_ple_f16": (c_int, [POINTER(EmbedPleArgs), c_int64, S]),
    "wzyb_shard_rows": (c_int, [c_int64, c_int, c_int, POINTER(c_int64), POINTER(c_int64)]),
    "wzyb_ple_halo": (c_int, [POINTER(c_int32), c_int64, POINTER(c_int32), POINTER(c_int32)]),
    "wzyb_prepare_device": (c_int, []),
    "wzyb_read_faults": (c_int, [POINTER(c_uint32), c_int]),
    "wzyb_set_launch_tuning": (c_int, [c_int, c_int, c_int]),
    "wzyb_set_kernel_variant": (c_int, [c_int, c_int]),
    "wzyb_status_string": (ctypes.c_char_p, [c_int]),
    "wzyb_version": (c_int, []),
}

_lib = None


def lib() -> ctypes.CDLL:
    """Load libwzyb200.so once (raises OSError when it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"{LIB_PATH} is missing: build it with `make -C wzy-flash-serve_b200`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def status_string(code: int) -> str:
    return lib().wzyb_status_string(code).decode()


def check(fn: str, code: int) -> None:
    if code != OK:
        raise WzybError(fn, code, status_string(code))


def call(fn: str, *args) -> None:
    """Call an int-returning entry point and raise WzybError on a non-zero status."""
    check(fn, getattr(lib(), fn)(*args))


# ------------------------------------------------------------------------------------------------
# torch-tensor wrappers (device pointers + the current stream)
# ------------------------------------------------------------------------------------------------
def _stream(stream=None):
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return c_void_p(s.cuda_stream)


def _ptr(t):
    return c_void_p(t.data_ptr()) if t is not None else c_void_p(0)


def add_rmsnorm_f16(x, residual, weight, y, eps=1e-6, w_offset=1.0, stream=None):
    T, hidden = residual.shape
    call("wzyb_add_rmsnorm_f16", _ptr(x), _ptr(residual), _ptr(weight), _ptr(y), T, hidden, eps, w_offset,
         _stream(stream))


def gr_norm_f32(R, w_norm, bo_prev, inj_prev, xn, T, n_embd, hc, eps=1e-6, stream=None):
    fn = "wzyb_gr_norm_f32" if xn.element_size() == 4 else "wzyb_gr_norm_f32_f16"
    call(fn, _ptr(R), _ptr(w_norm), _ptr(bo_prev), _ptr(inj_prev), _ptr(xn), T, n_embd, hc, eps, _stream(stream))


def gr_norm_q8_f32(R, w_norm, bo_prev, inj_prev, xn, xq8, xs8, T, n_embd, hc, eps=1e-6, stream=None):
    call("wzyb_gr_norm_q8_f32", _ptr(R), _ptr(w_norm), _ptr(bo_prev), _ptr(inj_prev), _ptr(xn), _ptr(xq8), _ptr(xs8),
         T, n_embd, hc, eps, _stream(stream))


def swiglu_q8_f32(gate, up, q32, s32, stream=None):
    call("wzyb_swiglu_q8_f32", _ptr(gate), _ptr(up), _ptr(q32), _ptr(s32), gate.numel(), _stream(stream))


def quant_act_f32(x, q32, s32, q16, s16, T, cols, stream=None):
    """int8 per-32 (q32/s32) and/or per-16 (q16/s16) quantisation of fp32 rows x [T, cols]."""
    call("wzyb_quant_act_f32", _ptr(x), _ptr(q32), _ptr(s32), _ptr(q16), _ptr(s16), T, cols, _stream(stream))


BLOCK_MXFP8, BLOCK_NVFP4 = 0, 1
SF_ROW_MAJOR, SF_TILED_128X4 = 0, 1


def sf_tiled_bytes(rows, cols, fmt="mxfp8"):
    """Bytes of a tiled-128x4 scale buffer for codes [rows, cols]."""
    scols = cols // (32 if fmt == "mxfp8" else 16)
    return -(-rows // 128) * 128 * (-(-scols // 4)) * 4


def quant_act_block(x, q, s, T, cols, fmt="mxfp8", global_scale=1.0, stream=None, sf_layout=None):
    """MXFP8 (fmt "mxfp8") or NVFP4 ("nvfp4") codes and scale bytes of fp32 rows x [T, cols]; sf_layout
    SF_TILED_128X4 writes the scales in the block-scaled MMA operand layout."""
    if sf_layout is not None:
        call("wzyb_quant_act_block_f32", _ptr(x), _ptr(q), _ptr(s), BLOCK_MXFP8 if fmt == "mxfp8" else BLOCK_NVFP4,
             sf_layout, global_scale, T, cols, _stream(stream))
    elif fmt == "mxfp8":
        call("wzyb_quant_act_mxfp8_f32", _ptr(x), _ptr(q), _ptr(s), T, cols, _stream(stream))
    else:
        call("wzyb_quant_act_nvfp4_f32", _ptr(x), _ptr(q), _ptr(s), global_scale, T, cols, _stream(stream))


def swiglu_block(gate, up, q, s, fmt="mxfp8", global_scale=1.0, stream=None, sf_layout=None, cols=None):
    """SwiGLU to MXFP8 / NVFP4; with sf_layout (and the row width `cols`) the scales may be tiled."""
    if sf_layout is not None:
        call("wzyb_swiglu_block_f32", _ptr(gate), _ptr(up), _ptr(q), _ptr(s), BLOCK_MXFP8 if fmt == "mxfp8" else
             BLOCK_NVFP4, sf_layout, global_scale, gate.numel() // cols, cols, _stream(stream))
    elif fmt == "mxfp8":
        call("wzyb_swiglu_mxfp8_f32", _ptr(gate), _ptr(up), _ptr(q), _ptr(s), gate.numel(), _stream(stream))
    else:
        call("wzyb_swiglu_nvfp4_f32", _ptr(gate), _ptr(up), _ptr(q), _ptr(s), global_scale, gate.numel(),
             _stream(stream))


def gr_norm_block(R, w_norm, bo_prev, inj_prev, xn, xq, xs, T, n_embd, hc, fmt="mxfp8", global_scale=1.0, eps=1e-6,
                  stream=None, sf_layout=None):
    if sf_layout is not None:
        call("wzyb_gr_norm_block_f32", _ptr(R), _ptr(w_norm), _ptr(bo_prev), _ptr(inj_prev), _ptr(xn), _ptr(xq),
             _ptr(xs), BLOCK_MXFP8 if fmt == "mxfp8" else BLOCK_NVFP4, sf_layout, global_scale, T, n_embd, hc, eps,
             _stream(stream))
    elif fmt == "mxfp8":
        call("wzyb_gr_norm_mxfp8_f32", _ptr(R), _ptr(w_norm), _ptr(bo_prev), _ptr(inj_prev), _ptr(xn), _ptr(xq),
             _ptr(xs), T, n_embd, hc, eps, _stream(stream))
    else:
        call("wzyb_gr_norm_nvfp4_f32", _ptr(R), _ptr(w_norm), _ptr(bo_prev), _ptr(inj_prev), _ptr(xn), _ptr(xq),
             _ptr(xs), global_scale, T, n_embd, hc, eps, _stream(stream))


def gr_write_f32(R, blk, inj, T, n_embd, hc, stream=None):
    """R[t,c,:] += blk[t,:] * 2*sigmoid(inj[t,c]/hc) in place (gate 1.0 with inj None)."""
    call("wzyb_gr_write_f32", _ptr(R), _ptr(blk), _ptr(inj), T, n_embd, hc, _stream(stream))


def hc_mix(xn, gg, mixed, mixed_f16, T, n_embd, hc, stream=None):
    """mixed[t,:] = mean_c xn[t,c,:] * sigmoid(gg[t,c,:]); fp16 inputs may write either output."""
    if xn.element_size() == 2:
        call("wzyb_hc_mix_f16", _ptr(xn), _ptr(gg), _ptr(mixed), _ptr(mixed_f16), T, n_embd, hc, _stream(stream))
    else:
        call("wzyb_hc_mix_f32", _ptr(xn), _ptr(gg), _ptr(mixed), T, n_embd, hc, _stream(stream))


def silu_scale_f16(lo, out, scale, stream=None):
    call("wzyb_silu_scale_f16", _ptr(lo), _ptr(out), lo.numel(), scale, _stream(stream))


def head_norm_rope(data, gamma, cos_tab, sin_tab, T, heads, head_dim, head_stride, row_stride, rot_dims=64,
                   eps=1e-6, w_offset=0.0, d_base_pos=None, pos_offset=0, stream=None):
    fn = "wzyb_head_norm_rope_f16" if data.element_size() == 2 else "wzyb_head_norm_rope_f32"
    rows = cos_tab.numel() // max(1, rot_dims // 2) if cos_tab is not None else 0
    call(fn, _ptr(data), _ptr(gamma), _ptr(cos_tab), _ptr(sin_tab), rows, _ptr(d_base_pos), pos_offset, T, heads,
         head_dim, head_stride, row_stride, rot_dims, eps, w_offset, _stream(stream))


def head_tensor(data, gamma, heads, head_stride, row_stride) -> HeadTensor:
    """A wzyb_head_tensor over torch tensors. The C struct holds raw pointers only; the element size of
    data is kept on the Python object (elem_size) so wrappers can check it against the call's type."""
    if data.element_size() != gamma.element_size():
        raise ValueError("head_tensor: data and gamma must have the same element type")
    t = HeadTensor(data.data_ptr(), gamma.data_ptr(), heads, head_stride, row_stride)
    t.elem_size = data.element_size()
    return t


def qk_norm_rope_f16(q: HeadTensor, k: HeadTensor | None, cos_tab, sin_tab, T, head_dim, rot_dims=64, eps=1e-6,
                     w_offset=1.0, d_base_pos=None, pos_offset=0, stream=None):
    rows = cos_tab.numel() // max(1, rot_dims // 2)
    call("wzyb_qk_norm_rope_f16", ctypes.byref(q), ctypes.byref(k) if k is not None else None, _ptr(cos_tab),
         _ptr(sin_tab), rows, _ptr(d_base_pos), pos_offset, T, head_dim, rot_dims, eps, w_offset, _stream(stream))


def kv_cache(ring_k_q, ring_k_s, ring_v_q, ring_v_s, ring_cap, max_ctx, full_k_q=None, full_k_s=None, full_v_q=None,
             full_v_s=None) -> KvCache:
    """Cache descriptor from device tensors (scales: int16/uint16 tensors holding fp16 bits)."""
    return KvCache(ring_k_q.data_ptr(), ring_k_s.data_ptr(), ring_v_q.data_ptr(), ring_v_s.data_ptr(),
                   _ptr(full_k_q).value, _ptr(full_k_s).value, _ptr(full_v_q).value, _ptr(full_v_s).value, ring_cap,
                   max_ctx)


def kv_append_int8_f32(k, v, T, kv_heads, head_dim, cache: KvCache, d_base_pos=None, pos_offset=0, stream=None):
    call("wzyb_kv_append_int8_f32", _ptr(k), _ptr(v), T, kv_heads, head_dim, _ptr(d_base_pos), pos_offset,
         ctypes.byref(cache), _stream(stream))


def k_rope_kv_append(k, k_gamma, v, cos_tab, sin_tab, T, kv_heads, head_dim, cache: KvCache, rot_dims=64, eps=1e-6,
                     w_offset=0.0, d_base_pos=None, pos_offset=0, stream=None, q: HeadTensor | None = None):
    """k norm + RoPE + INT8 KV append; with q (a HeadTensor of the same element type) the q heads are
    normed and rotated in the same launch."""
    f16 = k.element_size() == 2
    if q is not None:
        qsize = getattr(q, "elem_size", None)
        if qsize is not None and qsize != k.element_size():
            raise ValueError(f"k_rope_kv_append: q has {qsize}-byte elements, k has {k.element_size()}-byte; "
                             "the fused q heads must have k's element type")
    rows = cos_tab.numel() // max(1, rot_dims // 2) if cos_tab is not None else 0
    args = (_ptr(k), _ptr(k_gamma), _ptr(v), _ptr(cos_tab), _ptr(sin_tab), rows, _ptr(d_base_pos), pos_offset, T,
            kv_heads, head_dim, rot_dims, eps, w_offset, ctypes.byref(cache), _stream(stream))
    if q is not None:
        call("wzyb_qk_rope_kv_append_f16" if f16 else "wzyb_qk_rope_kv_append_f32", ctypes.byref(q), *args)
    else:
        call("wzyb_k_rope_kv_append_f16" if f16 else "wzyb_k_rope_kv_append_f32", *args)


def rope_table(cos_tab, sin_tab, rows, rot_dims=64, theta=1e7, stream=None):
    call("wzyb_rope_table_f32", _ptr(cos_tab), _ptr(sin_tab), rows, rot_dims, theta, _stream(stream))


def rope_table_host(rows, rot_dims=64, theta=1e7):
    """The RoPE cos/sin tables [rows, rot_dims/2] fp32 built on the host by the reference's own procedure
    (build_rope_cos_sin_host: fp64 angle, libm cos/sin, rounded to fp32), as numpy arrays."""
    import numpy as np

    c = np.empty((rows, rot_dims // 2), dtype=np.float32)
    s = np.empty((rows, rot_dims // 2), dtype=np.float32)
    call("wzyb_rope_table_host_f32", c.ctypes.data, s.ctypes.data, rows, rot_dims, theta)
    return c, s


def gdn_gated_norm(o, z, gamma, y, T, heads, head_dim=128, eps=1e-6, w_offset=0.0, gate_mode=GATE_SIGMOID,
                   stream=None):
    fn = "wzyb_gdn_gated_norm_f16" if o.element_size() == 2 else "wzyb_gdn_gated_norm_f32_f16"
    call(fn, _ptr(o), _ptr(z), _ptr(gamma), _ptr(y), T, heads, head_dim, eps, w_offset, gate_mode, _stream(stream))


def swiglu(gate, up, out, stream=None):
    fn = "wzyb_swiglu_f16" if gate.element_size() == 2 else "wzyb_swiglu_f32"
    call(fn, _ptr(gate), _ptr(up), _ptr(out), gate.numel(), _stream(stream))


def swiglu_interleaved(gu, out, T, nff, stream=None):
    fn = "wzyb_swiglu_interleaved_f16" if gu.element_size() == 2 else "wzyb_swiglu_interleaved_f32_f16"
    call(fn, _ptr(gu), _ptr(out), T, nff, _stream(stream))


def embed_gather_rows(table, ids, out, oob_policy=OOB_CLAMP, oob_count=None, stream=None):
    """Row copy of a [vocab, row_bytes] byte view of any table (row_bytes % 16 == 0)."""
    vocab = table.shape[0]
    row_bytes = table[0].numel() * table.element_size()
    call("wzyb_embed_gather_rows", _ptr(table), vocab, row_bytes, _ptr(ids), ids.numel(), _ptr(out), oob_policy,
         _ptr(oob_count), _stream(stream))


def embed_gather_f16(table, ids, out, oob_policy=OOB_CLAMP, oob_count=None, stream=None):
    vocab, hidden = table.shape
    call("wzyb_embed_gather_f16", _ptr(table), vocab, hidden, _ptr(ids), ids.numel(), _ptr(out), oob_policy,
         _ptr(oob_count), _stream(stream))


def embed_gather_bf16_f32(table, ids, out, oob_policy=OOB_CLAMP, oob_count=None, stream=None):
    vocab, hidden = table.shape
    call("wzyb_embed_gather_bf16_f32", _ptr(table), vocab, hidden, _ptr(ids), ids.numel(), _ptr(out), oob_policy,
         _ptr(oob_count), _stream(stream))


def ple_gather_f16(tables, ids, out, prev_ids=None, eos_id=PLE_EOS_DEFAULT, hash_variant=PLE_HASH_C_PRECEDENCE,
                   stream=None):
    heads = len(tables)
    rows, hd = tables[0].shape
    arr = (c_void_p * heads)(*[t.data_ptr() for t in tables])
    prev = (c_int32 * 2)(*prev_ids) if prev_ids is not None else None
    call("wzyb_ple_gather_f16", arr, heads, rows, hd, _ptr(ids), ids.numel(), prev, eos_id, hash_variant, _ptr(out),
         _stream(stream))


def embed_ple_args(table, ple_tables, ids, emb_out, ple_out, prev_ids=None, eos_id=PLE_EOS_DEFAULT,
                   hash_variant=PLE_HASH_C_PRECEDENCE, oob_policy=OOB_CLAMP, oob_count=None) -> EmbedPleArgs:
    """Arguments of wzyb_embed_ple_f16 (the token-embedding and PLE gathers of the same ids, one launch).
    The returned struct keeps its host arrays alive."""
    a = EmbedPleArgs()
    a.ids, a.table = ids.data_ptr(), table.data_ptr()
    a.vocab, a.hidden = table.shape
    a.oob_policy, a.d_oob_count, a.emb_out = oob_policy, _ptr(oob_count), emb_out.data_ptr()
    a._tabs = (c_void_p * len(ple_tables))(*[t.data_ptr() for t in ple_tables])
    a.ple_tables = ctypes.cast(a._tabs, POINTER(c_void_p))
    a.ple_heads = len(ple_tables)
    a.ple_rows, a.ple_head_dim = ple_tables[0].shape
    a._prev = (c_int32 * 2)(*prev_ids) if prev_ids is not None else None
    a.prev_ids = ctypes.cast(a._prev, POINTER(c_int32)) if a._prev is not None else None
    a.eos_id, a.hash_variant, a.ple_out = eos_id, hash_variant, ple_out.data_ptr()
    return a


def embed_ple_f16(args: EmbedPleArgs, T: int, stream=None):
    call("wzyb_embed_ple_f16", ctypes.byref(args), T, _stream(stream))


def ple_row_index(t0, t1, t2, head, rows, eos_id=PLE_EOS_DEFAULT, hash_variant=PLE_HASH_C_PRECEDENCE) -> int:
    return int(lib().wzyb_ple_row_index(t0, t1, t2, head, rows, eos_id, hash_variant))


def ple_fp8_hash(vocab=None, mult=None) -> PleFp8Hash:
    """The reference's hash constants, or sub-tables of the given sizes packed end to end."""
    h = PleFp8Hash()
    check("wzyb_ple_fp8_reference_hash", lib().wzyb_ple_fp8_reference_hash(ctypes.byref(h)))
    if mult is not None:
        for i in range(3):
            h.mult[i] = int(mult[i])
    if vocab is not None:
        off = 0
        for i in range(16):
            h.vocab[i] = int(vocab[i])
            h.off[i] = off
            off += int(vocab[i])
    return h


def ple_gather_fp8_f32(table, row_bytes, scale, hsh: PleFp8Hash, ids, out, prev_ids=None, eos_id=PLE_EOS_DEFAULT,
                       stream=None):
    prev = (c_int32 * 2)(*prev_ids) if prev_ids is not None else None
    call("wzyb_ple_gather_fp8_f32", _ptr(table), table.numel() // row_bytes, row_bytes, scale, ctypes.byref(hsh),
         _ptr(ids), ids.numel(), prev, eos_id, _ptr(out), _stream(stream))


def ple_gate_f32(key, query, value, gv, T, n_embd, hc, stream=None):
    call("wzyb_ple_gate_f32", _ptr(key), _ptr(query), _ptr(value), _ptr(gv), T, n_embd, hc, _stream(stream))


def ple_conv_f32(norm, cw, hist, gv, R, T, hcd, hist_snaps=None, stream=None):
    call("wzyb_ple_conv_f32", _ptr(norm), _ptr(cw), _ptr(hist), _ptr(gv), _ptr(R), T, hcd, _ptr(hist_snaps),
         _stream(stream))


def shard_rows(total: int, world: int, rank: int) -> tuple[int, int]:
    r0, n = c_int64(), c_int64()
    call("wzyb_shard_rows", total, world, rank, ctypes.byref(r0), ctypes.byref(n))
    return r0.value, n.value


def ple_halo(ids_host, row0: int, seq_prev=None) -> tuple[int, int]:
    """ids_host: a contiguous int32 numpy array (the whole sequence on the host)."""
    import numpy as np

    arr = np.ascontiguousarray(ids_host, dtype=np.int32)
    out = (c_int32 * 2)()
    sp = (c_int32 * 2)(*seq_prev) if seq_prev is not None else None
    call("wzyb_ple_halo", arr.ctypes.data_as(POINTER(c_int32)) if arr.size else None, row0, sp, out)
    return int(out[0]), int(out[1])


def read_faults(clear=True) -> int:
    v = c_uint32()
    call("wzyb_read_faults", ctypes.byref(v), 1 if clear else 0)
    return int(v.value)


def set_launch_tuning(family: int, ctas_per_sm: int, stages: int = 0) -> None:
    call("wzyb_set_launch_tuning", family, ctas_per_sm, stages)


def set_kernel_variant(family: int, variant: int) -> None:
    call("wzyb_set_kernel_variant", family, variant)


def declared_functions(header_path: str = HEADER_PATH) -> list[str]:
    """Names of every function the C header declares."""
    import re

    text = open(header_path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(wzyb_[a-z0-9_]+)\s*\(", text)))
