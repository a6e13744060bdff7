"""CPU checks of the C ABI: the library loads, exports every declared entry point, validates
arguments on the host before touching the GPU, and its host-side helpers agree with the oracle.
No kernel is launched here."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest


def test_exports_every_declared_symbol(wz):
    names = wz.declared_functions()
    assert len(names) >= 25
    missing = [n for n in names if not hasattr(wz.lib(), n)]
    assert not missing, missing
    # and the binding declares a signature for each of them
    assert set(names) <= set(wz._SIGS), set(names) - set(wz._SIGS)


def test_status_strings(wz):
    assert wz.status_string(0) == "ok"
    for code in (wz.ERR_NULL, wz.ERR_ALIGN, wz.ERR_SHAPE, wz.ERR_DEVICE, wz.ERR_VALUE):
        assert "unknown" not in wz.status_string(code) or code == wz.ERR_VALUE
    assert wz.lib().wzyb_version() >= 100


NULL = ctypes.c_void_p(0)
A16 = ctypes.c_void_p(0x10000)      # aligned, never dereferenced: validation fails first
A8 = ctypes.c_void_p(0x10008)       # 8-byte aligned only


def test_argument_validation_before_any_cuda_call(wz):
    L = wz.lib()
    # NULL operands
    assert L.wzyb_add_rmsnorm_f16(NULL, NULL, A16, A16, 4, 2048, 1e-6, 1.0, NULL) == wz.ERR_NULL
    # unsupported hidden (not a multiple of 8)
    assert L.wzyb_add_rmsnorm_f16(A16, A16, A16, A16, 4, 2044, 1e-6, 1.0, NULL) == wz.ERR_SHAPE
    # misaligned pointer
    assert L.wzyb_add_rmsnorm_f16(A8, A16, A16, A16, 4, 2048, 1e-6, 1.0, NULL) == wz.ERR_ALIGN
    # head_dim / rot_dims outside the supported set
    args = [A16, A16, A16, A16, 4096, NULL, 0, 8, 16, 96, 96, 16 * 96, 64, 1e-6, 1.0, NULL]
    assert L.wzyb_head_norm_rope_f16(*args) == wz.ERR_SHAPE
    args = [A16, A16, A16, A16, 4096, NULL, 0, 8, 16, 256, 256, 16 * 256, 72, 1e-6, 1.0, NULL]
    assert L.wzyb_head_norm_rope_f16(*args) == wz.ERR_SHAPE
    # rotary requested without a table
    args = [A16, A16, NULL, NULL, 4096, NULL, 0, 8, 16, 256, 256, 16 * 256, 64, 1e-6, 1.0, NULL]
    assert L.wzyb_head_norm_rope_f16(*args) == wz.ERR_NULL
    # misaligned head stride (fp16: stride*2 must be a multiple of 16)
    args = [A16, A16, A16, A16, 4096, NULL, 0, 8, 2, 256, 260, 1024, 64, 1e-6, 1.0, NULL]
    assert L.wzyb_head_norm_rope_f16(*args) == wz.ERR_ALIGN
    # gate mode
    assert L.wzyb_gdn_gated_norm_f16(A16, A16, A16, A16, 4, 32, 128, 1e-6, 0.0, 7, NULL) == wz.ERR_VALUE
    assert L.wzyb_gdn_gated_norm_f16(A16, A16, A16, A16, 4, 32, 96, 1e-6, 0.0, 0, NULL) == wz.ERR_SHAPE
    # SwiGLU sizes
    assert L.wzyb_swiglu_f16(A16, A16, A16, 12, NULL) == wz.ERR_SHAPE
    assert L.wzyb_swiglu_interleaved_f16(A16, A16, 4, 12, NULL) == wz.ERR_SHAPE
    # gathers
    assert L.wzyb_embed_gather_rows(A16, 100, 24, A16, 4, A16, 0, NULL, NULL) == wz.ERR_SHAPE
    assert L.wzyb_embed_gather_rows(A16, 100, 32, A16, 4, A16, 9, NULL, NULL) == wz.ERR_VALUE
    assert L.wzyb_embed_gather_f16(A16, 0, 2048, A16, 4, A16, 0, NULL, NULL) == wz.ERR_SHAPE
    tables = (ctypes.c_void_p * 2)(0x10000, 0)
    assert L.wzyb_ple_gather_f16(tables, 2, 1 << 20, 128, A16, 4, None, 248044, 0, A16, NULL) == wz.ERR_NULL
    assert L.wzyb_ple_gather_f16(tables, 33, 1 << 20, 128, A16, 4, None, 248044, 0, A16, NULL) == wz.ERR_SHAPE
    assert L.wzyb_ple_gather_f16(tables, 1, 1 << 20, 128, A16, 4, None, 248044, 5, A16, NULL) == wz.ERR_VALUE
    # Q8_0 side outputs: whole 32-wide groups, n_embd <= 4096, every buffer 16-byte aligned
    assert L.wzyb_gr_norm_q8_f32(A16, A16, A16, A16, A16, NULL, A16, 4, 2560, 4, 1e-6, NULL) == wz.ERR_NULL
    assert L.wzyb_gr_norm_q8_f32(A16, A16, A16, A16, A16, A16, A16, 4, 2568, 4, 1e-6, NULL) == wz.ERR_SHAPE
    assert L.wzyb_gr_norm_q8_f32(A16, A16, A16, A16, A16, A16, A16, 4, 16416, 4, 1e-6, NULL) == wz.ERR_SHAPE
    assert L.wzyb_gr_norm_q8_f32(A16, A16, A16, A16, A16, A8, A16, 4, 2560, 4, 1e-6, NULL) == wz.ERR_ALIGN
    assert L.wzyb_gr_norm_q8_f32(A16, A16, A16, A16, A16, A16, A16, 0, 2560, 4, 1e-6, NULL) == wz.OK
    assert L.wzyb_swiglu_q8_f32(A16, A16, NULL, A16, 64, NULL) == wz.ERR_NULL
    assert L.wzyb_swiglu_q8_f32(A16, A16, A16, A16, 48, NULL) == wz.ERR_SHAPE
    assert L.wzyb_swiglu_q8_f32(A16, A16, A16, A8, 64, NULL) == wz.ERR_ALIGN
    assert L.wzyb_swiglu_q8_f32(A16, A16, A16, A16, 0, NULL) == wz.OK
    # int8 activation quantisation
    assert L.wzyb_quant_act_f32(A16, NULL, NULL, NULL, NULL, 4, 2560, NULL) == wz.ERR_NULL
    assert L.wzyb_quant_act_f32(A16, A16, NULL, NULL, NULL, 4, 2560, NULL) == wz.ERR_NULL
    assert L.wzyb_quant_act_f32(A16, A16, A16, NULL, NULL, 4, 2576, NULL) == wz.ERR_SHAPE
    assert L.wzyb_quant_act_f32(A16, A8, A16, NULL, NULL, 4, 2560, NULL) == wz.ERR_ALIGN
    # block-scaled formats: group sizes 32 (MXFP8) / 16 (NVFP4)
    assert L.wzyb_quant_act_mxfp8_f32(A16, NULL, A16, 4, 2560, NULL) == wz.ERR_NULL
    assert L.wzyb_quant_act_mxfp8_f32(A16, A16, A16, 4, 2576, NULL) == wz.ERR_SHAPE
    # the general block quantisers: format and scale layout are checked before anything is enqueued
    assert L.wzyb_quant_act_block_f32(A16, A16, A16, 7, wz.SF_ROW_MAJOR, 1.0, 4, 2560, NULL) == wz.ERR_VALUE
    assert L.wzyb_quant_act_block_f32(A16, A16, A16, wz.BLOCK_MXFP8, 5, 1.0, 4, 2560, NULL) == wz.ERR_VALUE
    assert L.wzyb_quant_act_block_f32(A16, NULL, A16, wz.BLOCK_NVFP4, wz.SF_TILED_128X4, 1.0, 4, 2560, NULL) == wz.ERR_NULL
    assert L.wzyb_swiglu_block_f32(A16, A16, A16, A16, 2, wz.SF_ROW_MAJOR, 1.0, 4, 512, NULL) == wz.ERR_VALUE
    assert L.wzyb_swiglu_block_f32(A16, A16, A16, A16, wz.BLOCK_MXFP8, 4, 1.0, 4, 512, NULL) == wz.ERR_VALUE
    assert L.wzyb_swiglu_block_f32(A16, A16, A16, A16, wz.BLOCK_MXFP8, wz.SF_TILED_128X4, 1.0, 4, 520, NULL) == \
        wz.ERR_SHAPE
    assert L.wzyb_gr_norm_block_f32(A16, A16, A16, A16, A16, A16, A16, 3, wz.SF_ROW_MAJOR, 1.0, 4, 2560, 4, 1e-6,
                                    NULL) == wz.ERR_VALUE
    assert L.wzyb_gr_norm_block_f32(A16, A16, A16, A16, A16, A16, A16, wz.BLOCK_MXFP8, 9, 1.0, 4, 2560, 4, 1e-6,
                                    NULL) == wz.ERR_VALUE
    assert L.wzyb_gr_norm_block_f32(A16, A16, A16, A16, A16, NULL, A16, wz.BLOCK_NVFP4, wz.SF_TILED_128X4, 1.0, 4,
                                    2560, 4, 1e-6, NULL) == wz.ERR_NULL
    assert L.wzyb_quant_act_nvfp4_f32(A16, A16, A16, 1.0, 4, 2568, NULL) == wz.ERR_SHAPE
    assert L.wzyb_quant_act_nvfp4_f32(A8, A16, A16, 1.0, 4, 2560, NULL) == wz.ERR_ALIGN
    assert L.wzyb_swiglu_mxfp8_f32(A16, A16, A16, A16, 48, NULL) == wz.ERR_SHAPE
    assert L.wzyb_swiglu_nvfp4_f32(A16, A16, NULL, A16, 1.0, 64, NULL) == wz.ERR_NULL
    assert L.wzyb_gr_norm_mxfp8_f32(A16, A16, A16, A16, A16, A16, A16, 4, 2568, 4, 1e-6, NULL) == wz.ERR_SHAPE
    assert L.wzyb_gr_norm_nvfp4_f32(A16, A16, A16, A16, A16, A8, A16, 1.0, 4, 2560, 4, 1e-6, NULL) == wz.ERR_ALIGN
    assert L.wzyb_gr_norm_nvfp4_f32(A16, A16, A16, A16, A16, A16, A16, 1.0, 0, 2560, 4, 1e-6, NULL) == wz.OK
    # multi-stream residual
    assert L.wzyb_gr_write_f32(NULL, A16, NULL, 4, 2560, 4, NULL) == wz.ERR_NULL
    assert L.wzyb_gr_write_f32(A16, A16, NULL, 4, 2564, 4, NULL) == wz.ERR_SHAPE
    assert L.wzyb_gr_write_f32(A16, A16, NULL, 4, 2560, 0, NULL) == wz.ERR_SHAPE
    assert L.wzyb_gr_write_f32(A8, A16, NULL, 4, 2560, 4, NULL) == wz.ERR_ALIGN
    assert L.wzyb_hc_mix_f16(A16, A16, NULL, NULL, 4, 2560, 4, NULL) == wz.ERR_NULL
    assert L.wzyb_hc_mix_f16(A16, A16, A16, NULL, 4, 2562, 4, NULL) == wz.ERR_SHAPE
    assert L.wzyb_hc_mix_f16(A16, A16, NULL, A8, 4, 2560, 4, NULL) == wz.ERR_ALIGN
    assert L.wzyb_hc_mix_f32(A16, A16, NULL, 4, 2560, 4, NULL) == wz.ERR_NULL
    assert L.wzyb_hc_mix_f32(A16, A16, A16, 0, 2560, 4, NULL) == wz.OK
    assert L.wzyb_silu_scale_f16(A16, A16, 12, 0.25, NULL) == wz.ERR_SHAPE
    assert L.wzyb_silu_scale_f16(A16, A8, 16, 0.25, NULL) == wz.ERR_ALIGN
    # INT8 KV append: ring planes required, the mirror all-or-none, scales 2-byte aligned
    a = 0x10000
    kc = ctypes.byref(wz.KvCache(a, a, a, a, None, None, None, None, 64, 128))
    assert L.wzyb_kv_append_int8_f32(A16, A16, 4, 2, 256, None, 0, None, NULL) == wz.ERR_NULL
    assert L.wzyb_kv_append_int8_f32(A16, A16, 4, 2, 96, None, 0, kc, NULL) == wz.ERR_SHAPE
    assert L.wzyb_kv_append_int8_f32(A8, A16, 4, 2, 256, None, 0, kc, NULL) == wz.ERR_ALIGN
    assert L.wzyb_kv_append_int8_f32(A16, A16, 0, 2, 256, None, 0, kc, NULL) == wz.OK
    part = ctypes.byref(wz.KvCache(a, a, a, a, a, None, None, None, 64, 128))
    assert L.wzyb_kv_append_int8_f32(A16, A16, 4, 2, 256, None, 0, part, NULL) == wz.ERR_NULL
    odd = ctypes.byref(wz.KvCache(a, a + 1, a, a, None, None, None, None, 64, 128))
    assert L.wzyb_kv_append_int8_f32(A16, A16, 4, 2, 256, None, 0, odd, NULL) == wz.ERR_ALIGN
    # PLE in the reference format: every hashed row inside the table, whole 16-byte chunks
    h = wz.ple_fp8_hash()
    assert [h.off[i] for i in range(3)] == [0, 20000003, 40000026] and h.off[15] + h.vocab[15] == 320001446
    hb = ctypes.byref(h)
    g8 = L.wzyb_ple_gather_fp8_f32
    assert g8(A16, 320001446, 160, 1.0, None, A16, 4, None, 248044, A16, NULL) == wz.ERR_NULL
    assert g8(A16, 320001445, 160, 1.0, hb, A16, 4, None, 248044, A16, NULL) == wz.ERR_SHAPE
    assert g8(A16, 320001446, 150, 1.0, hb, A16, 4, None, 248044, A16, NULL) == wz.ERR_SHAPE
    assert g8(A8, 320001446, 160, 1.0, hb, A16, 4, None, 248044, A16, NULL) == wz.ERR_ALIGN
    assert g8(A16, 320001446, 160, 1.0, hb, A16, 0, None, 248044, A16, NULL) == wz.OK
    assert L.wzyb_ple_gate_f32(A16, A16, NULL, A16, 4, 2560, 4, NULL) == wz.ERR_NULL
    assert L.wzyb_ple_gate_f32(A16, A16, A16, A16, 4, 2564, 4, NULL) == wz.ERR_SHAPE
    assert L.wzyb_ple_conv_f32(A16, A16, A16, A16, NULL, 4, 10240, NULL, NULL) == wz.ERR_NULL
    assert L.wzyb_ple_conv_f32(A16, A16, A16, A16, A16, 4, 10242, NULL, NULL) == wz.ERR_SHAPE
    assert L.wzyb_ple_conv_f32(A16, A8, A16, A16, A16, 4, 10240, NULL, NULL) == wz.ERR_ALIGN
    fused = L.wzyb_k_rope_kv_append_f16
    assert fused(A16, NULL, A16, A16, A16, 64, None, 0, 4, 2, 256, 64, 1e-6, 1.0, kc, NULL) == wz.ERR_NULL
    assert fused(A16, A16, A16, A16, A16, 64, None, 0, 4, 2, 256, 24, 1e-6, 1.0, kc, NULL) == wz.ERR_SHAPE
    assert fused(A16, A16, A16, NULL, NULL, 64, None, 0, 4, 2, 256, 64, 1e-6, 1.0, kc, NULL) == wz.ERR_NULL
    # empty work is a no-op that succeeds without a device
    assert L.wzyb_swiglu_f16(A16, A16, A16, 0, NULL) == wz.OK
    assert L.wzyb_add_rmsnorm_f16(A16, A16, A16, A16, 0, 2048, 1e-6, 1.0, NULL) == wz.OK
    # tuning knobs
    assert L.wzyb_qk_rope_kv_append_f32(None, A16, A16, A16, A16, A16, 64, NULL, 0, 4, 2, 256, 64, 1e-6, 1.0,
                                        None, NULL) == wz.ERR_NULL
    assert L.wzyb_attn_prep_f16(None, 4, NULL) == wz.ERR_NULL
    assert L.wzyb_act_f16(None, 4, NULL) == wz.ERR_NULL
    bad = wz.ActArgs()
    bad.act_rows, bad.ffn = -1, 512
    assert L.wzyb_act_f16(ctypes.byref(bad), 4, NULL) == wz.ERR_SHAPE
    assert L.wzyb_set_launch_tuning(9, 1, 0) == wz.ERR_VALUE
    assert L.wzyb_set_launch_tuning(0, 0, 0) == wz.ERR_VALUE


def test_qk_kv_append_q_validation(wz):
    """Every argument error of the fused q heads of wzyb_qk_rope_kv_append_* is returned on the host before
    any CUDA call. (No entry point can pass q heads to a call without norm + RoPE: the append-only
    wzyb_kv_append_int8_f32 has no q argument.)"""
    L = wz.lib()
    kc = ctypes.byref(wz.KvCache(0x10000, 0x10000, 0x10000, 0x10000, None, None, None, None, 64, 128))
    k, v = 0x100000, 0x200000  # k, v [4, 2 x 256] fp16: 4 KB each, far from q

    def call(qt, T=4):
        return L.wzyb_qk_rope_kv_append_f16(ctypes.byref(qt), ctypes.c_void_p(k), A16, ctypes.c_void_p(v), A16, A16,
                                            64, NULL, 0, T, 2, 256, 64, 1e-6, 1.0, kc, NULL)

    q = 0x400000
    ok_rs = 24 * 2 * 256
    assert call(wz.HeadTensor(q, 0x10000, 300, 512, 300 * 512)) == wz.ERR_SHAPE    # q_heads > 256
    assert call(wz.HeadTensor(q, 0x10000, -1, 512, ok_rs)) == wz.ERR_SHAPE          # q_heads < 0
    assert call(wz.HeadTensor(None, 0x10000, 24, 512, ok_rs)) == wz.ERR_NULL        # q->data NULL
    assert call(wz.HeadTensor(q, None, 24, 512, ok_rs)) == wz.ERR_NULL              # q->gamma NULL
    assert call(wz.HeadTensor(q, 0x10000, 24, 100, ok_rs)) == wz.ERR_SHAPE         # heads overlap
    assert call(wz.HeadTensor(q, 0x10000, 24, 516, 24 * 516 + 4)) == wz.ERR_ALIGN   # head stride * 2 % 16
    assert call(wz.HeadTensor(q, 0x10000, 24, 512, ok_rs + 4)) == wz.ERR_ALIGN      # row stride * 2 % 16
    assert call(wz.HeadTensor(q + 8, 0x10000, 24, 512, ok_rs)) == wz.ERR_ALIGN      # q not 16-byte aligned
    # tokens' q rows overlapping each other (row stride shorter than one token's heads), T > 1 only
    assert call(wz.HeadTensor(q, 0x10000, 24, 512, 0)) == wz.ERR_SHAPE
    assert call(wz.HeadTensor(q, 0x10000, 24, 512, 8 * 512)) == wz.ERR_SHAPE
    # q sharing bytes with k or v
    assert call(wz.HeadTensor(k, 0x10000, 2, 256, 512)) == wz.ERR_SHAPE
    assert call(wz.HeadTensor(v + 1024, 0x10000, 1, 256, 512)) == wz.ERR_SHAPE
    # empty call with valid arguments: a no-op that needs no device
    assert call(wz.HeadTensor(q, 0x10000, 24, 512, ok_rs), T=0) == wz.OK


def test_bundle_validation(wz):
    """The one-launch bundles validate both ops' arguments before anything is enqueued, and accept the
    SPLIT design switch of their family."""
    L = wz.lib()
    assert L.wzyb_embed_ple_f16(None, 4, NULL) == wz.ERR_NULL
    e = wz.EmbedPleArgs()
    e.ids, e.table, e.vocab, e.hidden, e.emb_out = 0x10000, 0x20000, 100, 2048, 0x30000
    tabs = (ctypes.c_void_p * 16)(*([0x40000] * 16))
    e.ple_tables, e.ple_heads, e.ple_rows, e.ple_head_dim, e.ple_out = (ctypes.cast(tabs, ctypes.POINTER(
        ctypes.c_void_p)), 16, 1 << 20, 128, 0x50000)
    e.hidden = 2044
    assert L.wzyb_embed_ple_f16(ctypes.byref(e), 4, NULL) == wz.ERR_SHAPE
    e.hidden, e.oob_policy = 2048, 7
    assert L.wzyb_embed_ple_f16(ctypes.byref(e), 4, NULL) == wz.ERR_VALUE
    e.oob_policy, e.hash_variant = 0, 9
    assert L.wzyb_embed_ple_f16(ctypes.byref(e), 4, NULL) == wz.ERR_VALUE
    e.hash_variant, e.ple_out = 0, 0x50008
    assert L.wzyb_embed_ple_f16(ctypes.byref(e), 4, NULL) == wz.ERR_ALIGN
    e.ple_out = 0x50000
    assert L.wzyb_embed_ple_f16(ctypes.byref(e), 0, NULL) == wz.OK
    # attn_prep: an invalid q/k argument is reported although the norm's arguments are valid
    a = wz.AttnPrepArgs()
    a.x, a.residual, a.norm_weight, a.normed, a.hidden = 0x10000, 0x20000, 0x30000, 0x40000, 2048
    a.q = wz.HeadTensor(0x50000, 0x60000, 16, 256, 4096)
    a.k = wz.HeadTensor(0x70000, 0x60000, 2, 256, 512)
    a.head_dim, a.rot_dims, a.cos_tab, a.sin_tab, a.table_rows = 96, 64, 0x80000, 0x90000, 4096
    assert L.wzyb_attn_prep_f16(ctypes.byref(a), 4, NULL) == wz.ERR_SHAPE
    a.head_dim = 256
    assert L.wzyb_attn_prep_f16(ctypes.byref(a), 0, NULL) == wz.OK
    a.hidden = 2044
    assert L.wzyb_attn_prep_f16(ctypes.byref(a), 4, NULL) == wz.ERR_SHAPE
    assert L.wzyb_set_kernel_variant(wz.FAM_BUNDLE, wz.VARIANT_SPLIT) == wz.OK
    assert L.wzyb_set_kernel_variant(wz.FAM_BUNDLE, wz.VARIANT_AUTO) == wz.OK
    assert L.wzyb_set_kernel_variant(wz.FAM_BUNDLE, 7) == wz.ERR_VALUE
    assert L.wzyb_set_kernel_variant(7, 0) == wz.ERR_VALUE


def test_head_tensor_element_type_checked(wz):
    import torch

    q16 = torch.zeros((2, 4, 512), dtype=torch.float16)
    g32 = torch.zeros(256, dtype=torch.float32)
    with pytest.raises(ValueError):
        wz.head_tensor(q16, g32, 4, 512, 2048)
    t = wz.head_tensor(q16, g32.half(), 4, 512, 2048)
    assert t.elem_size == 2
    k32 = torch.zeros((2, 512), dtype=torch.float32)
    with pytest.raises(ValueError):
        wz.k_rope_kv_append(k32, g32, k32, None, None, 2, 2, 256, wz.KvCache(), q=t)


def test_no_device_is_reported_not_crashed(wz):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert wz.lib().wzyb_prepare_device() == wz.ERR_DEVICE


@pytest.mark.parametrize("total,world", [(4096, 1), (4096, 2), (4096, 8), (262144, 8), (17, 4), (3, 8), (0, 2)])
def test_shard_rows_partition(wz, total, world):
    seen = []
    for r in range(world):
        r0, n = wz.shard_rows(total, world, r)
        assert n >= 0
        seen.extend(range(r0, r0 + n))
    assert seen == list(range(total))


def test_ple_halo(wz):
    ids = np.arange(100, 120, dtype=np.int32)
    assert wz.ple_halo(ids, 0) == (-1, -1)
    assert wz.ple_halo(ids, 0, (7, 8)) == (7, 8)
    assert wz.ple_halo(ids, 1, (7, 8)) == (8, 100)
    assert wz.ple_halo(ids, 5) == (103, 104)


def test_ple_row_index_matches_oracle(wz, orc):
    rng = np.random.default_rng(5)
    for _ in range(500):
        t0, t1, t2 = (int(v) for v in rng.integers(-3, 300000, 3))
        h = int(rng.integers(0, 16))
        for rows in (1 << 20, 20000003):
            for var in (0, 1):
                assert wz.ple_row_index(t0, t1, t2, h, rows, 248044, var) == orc.ple_row(t0, t1, t2, h, rows,
                                                                                         248044, var)


def test_host_rope_table_matches_oracle(wz, orc):
    rows, rot = 3000, 64
    c = np.empty((rows, rot // 2), np.float32)
    s = np.empty((rows, rot // 2), np.float32)
    wz.call("wzyb_rope_table_host_f32", c.ctypes.data, s.ctypes.data, rows, rot, 1e7)
    oc, os_ = orc.rope_table(rows, rot, 1e7)
    assert np.array_equal(c, oc) and np.array_equal(s, os_)
