// stage_dropin.cu -- TEST INFRASTRUCTURE ONLY: the compiler's check that libwzyb200 drops into the
// reference's layer executors.
//
// One translation unit includes the reference's executor headers, unmodified and in its engine's
// order (src/wzy_engine_v2.cu), and after them include/wzyb200.h. The reference's headers put the
// model constants (NE, HC, QH, HD, EPS, PLE_EOS, ...), the buffer type Dev{float* p; size_t n}
// (src/wzy_stage_v2.cuh:91-93), the layer weights LayerW (:197-221) and the executor StageGpu
// (:334-857) at global scope. The functions below make each launch-site replacement the integration
// notes give, with those globals and the executor's own members and raw pointer types (float*,
// __half*, signed char*, unsigned short*, int* dpos, cudaStream_t), at:
//   StageGpu::record_forward      src/wzy_stage_v2.cuh:476-857
//   PrefillStageCtx::run_stage_prefill  src/wzy_prefill_tc.cuh:546-1058
// so compiling this file proves that the header declares nothing that clashes with the reference's
// globals and that each replacement type-checks where it would be written. The site functions are
// compiled, never called (the reference's executors own the buffers they name). The one extern "C"
// function at the end runs the decode-window residual norm replacement on Dev buffers; the GPU test
// links it against libwzyb200.so and compares it with the reference's own fused_gr_norm_multi.
#include "wzy_stage_v2.cuh"
#include "wzy_mtp.cuh"
#include "wzy_prefill_tc.cuh"

#include "wzyb200.h"

#define WZYB_CHECK(x)                                                                                        \
    do {                                                                                                     \
        int _r = (x);                                                                                        \
        if (_r != WZYB_OK) {                                                                                 \
            std::fprintf(stderr, "wzyb: %s at %s:%d\n", wzyb_status_string(_r), __FILE__, __LINE__);        \
            std::exit(1);                                                                                    \
        }                                                                                                    \
    } while (0)

// The replacements inside StageGpu::record_forward (decode / verify window of T tokens). Argument
// names are the executor's: its members through S, the layer's weights w, and the locals of the
// sites (bo_prev / inj_prev from gr_read_fused, dpos, the layer's KV cache slices l_*).
void dropin_record_forward_sites(StageGpu& S, const LayerW& w, const Dev& gn, const float* bo_prev,
                                 const float* inj_prev, const int* dpos, signed char* l_vkq, unsigned short* l_vks,
                                 signed char* l_vvq, unsigned short* l_vvs, signed char* l_hkq,
                                 unsigned short* l_hks, signed char* l_hvq, unsigned short* l_hvs, int T) {
    cudaStream_t stream = S.stream;
    Dev &R = S.R, &xn = S.xn, &mixed2 = S.mixed2, &block = S.block, &inject = S.inject;
    Dev &qg = S.qg, &kk = S.kk, &vv = S.vv, &cos_tab = S.cos_tab, &sin_tab = S.sin_tab;
    Dev &sff = S.sff, &sup = S.sup, &tmp_ff = S.tmp_ff;
    const int ctx_max = S.ctx_max;

    // gr_read_fused (src/wzy_stage_v2.cuh:466), with and without the Q8_0 side output
    WZYB_CHECK(wzyb_gr_norm_q8_f32(R.p, gn.p, bo_prev, inj_prev, xn.p, (int8_t*)S.xq8, S.xs8, T, NE, HC, EPS,
                                   stream));
    WZYB_CHECK(wzyb_gr_norm_f32(R.p, gn.p, bo_prev, inj_prev, xn.p, T, NE, HC, EPS, stream));
    // ple_group_multi on ple_k, in place (src/wzy_stage_v2.cuh:590)
    WZYB_CHECK(wzyb_gr_norm_f32(S.ple_k.p, S.ple_nk.p, nullptr, nullptr, S.ple_k.p, T, NE, HC, EPS, stream));
    // gr_write_multi (src/wzy_stage_v2.cuh:585)
    WZYB_CHECK(wzyb_gr_write_f32(R.p, block.p, inject.p, T, NE, HC, stream));
    // quant_act_multi (src/wzy_stage_v2.cuh:697) and silu_mul_quant32_multi (:713)
    WZYB_CHECK(wzyb_quant_act_f32(mixed2.p, (int8_t*)S.eq32, S.es32, (int8_t*)S.eq16, S.es16, T, NE, stream));
    WZYB_CHECK(wzyb_swiglu_q8_f32(sff.p, sup.p, (int8_t*)S.xq8, S.xs8, (int64_t)NFF * T, stream));
    // q / k / indexer-q norm + RoPE (src/wzy_stage_v2.cuh:638-643)
    WZYB_CHECK(wzyb_head_norm_rope_f32(qg.p, w.q_norm.p, cos_tab.p, sin_tab.p, /*table_rows=*/ctx_max, dpos,
                                       /*pos_offset=*/0, T, QH, HD, 2 * HD, 2 * QD, /*rot_dims=*/NROT, EPS,
                                       /*w_offset=*/0.0f, stream));
    WZYB_CHECK(wzyb_head_norm_rope_f32(S.q_idx.p, w.idx_qn.p, cos_tab.p, sin_tab.p, ctx_max, dpos, 0, T, IDX_HEADS,
                                       IDX_DIM, IDX_DIM, IDX_HEADS * IDX_DIM, NROT, EPS, 0.0f, stream));
    // k norm + RoPE + kv_append_int8_multi (src/wzy_stage_v2.cuh:640-655) as one launch, then with q
    const wzyb_kv_cache cache = {(int8_t*)l_vkq, l_vks, (int8_t*)l_vvq, l_vvs, (int8_t*)l_hkq, l_hks,
                                 (int8_t*)l_hvq, l_hvs, KV_VRAM_RING, ctx_max};
    WZYB_CHECK(wzyb_k_rope_kv_append_f32(kk.p, w.k_norm.p, vv.p, cos_tab.p, sin_tab.p, ctx_max, dpos, 0, T, KVH, HD,
                                         NROT, EPS, 0.0f, &cache, stream));
    const wzyb_head_tensor q = {qg.p, w.q_norm.p, QH, 2 * HD, 2 * QD};
    WZYB_CHECK(wzyb_qk_rope_kv_append_f32(&q, kk.p, w.k_norm.p, vv.p, cos_tab.p, sin_tab.p, ctx_max, dpos, 0, T,
                                          KVH, HD, NROT, EPS, 0.0f, &cache, stream));
    WZYB_CHECK(wzyb_kv_append_int8_f32(kk.p, vv.p, T, KVH, HD, dpos, 0, &cache, stream));
    // silu_mul_multi (src/wzy_stage_v2.cuh:733)
    WZYB_CHECK(wzyb_swiglu_f32(sff.p, sup.p, tmp_ff.p, (int64_t)NFF * T, stream));
    // PLE block (src/wzy_stage_v2.cuh:592-594)
    WZYB_CHECK(wzyb_ple_gate_f32(S.ple_k.p, S.ple_q.p, S.ple_v.p, S.ple_gat.p, T, NE, HC, stream));
    WZYB_CHECK(wzyb_ple_conv_f32(S.ple_n.p, S.ple_cv.p, S.ple_hist.p, S.ple_gat.p, R.p, T, HCD, S.ple_snaps.p,
                                 stream));
    // embedding rows from the device-resident bf16 table (src/wzy_stage_v2.cuh:563-575)
    WZYB_CHECK(wzyb_embed_gather_bf16_f32(S.d_emb_table, NVOCAB, NE, S.d_toks, T, S.mixed.p, WZYB_OOB_CLAMP, nullptr,
                                          stream));
}

// The replacements inside PrefillStageCtx::run_stage_prefill for a chunk of B tokens, with the
// prefill workspace's own pointer types (src/wzy_prefill_tc.cuh:620-650).
void dropin_prefill_sites(StageGpu& s, const LayerW& w, const Dev& gn, float* R_pf, const float* bo_prev,
                          const float* inj_prev, __half* xn_h, const __half* gg_h, float* mx, __half* mx_h,
                          const float* lo_pf, __half* lo_h, const float* xn_pf, const float* bufB_pf,
                          __half* xfp16_pf, const float* sff_pf, int B) {
    // pf_gr_norm_fp16 (src/wzy_prefill_tc.cuh:697)
    WZYB_CHECK(wzyb_gr_norm_f32_f16(R_pf, gn.p, bo_prev, inj_prev, (uint16_t*)xn_h, B, NE, HC, EPS, s.stream));
    // silu_div_hc_to_fp16_kernel (:706) and pf_gr_up_mean_fp16 (:712)
    WZYB_CHECK(wzyb_silu_scale_f16(lo_pf, (uint16_t*)lo_h, (int64_t)B * HCLR, 1.0f / (float)HC, s.stream));
    WZYB_CHECK(wzyb_hc_mix_f16((const uint16_t*)xn_h, (const uint16_t*)gg_h, mx, (uint16_t*)mx_h, B, NE, HC,
                               s.stream));
    // pf_gdn_rmsnorm_gate_parallel (:845)
    WZYB_CHECK(wzyb_gdn_gated_norm_f32_f16(xn_pf, bufB_pf, w.ssm_norm.p, (uint16_t*)xfp16_pf, B, VH, 128, EPS,
                                           /*w_offset=*/0.0f, WZYB_GATE_SIGMOID, s.stream));
    // pf_silu_mul_interleaved_to_fp16 (:942)
    WZYB_CHECK(wzyb_swiglu_interleaved_f32_f16(sff_pf, (uint16_t*)xfp16_pf, B, NFF, s.stream));
}

// The engine's PLE staging (stage_ple_window, src/wzy_engine_v2.cu:943-978) as a device gather from
// the HBM copy of ple-fp8.gguf, with the reference's hash constants and PLE_HEAD / PLE_EOS.
void dropin_ple_site(StageGpu& S, const uint8_t* d_ple_fp8, int64_t ple_rows, float ple_scale,
                     const int ple_prev[2], int T) {
    wzyb_ple_fp8_hash hash;
    WZYB_CHECK(wzyb_ple_fp8_reference_hash(&hash));
    const int32_t prev[2] = {ple_prev[0], ple_prev[1]};
    WZYB_CHECK(wzyb_ple_gather_fp8_f32(d_ple_fp8, ple_rows, PLE_HEAD, ple_scale, &hash, S.d_toks, T, prev, PLE_EOS,
                                       S.d_ple_emb.p, S.stream));
}

extern "C" {

// Runs gr_read_fused's replacement (src/wzy_stage_v2.cuh:466) on the reference's Dev buffers, at the
// reference model's own NE / HC / EPS: R [T, HC, NE], gn [HC, NE], xn [T, HC, NE] fp32, no pending
// residual. Returns the library's status.
int dropin_gr_read_fused(float* R_p, const float* gn_p, float* xn_p, int T, cudaStream_t stream) {
    Dev R, gn, xn;
    R.p = R_p;
    R.n = (size_t)T * HCD;
    gn.p = const_cast<float*>(gn_p);
    gn.n = (size_t)HCD;
    xn.p = xn_p;
    xn.n = (size_t)T * HCD;
    return wzyb_gr_norm_f32(R.p, gn.p, nullptr, nullptr, xn.p, T, NE, HC, EPS, stream);
}

// The reference constants this unit saw, for the test to size its buffers: {NE, HC, HCD}.
void dropin_constants(int* out3) {
    out3[0] = NE;
    out3[1] = HC;
    out3[2] = HCD;
}

}  // extern "C"
