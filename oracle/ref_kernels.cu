// ref_kernels.cu -- TEST INFRASTRUCTURE ONLY: extern "C" launchers for the reference's OWN
// elementwise kernels, compiled from its unmodified headers (include path = the reference's src/).
// Used by the GPU parity tests to pin the CPU oracle against the reference itself, and never by the
// product library. Launch shapes are the reference's own (grid/block as at its call sites).
// Same include order as the reference engine (src/wzy_engine_v2.cu), since wzy_prefill_tc.cuh
// uses helpers from wzy_mtp.cuh.
#include "wzy_stage_v2.cuh"
#include "wzy_mtp.cuh"
#include "wzy_prefill_tc.cuh"

extern "C" {

// fused_gr_norm_multi (src/wzy_kernels_v2.cuh:409-456), launched as in gr_read_fused
// (src/wzy_stage_v2.cuh:466): grid (hc, T) x 256.
int ref_fused_gr_norm_multi(float* R, const float* w_norm, const float* bo_prev, const float* inj_prev, float* xn,
                            int T, int n_embd, int hc, float eps, cudaStream_t s) {
    fused_gr_norm_multi<<<dim3(hc, T), 256, 0, s>>>(R, w_norm, bo_prev, inj_prev, xn, n_embd, hc, eps, nullptr,
                                                     nullptr);
    return (int)cudaGetLastError();
}

// fused_gr_norm_multi with its Q8_0 side output (xq8 / xs8), as gr_read_fused passes them.
int ref_fused_gr_norm_multi_q8(float* R, const float* w_norm, const float* bo_prev, const float* inj_prev, float* xn,
                               signed char* xq8, float* xs8, int T, int n_embd, int hc, float eps, cudaStream_t s) {
    fused_gr_norm_multi<<<dim3(hc, T), 256, 0, s>>>(R, w_norm, bo_prev, inj_prev, xn, n_embd, hc, eps, xq8, xs8);
    return (int)cudaGetLastError();
}

// silu_mul_quant32_multi (src/wzy_kernels_v2.cuh:1247-1279), launched as at src/wzy_stage_v2.cuh:713:
// one thread per 32-element group.
int ref_silu_mul_quant32_multi(const float* gate, const float* up, signed char* q32, float* s32, int total_g32,
                               cudaStream_t s) {
    silu_mul_quant32_multi<<<(total_g32 + 127) / 128, 128, 0, s>>>(gate, up, q32, s32, total_g32);
    return (int)cudaGetLastError();
}

// pf_gr_norm_fp16 (src/wzy_qsa_wmma.cuh:197-232), launched as at src/wzy_prefill_tc.cuh:697.
int ref_pf_gr_norm_fp16(float* R, const float* w_norm, const float* bo_prev, const float* inj_prev, __half* xn, int T,
                        int n_embd, int hc, float eps, cudaStream_t s) {
    pf_gr_norm_fp16<<<dim3(hc, T), 256, 0, s>>>(R, w_norm, bo_prev, inj_prev, xn, n_embd, hc, eps);
    return (int)cudaGetLastError();
}

// gr_write_multi (src/wzy_kernels_v2.cuh:813-828), launched as at src/wzy_stage_v2.cuh:692: grid (80, T) x 256.
int ref_gr_write_multi(float* R, const float* blk, const float* inj, int T, int n_embd, int hc, cudaStream_t s) {
    gr_write_multi<<<dim3(80, T), 256, 0, s>>>(R, blk, inj, n_embd, hc);
    return (int)cudaGetLastError();
}

// kv_append_int8_multi (src/wzy_qsa_256k.cuh:86-145), launched as at src/wzy_stage_v2.cuh:655:
// grid (8 groups, T) x 64 over the reference's KVD = 512.
int ref_kv_append_int8_multi(const float* k, const float* v, signed char* vkq, unsigned short* vks, signed char* vvq,
                             unsigned short* vvs, signed char* hkq, unsigned short* hks, signed char* hvq,
                             unsigned short* hvs, const int* dpos, int T, int ring_cap, int max_ctx, cudaStream_t s) {
    kv_append_int8_multi<<<dim3(8, T), 64, 0, s>>>(k, v, vkq, vks, vvq, vvs, hkq, hks, hvq, hvs, dpos, ring_cap,
                                                   max_ctx);
    return (int)cudaGetLastError();
}

// quant_act_multi (src/wzy_kernels_v2.cuh:58-111), launched as at src/wzy_stage_v2.cuh:697.
int ref_quant_act_multi(const float* x, signed char* q32, float* s32, signed char* q16, float* s16, int cols, int T,
                        cudaStream_t s) {
    quant_act_multi<<<((cols * T / 16) + 127) / 128, 128, 0, s>>>(x, q32, s32, q16, s16, cols, T);
    return (int)cudaGetLastError();
}

// pf_gr_up_mean_fp16 (src/wzy_qsa_wmma.cuh:234-253), launched as at src/wzy_prefill_tc.cuh:712.
int ref_pf_gr_up_mean_fp16(const __half* xn, const __half* gg, float* mixed, __half* mixed16, int T, int n_embd,
                           cudaStream_t s) {
    pf_gr_up_mean_fp16<<<(int)(((size_t)T * n_embd + 255) / 256), 256, 0, s>>>(xn, gg, mixed, mixed16, T, n_embd);
    return (int)cudaGetLastError();
}

// gr_up_gate_mean_pf_kernel (src/wzy_prefill_tc.cuh:37-51), one element per thread.
int ref_gr_up_gate_mean_pf(const float* xn, const float* gg, float* mixed, int T, int n_embd, cudaStream_t s) {
    gr_up_gate_mean_pf_kernel<<<(int)(((size_t)T * n_embd + 255) / 256), 256, 0, s>>>(xn, gg, mixed, T, n_embd);
    return (int)cudaGetLastError();
}

// silu_div_hc_to_fp16_kernel (src/wzy_prefill_tc.cuh:24-35), launched as at src/wzy_prefill_tc.cuh:706.
int ref_silu_div_hc_to_fp16(const float* lo, __half* out, int n, float inv_hc, cudaStream_t s) {
    silu_div_hc_to_fp16_kernel<<<(int)((((size_t)n + 1) / 2 + 255) / 256), 256, 0, s>>>(lo, out, n, inv_hc);
    return (int)cudaGetLastError();
}

// fused_head_norm_rope_multi (src/wzy_qsa_256k.cuh:50-84), grid (heads, T) x 128 (T <= 65535).
int ref_fused_head_norm_rope_multi(float* data, const float* gamma, const float* cos_tab, const float* sin_tab,
                                   const int* base_pos_dev, int T, int heads, int hd, int head_stride, int row_stride,
                                   float eps, cudaStream_t s) {
    fused_head_norm_rope_multi<<<dim3(heads, T), 128, 0, s>>>(data, gamma, cos_tab, sin_tab, base_pos_dev, heads, hd,
                                                              head_stride, row_stride, eps);
    return (int)cudaGetLastError();
}

// build_rope_cos_sin_host (src/wzy_qsa_256k.cuh:33-46): the reference's host table (32 pairs).
void ref_build_rope_cos_sin_host(int max_ctx, float theta, float* h_cos, float* h_sin) {
    build_rope_cos_sin_host(max_ctx, theta, h_cos, h_sin);
}

// pf_gdn_rmsnorm_gate_parallel (src/wzy_qsa_wmma.cuh:178-195), grid (hv, T) x 128.
int ref_pf_gdn_rmsnorm_gate_parallel(const float* o, const float* z, const float* gamma, __half* y, int T, int hv,
                                     float eps, cudaStream_t s) {
    pf_gdn_rmsnorm_gate_parallel<<<dim3(hv, T), 128, 0, s>>>(o, z, gamma, y, hv, eps);
    return (int)cudaGetLastError();
}

// silu_mul_multi (src/wzy_kernels_v2.cuh:1240-1244), launched as at src/wzy_stage_v2.cuh:733.
int ref_silu_mul_multi(const float* gate, const float* up, float* out, int total, cudaStream_t s) {
    silu_mul_multi<<<(total + 255) / 256, 256, 0, s>>>(gate, up, out, total);
    return (int)cudaGetLastError();
}

// pf_silu_mul_interleaved_to_fp16 (src/wzy_prefill_tc.cuh:69-80), launched as at :942.
int ref_pf_silu_mul_interleaved_to_fp16(const float* gu, __half* out, int T, int nff, cudaStream_t s) {
    pf_silu_mul_interleaved_to_fp16<<<(int)((((size_t)T * nff + 1) / 2 + 255) / 256), 256, 0, s>>>(gu, out, T, nff);
    return (int)cudaGetLastError();
}

// mtp_gather_bf16_emb (src/wzy_kernels_v2.cuh:27-36): table [NVOCAB=248320, NE=2560] bf16, launched as at
// src/wzy_stage_v2.cuh:567-568.
int ref_mtp_gather_bf16_emb(const uint16_t* table, const int* toks, float* out, int T, cudaStream_t s) {
    mtp_gather_bf16_emb<<<dim3((NE + 255) / 256, T), 256, 0, s>>>(table, toks, out, T);
    return (int)cudaGetLastError();
}

// ple_group_multi (src/wzy_kernels_v2.cuh:1299-1319): row RMSNorm twin, grid (hc, T) x 256.
int ref_ple_group_multi(const float* x, const float* gamma, float* y, int T, int n_embd, int hc, float eps,
                        cudaStream_t s) {
    ple_group_multi<<<dim3(hc, T), 256, 0, s>>>(x, gamma, y, n_embd, hc, eps);
    return (int)cudaGetLastError();
}

// ple_gate_gv_multi (src/wzy_kernels_v2.cuh:1321-1346), launched as at src/wzy_stage_v2.cuh:592.
int ref_ple_gate_gv_multi(const float* key, const float* query, const float* value, float* gv, int T, int hc,
                          int n_embd, cudaStream_t s) {
    ple_gate_gv_multi<<<dim3(hc, T), 256, 0, s>>>(key, query, value, gv, hc, n_embd);
    return (int)cudaGetLastError();
}

// ple_conv_multi (src/wzy_kernels_v2.cuh:1348-1373), launched as at src/wzy_stage_v2.cuh:594.
int ref_ple_conv_multi(const float* norm, const float* cw, float* hist, const float* gv, float* R, int hcd, int T,
                       float* snaps, cudaStream_t s) {
    ple_conv_multi<<<(hcd + 255) / 256, 256, 0, s>>>(norm, cw, hist, gv, R, hcd, PLE_NG, PLE_KERN, T, snaps);
    return (int)cudaGetLastError();
}

// The reference's PLE row source (PleSrc, src/wzy_stage_v2.cuh:215-324) opened on a GGUF file and asked
// for rows idx[0..n): its own header parse (scale key, tensor offset) and fp8 decode (the 256-entry
// table with the NaN codes as 0, times the scale), through its row cache. Host code.
int ref_ple_src_rows(const char* path, const uint64_t* idx, int n, float* out, float* scale_out,
                     int* row_bytes_out, uint64_t* rows_out) {
    PleSrc* src = new PleSrc();
    if (!src->open(path)) {
        if (src->base) munmap(src->base, src->sz);
        delete src;
        return 1;
    }
    for (int i = 0; i < n; ++i) src->row(idx[i], out + (size_t)i * PLE_HEAD);
    *scale_out = src->scale;
    *row_bytes_out = src->row_bytes;
    *rows_out = src->rows;
    munmap(src->base, src->sz);
    delete src;
    return 0;
}

int ref_dims(int* ne, int* nvocab) {
    *ne = NE;
    *nvocab = NVOCAB;
    return 0;
}

}  // extern "C"
