/*
 * wzyb_oracle.h -- CPU restatement of wzy-flash-serve's per-layer elementwise math.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker for the CUDA path and the timed CPU
 * baseline; it is never linked into, loaded by, or called from the product library
 * (wzy-flash-serve_b200/). Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it.
 *
 * Arithmetic: fp32 as written (built with -ffp-contract=off), libm expf / sqrtf, fp16 inputs
 * widened exactly, fp16 outputs rounded to nearest-even once. Sums of squares are accumulated in
 * double (the reference accumulates in fp32 in a thread/shuffle order that no CPU loop reproduces;
 * the double sum is the value both approximate). Rows run in parallel with OpenMP.
 */
#ifndef WZYB_ORACLE_H
#define WZYB_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

float or_h2f(uint16_t h);
uint16_t or_f2h(float f);
void or_h2f_array(const uint16_t* in, float* out, int64_t n);
void or_f2h_array(const float* in, uint16_t* out, int64_t n);

void or_set_threads(int n);
int or_get_threads(void);

/* residual add + RMSNorm (fp16 I/O); x may be NULL (plain RMSNorm, residual untouched) */
void or_add_rmsnorm_f16(const uint16_t* x, uint16_t* res, const uint16_t* w, uint16_t* y, int64_t T, int n,
                        float eps, float w_offset);
/* CPU-baseline timing loop of the above on the calling thread: per-call wall time (ns) of `reps` calls */
void or_time_add_rmsnorm_f16(const uint16_t* x, uint16_t* res, const uint16_t* w, uint16_t* y, int64_t T, int n,
                             float eps, float w_offset, int reps, double* samples_ns);
/* hyper-connection form, fp32 I/O (xn_h16 != NULL additionally writes an fp16 copy of xn) */
void or_gr_norm_f32(float* R, const float* w, const float* bo, const float* inj, float* xn, uint16_t* xn_h16,
                    int64_t T, int n, int hc, float eps);
/* ... plus the Q8_0 side output of xn (per 32 elements: int8 codes, fp32 scale) */
void or_gr_norm_q8_f32(float* R, const float* w, const float* bo, const float* inj, float* xn, int8_t* q8,
                       float* s8, int64_t T, int n, int hc, float eps);
/* int8 activation quantisation per 32 and/or per 16 elements over n (multiple of 32 with q32) */
void or_quant_act_f32(const float* x, int8_t* q32, float* s32, int8_t* q16, float* s16, int64_t n);
/* block-scaled formats: element codecs and the MXFP8 / NVFP4 quantisers over n (a multiple of 32 / 16) */
uint8_t or_f2e4m3(float f);
float or_e4m32f(uint8_t b);
uint8_t or_f2e2m1(float f);
void or_quant_mxfp8(const float* x, uint8_t* q, uint8_t* s, int64_t n);
void or_quant_nvfp4(const float* x, uint8_t* q, uint8_t* s, float gs, int64_t n);
/* SwiGLU fused with Q8_0 quantisation (no activation output) */
void or_swiglu_q8_f32(const float* g, const float* u, int8_t* q, float* s, int64_t n);
/* multi-stream residual: gated write, stream mixing, scaled SiLU to fp16 */
void or_gr_write_f32(float* R, const float* blk, const float* inj, int64_t T, int n, int hc);
void or_hc_mix_f16(const uint16_t* xn, const uint16_t* gg, float* mixed, uint16_t* mixed_h16, int64_t T, int n,
                   int hc);
void or_hc_mix_f32(const float* xn, const float* gg, float* mixed, int64_t T, int n, int hc);
void or_silu_scale_f16(const float* lo, uint16_t* out, int64_t n, float scale);
/* per-head RMSNorm + partial NeoX RoPE, in place */
void or_head_norm_rope_f16(uint16_t* data, const uint16_t* gamma, const float* cos_tab, const float* sin_tab,
                           int64_t table_rows, int64_t base_pos, int64_t T, int heads, int hd, int64_t head_stride,
                           int64_t row_stride, int rot, float eps, float w_offset);
void or_head_norm_rope_f32(float* data, const float* gamma, const float* cos_tab, const float* sin_tab,
                           int64_t table_rows, int64_t base_pos, int64_t T, int heads, int hd, int64_t head_stride,
                           int64_t row_stride, int rot, float eps, float w_offset);
void or_rope_table(float* cos_tab, float* sin_tab, int64_t rows, int rot, double theta);
/* INT8 KV append (base_pos = device base + pos_offset); the full-mirror pointers may all be NULL */
void or_kv_append_int8_f32(const float* k, const float* v, int64_t T, int kvd, int64_t base_pos, int8_t* rkq,
                           uint16_t* rks, int8_t* rvq, uint16_t* rvs, int8_t* fkq, uint16_t* fks, int8_t* fvq,
                           uint16_t* fvs, int64_t ring_cap, int64_t max_ctx);
void or_k_rope_kv_append_f16(uint16_t* k, const uint16_t* gamma, const uint16_t* v, const float* cos_tab,
                             const float* sin_tab, int64_t table_rows, int64_t base_pos, int64_t T, int kv_heads, int hd,
                             int rot, float eps, float w_offset, int8_t* rkq, uint16_t* rks, int8_t* rvq, uint16_t* rvs,
                             int8_t* fkq, uint16_t* fks, int8_t* fvq, uint16_t* fvs, int64_t ring_cap, int64_t max_ctx);
/* GDN gated RMSNorm; gate_mode 0 = sigmoid(z) (reference), 1 = z*sigmoid(z) */
void or_gdn_gated_norm_f16(const uint16_t* o, const uint16_t* z, const uint16_t* gamma, uint16_t* y, int64_t T,
                           int heads, int hd, float eps, float w_offset, int gate_mode);
void or_gdn_gated_norm_f32(const float* o, const float* z, const float* gamma, float* y, int64_t T, int heads, int hd,
                           float eps, float w_offset, int gate_mode);
/* SwiGLU */
void or_swiglu_f16(const uint16_t* g, const uint16_t* u, uint16_t* out, int64_t n);
void or_swiglu_f32(const float* g, const float* u, float* out, int64_t n);
void or_swiglu_interleaved_f16(const uint16_t* gu, uint16_t* out, int64_t T, int nff);
void or_swiglu_interleaved_f32(const float* gu, float* out, int64_t T, int nff);
/* gathers; return the number of out-of-range ids */
uint32_t or_embed_gather_rows(const void* table, int64_t vocab, int64_t row_bytes, const int32_t* ids, int64_t T,
                              void* out, int oob_policy);
uint32_t or_embed_gather_bf16_f32(const uint16_t* table, int64_t vocab, int hidden, const int32_t* ids, int64_t T,
                                  float* out, int oob_policy);
uint32_t or_ple_row(int32_t t0, int32_t t1, int32_t t2, int head, int64_t rows, int32_t eos, int variant);
void or_ple_gather_f16(const uint16_t* const* tables, int heads, int64_t rows, int hd, const int32_t* ids, int64_t T,
                       const int32_t* prev_ids, int32_t eos, int variant, uint16_t* out);
/* the reference model's PLE: fp8 rows by the u64 n-gram hash, then the gate and the causal conv */
uint32_t or_ple_fp8_row(int32_t cur, int32_t p1, int32_t p0, int h, const uint64_t* mult, const uint64_t* vocab,
                        const uint64_t* off, int32_t eos);
void or_ple_gather_fp8_f32(const uint8_t* table, int row_bytes, float scale, const uint64_t* mult,
                           const uint64_t* vocab, const uint64_t* off, const int32_t* ids, int64_t T,
                           const int32_t* prev_ids, int32_t eos, float* out);
void or_ple_gate_f32(const float* key, const float* query, const float* value, float* gv, int64_t T, int n, int hc);
void or_ple_conv_f32(const float* norm, const float* cw, float* hist, const float* gv, float* R, int64_t T, int hcd,
                     float* snaps);

#ifdef __cplusplus
}
#endif
#endif
