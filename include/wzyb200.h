/*
 * wzyb200.h -- C ABI of the B200 (sm_100a) per-layer fused elementwise kernels.
 *
 * Drop-in replacements for the elementwise kernels that the layer executors of wzy-flash-serve
 * launch directly with <<<grid, block, 0, stream>>>:
 *   StageGpu::record_forward            (src/wzy_stage_v2.cuh:476-857, decode / verify, T <= 8)
 *   PrefillStageCtx::run_stage_prefill  (src/wzy_prefill_tc.cuh:546-1058, chunked prefill)
 * plus the token-embedding and 3-gram PLE gathers that the engine driver does on the host
 * (src/wzy_engine_v2.cu:862-875, :943-978, :1210-1265).
 *
 * Conventions (shared by every entry point):
 *  - All tensors are caller-owned DEVICE buffers; nothing here allocates, synchronises or reads
 *    device memory from the host, so every launcher may be recorded into a CUDA graph by stream
 *    capture (call wzyb_prepare_device() once per device before the first capture).
 *  - fp16 tensors are passed as uint16_t* (IEEE binary16 bit patterns, i.e. __half storage);
 *    fp32 tensors as float*. Arithmetic is fp32; fp16 outputs are rounded to nearest-even once.
 *  - Row-major layouts; every row / head start must be 16-byte aligned (checked).
 *  - The kernel is enqueued on `stream` (a cudaStream_t) of the CURRENT device; the caller sets the
 *    device, as StageGpu does with cudaSetDevice(dev).
 *  - Return value: 0 = enqueued; > 0 = the cudaError_t of the launch; < 0 = WZYB_ERR_* argument
 *    error detected on the host before anything was enqueued. Launchers never exit the process.
 *  - Kernels never trap. If a device-side check fails (a position outside the RoPE table, a
 *    bounded wait that gave up) they record a WZYB_FAULT_* bit, skip the affected work and return;
 *    wzyb_read_faults() reports and clears those bits.
 */
#ifndef WZYB200_H
#define WZYB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* wzyb_stream_t; /* identical to cudaStream_t */

/* ---- status codes ------------------------------------------------------------------------ */
#define WZYB_OK 0
#define WZYB_ERR_NULL (-1)   /* a required pointer is NULL                                     */
#define WZYB_ERR_ALIGN (-2)  /* a pointer / row / head start is not 16-byte aligned            */
#define WZYB_ERR_SHAPE (-3)  /* a size is out of the supported range or inconsistent           */
#define WZYB_ERR_DEVICE (-4) /* the current device is not an sm_100 (B200) GPU, or no device   */
#define WZYB_ERR_VALUE (-5)  /* an enum / mode argument has an unknown value                   */

/* ---- device fault bits (wzyb_read_faults) ------------------------------------------------ */
#define WZYB_FAULT_WAIT_TIMEOUT 0x1u /* a TMA / mbarrier wait gave up after its time limit      */
#define WZYB_FAULT_POS_RANGE 0x2u    /* a RoPE position fell outside [0, table_rows)           */

/* ---- modes --------------------------------------------------------------------------------- */
#define WZYB_GATE_SIGMOID 0 /* y = norm(o)*gamma*sigmoid(z): what the reference computes        */
#define WZYB_GATE_SILU 1    /* y = norm(o)*gamma*z*sigmoid(z): the literal "silu(z)" reading    */

#define WZYB_OOB_CLAMP 0    /* out-of-range id -> clamp to [0, vocab-1] (device gather)          */
#define WZYB_OOB_ZERO_ID 1  /* out-of-range id -> row 0 (host gather)                            */

#define WZYB_PLE_HASH_C_PRECEDENCE 0 /* row = (a ^ b ^ (c + head)) mod rows  (formula as C parses it) */
#define WZYB_PLE_HASH_XOR_THEN_ADD 1 /* row = ((a ^ b ^ c) + head) mod rows                           */
#define WZYB_PLE_EOS_DEFAULT 248044  /* PLE_EOS, src/wzy_kernels_v2.cuh:19                            */

/* ============================================================================================
 * Residual add + RMSNorm.
 *   v = residual + x;  residual <- v (only when x != NULL);
 *   y = (v * rsqrt(mean(v^2) + eps)) * (w_offset + weight)
 * x == NULL: plain row RMSNorm of `residual` (residual is not written).
 * w_offset = 1.0f gives the zero-centred "(1+w)" weight, 0.0f the raw weight.
 * Shapes: x, residual, y [T, hidden]; weight [hidden]. hidden % 8 == 0, 8 <= hidden <= 16384.
 * Replaces fused_gr_norm_multi (src/wzy_kernels_v2.cuh:409-456, launched from gr_read_fused at
 * src/wzy_stage_v2.cuh:466) and pf_gr_norm_fp16 (src/wzy_qsa_wmma.cuh:197-232, launched at
 * src/wzy_prefill_tc.cuh:697) in their single-stream (hc = 1, inject gate 1.0) form.
 * ========================================================================================== */
int wzyb_add_rmsnorm_f16(const uint16_t* x, uint16_t* residual, const uint16_t* weight, uint16_t* y,
                         int64_t T, int hidden, float eps, float w_offset, wzyb_stream_t stream);

/* Hyper-connection form with the reference's own fp32 types, argument for argument:
 *   R [T, hc, n_embd] fp32 (in/out), w_norm [hc, n_embd], bo_prev [T, n_embd] or NULL,
 *   inj_prev [T, hc] or NULL, xn [T, hc, n_embd].
 *   v = R + bo_prev[t] * 2*sigmoid(inj_prev[t,c]/hc)   (gate 1.0 when inj_prev == NULL)
 *   R <- v (when bo_prev != NULL); xn = (v * rsqrt(mean(v^2) + eps)) * w_norm[c]
 * _f32 writes xn as fp32 (fused_gr_norm_multi, src/wzy_kernels_v2.cuh:409-456, without the
 * optional Q8 side output); _f32_f16 writes xn as fp16 (pf_gr_norm_fp16, src/wzy_qsa_wmma.cuh:197-232). */
int wzyb_gr_norm_f32(float* R, const float* w_norm, const float* bo_prev, const float* inj_prev, float* xn,
                     int64_t T, int n_embd, int hc, float eps, wzyb_stream_t stream);
int wzyb_gr_norm_f32_f16(float* R, const float* w_norm, const float* bo_prev, const float* inj_prev,
                         uint16_t* xn, int64_t T, int n_embd, int hc, float eps, wzyb_stream_t stream);
/* ... with fused_gr_norm_multi's optional Q8_0 side output as well (src/wzy_kernels_v2.cuh:440-454):
 * xq8 [T, hc, n_embd] int8 and xs8 [T, hc, n_embd/32] fp32; per 32-element group d = amax/127,
 * q = rint(xn * 127/amax) clamped to [-127, 127]. n_embd % 32 == 0, n_embd <= 16384. */
int wzyb_gr_norm_q8_f32(float* R, const float* w_norm, const float* bo_prev, const float* inj_prev, float* xn,
                        int8_t* xq8, float* xs8, int64_t T, int n_embd, int hc, float eps, wzyb_stream_t stream);

/* ============================================================================================
 * Multi-stream (hyper-connection) residual outside the norm. n_embd % 8 == 0, 1 <= hc <= 64.
 * ========================================================================================== */
/* R[t,c,:] += blk[t,:] * 2*sigmoid(inj[t,c]/hc)  (gate 1.0 when inj == NULL), fp32, in place.
 * R [T, hc, n_embd], blk [T, n_embd], inj [T, hc]. Replaces gr_write_multi
 * (src/wzy_kernels_v2.cuh:813-828; launched at src/wzy_stage_v2.cuh:585/693/800 and
 * src/wzy_prefill_tc.cuh:810/926/1054). */
int wzyb_gr_write_f32(float* R, const float* blk, const float* inj, int64_t T, int n_embd, int hc,
                      wzyb_stream_t stream);
/* Stream mixing  mixed[t,:] = (1/hc) * sum_c xn[t,c,:] / (1 + exp(-gg[t,c,:])).
 * xn, gg [T, hc, n_embd]; mixed [T, n_embd] fp32 and/or mixed_f16 [T, n_embd] fp16 (either may be
 * NULL, not both). _f16: pf_gr_up_mean_fp16 (src/wzy_qsa_wmma.cuh:234-253, launched at
 * src/wzy_prefill_tc.cuh:712), whose 4 streams give the scale 0.25. _f32: gr_up_gate_mean_pf_kernel
 * (src/wzy_prefill_tc.cuh:37-51). */
int wzyb_hc_mix_f16(const uint16_t* xn, const uint16_t* gg, float* mixed, uint16_t* mixed_f16, int64_t T,
                    int n_embd, int hc, wzyb_stream_t stream);
int wzyb_hc_mix_f32(const float* xn, const float* gg, float* mixed, int64_t T, int n_embd, int hc,
                    wzyb_stream_t stream);
/* out = fp16(silu(lo * scale)), n % 8 == 0: silu_div_hc_to_fp16_kernel (src/wzy_prefill_tc.cuh:24-35,
 * launched at :706 with scale 1/hc on the low-rank mixing activations). */
int wzyb_silu_scale_f16(const float* lo, uint16_t* out, int64_t n, float scale, wzyb_stream_t stream);

/* ============================================================================================
 * Per-head RMSNorm + partial NeoX RoPE, in place.
 *   p = data + t*row_stride + h*head_stride  (h < heads, head_dim elements)
 *   p *= rsqrt(mean(p^2) + eps) * (w_offset + gamma)           gamma [head_dim], shared by heads
 *   for i < rot_dims/2:  (a, d) = (p[i], p[i + rot_dims/2]);
 *       p[i] = a*cos - d*sin;  p[i + rot_dims/2] = a*sin + d*cos
 *   cos/sin = cos_tab/sin_tab[pos * (rot_dims/2) + i], pos = (d_base_pos ? *d_base_pos : 0)
 *             + pos_offset + t, and must lie in [0, table_rows) (else WZYB_FAULT_POS_RANGE and the
 *             token is left un-rotated).
 * head_dim in {64, 128, 256}; rot_dims % 16 == 0, 0 <= rot_dims <= head_dim; strides in elements.
 * Replaces fused_head_norm_rope_multi (src/wzy_qsa_256k.cuh:50-84; launched at
 * src/wzy_stage_v2.cuh:638-643 and src/wzy_prefill_tc.cuh:862-867), whose rot_dims is fixed at 64.
 * ========================================================================================== */
int wzyb_head_norm_rope_f16(uint16_t* data, const uint16_t* gamma, const float* cos_tab, const float* sin_tab,
                            int64_t table_rows, const int32_t* d_base_pos, int64_t pos_offset, int64_t T,
                            int heads, int head_dim, int64_t head_stride, int64_t row_stride, int rot_dims,
                            float eps, float w_offset, wzyb_stream_t stream);
int wzyb_head_norm_rope_f32(float* data, const float* gamma, const float* cos_tab, const float* sin_tab,
                            int64_t table_rows, const int32_t* d_base_pos, int64_t pos_offset, int64_t T,
                            int heads, int head_dim, int64_t head_stride, int64_t row_stride, int rot_dims,
                            float eps, float w_offset, wzyb_stream_t stream);

/* q and k of one token in ONE launch (what the reference does with two launches,
 * src/wzy_prefill_tc.cuh:862-865). Each tensor has its own gamma, head count and strides. */
typedef struct {
    void* data;          /* [T, ...]; element type set by the entry point: fp16 for the _f16 calls,
                            k's type for wzyb_qk_rope_kv_append_*                                 */
    const void* gamma;   /* [head_dim]                                                            */
    int heads;
    int64_t head_stride; /* elements between heads of one token                                  */
    int64_t row_stride;  /* elements between tokens                                              */
} wzyb_head_tensor;

int wzyb_qk_norm_rope_f16(const wzyb_head_tensor* q, const wzyb_head_tensor* k, const float* cos_tab,
                          const float* sin_tab, int64_t table_rows, const int32_t* d_base_pos, int64_t pos_offset,
                          int64_t T, int head_dim, int rot_dims, float eps, float w_offset, wzyb_stream_t stream);

/* RoPE cos/sin tables [rows, rot_dims/2] fp32: angle = pos * theta^(-2i/rot_dims) in fp64, then
 * cos/sin in fp64 rounded to fp32 -- build_rope_cos_sin_host (src/wzy_qsa_256k.cuh:33-46).
 * _host fills host arrays (the reference's own procedure, libm); the device version fills device
 * arrays on `stream` with CUDA's fp64 cos/sin. */
int wzyb_rope_table_host_f32(float* h_cos, float* h_sin, int64_t rows, int rot_dims, double theta);
int wzyb_rope_table_f32(float* d_cos, float* d_sin, int64_t rows, int rot_dims, double theta,
                        wzyb_stream_t stream);

/* ============================================================================================
 * INT8 KV-cache append, optionally fused with k's per-head RMSNorm + partial NeoX RoPE.
 * k, v [T, kv_heads * head_dim] (kvd = kv_heads * head_dim, head_dim in {64, 128, 256}).
 * Per 64-element group of k (after RoPE) and of v:  sh = fp16(max|x| / 127), d = float(sh),
 *   q = d > 0 ? rint(x / d) : 0 clamped to [-127, 127]; codes [cell, kvd] int8, scales
 *   [cell, kvd/64] fp16 (bits in uint16_t).
 * Cells, for pos = (d_base_pos ? *d_base_pos : 0) + pos_offset + t and end = that base + T:
 *   tokens with pos outside [0, max_ctx) are not appended;
 *   ring: ring_cap <= 8192  -> cell pos % ring_cap, written when pos >= end - ring_cap;
 *         ring_cap  > 8192  -> pos < 4096 (pinned sink): cell pos;
 *                              else cell 4096 + (pos - 4096) % (ring_cap - 4096), written when
 *                              pos >= max(4096, end - (ring_cap - 4096));
 *   full-context mirror (all four full_* pointers, or none): cell pos.
 * Replaces kv_append_int8_multi (src/wzy_qsa_256k.cuh:86-145 with kv_is_in_vram / kv_vram_slot at
 * :17-29; launched at src/wzy_stage_v2.cuh:655, src/wzy_prefill_tc.cuh:878 and src/wzy_mtp.cuh:681).
 * ========================================================================================== */
typedef struct {
    int8_t* ring_k_q;    /* [ring_cap, kvd]     */
    uint16_t* ring_k_s;  /* [ring_cap, kvd/64]  */
    int8_t* ring_v_q;
    uint16_t* ring_v_s;
    int8_t* full_k_q;    /* [max_ctx, kvd] or NULL */
    uint16_t* full_k_s;
    int8_t* full_v_q;
    uint16_t* full_v_s;
    int64_t ring_cap;
    int64_t max_ctx;
} wzyb_kv_cache;
/* The append alone (k as given): kv_append_int8_multi. */
int wzyb_kv_append_int8_f32(const float* k, const float* v, int64_t T, int kv_heads, int head_dim,
                            const int32_t* d_base_pos, int64_t pos_offset, const wzyb_kv_cache* cache,
                            wzyb_stream_t stream);
/* k normalised and rotated in place exactly as wzyb_head_norm_rope_* (head_stride = head_dim,
 * row_stride = kvd, gamma k_gamma), then k and v appended: the reference's k
 * fused_head_norm_rope_multi (src/wzy_stage_v2.cuh:640-641, src/wzy_prefill_tc.cuh:864-865) and
 * kv_append_int8_multi in one launch. */
int wzyb_k_rope_kv_append_f32(float* k, const float* k_gamma, const float* v, const float* cos_tab,
                              const float* sin_tab, int64_t table_rows, const int32_t* d_base_pos, int64_t pos_offset,
                              int64_t T, int kv_heads, int head_dim, int rot_dims, float eps, float w_offset,
                              const wzyb_kv_cache* cache, wzyb_stream_t stream);
/* The same with the token's q heads normed and rotated in place in the same launch (their own gamma
 * and strides in *q, e.g. the reference's q interleaved with its gate, head_stride = 2*head_dim): the
 * reference's three launches -- fused_head_norm_rope_multi on q and on k, then kv_append_int8_multi
 * (src/wzy_stage_v2.cuh:638-655, src/wzy_prefill_tc.cuh:862-878) -- as one. q->data and q->gamma
 * have the element type of k. The q heads of different tokens must not overlap (T > 1 needs
 * q->row_stride >= (q->heads - 1) * q->head_stride + head_dim) and q must not share bytes with k or v;
 * either is WZYB_ERR_SHAPE. */
int wzyb_qk_rope_kv_append_f32(const wzyb_head_tensor* q, float* k, const float* k_gamma, const float* v,
                               const float* cos_tab, const float* sin_tab, int64_t table_rows,
                               const int32_t* d_base_pos, int64_t pos_offset, int64_t T, int kv_heads, int head_dim,
                               int rot_dims, float eps, float w_offset, const wzyb_kv_cache* cache,
                               wzyb_stream_t stream);
int wzyb_qk_rope_kv_append_f16(const wzyb_head_tensor* q, uint16_t* k, const uint16_t* k_gamma, const uint16_t* v,
                               const float* cos_tab, const float* sin_tab, int64_t table_rows,
                               const int32_t* d_base_pos, int64_t pos_offset, int64_t T, int kv_heads, int head_dim,
                               int rot_dims, float eps, float w_offset, const wzyb_kv_cache* cache,
                               wzyb_stream_t stream);
int wzyb_k_rope_kv_append_f16(uint16_t* k, const uint16_t* k_gamma, const uint16_t* v, const float* cos_tab,
                              const float* sin_tab, int64_t table_rows, const int32_t* d_base_pos, int64_t pos_offset,
                              int64_t T, int kv_heads, int head_dim, int rot_dims, float eps, float w_offset,
                              const wzyb_kv_cache* cache, wzyb_stream_t stream);

/* ============================================================================================
 * GDN output gated RMSNorm, per head of head_dim:
 *   y = ((o * rsqrt(mean(o^2) + eps)) * (w_offset + gamma[col])) / (1 + exp(-z))    (SIGMOID)
 *   y = ((o * rsqrt(mean(o^2) + eps)) * (w_offset + gamma[col])) * (z / (1 + exp(-z))) (SILU)
 * o, z, y [T, heads, head_dim]; gamma [head_dim] shared by heads; head_dim in {64, 128, 256}.
 * Replaces pf_gdn_rmsnorm_gate_parallel (src/wzy_qsa_wmma.cuh:178-195, launched at
 * src/wzy_prefill_tc.cuh:845) and the gated-norm tail of fused_gdn_step_norm_multi
 * (src/wzy_kernels_v2.cuh:966-976). The reference multiplies by sigmoid(z) at every site.
 * ========================================================================================== */
int wzyb_gdn_gated_norm_f16(const uint16_t* o, const uint16_t* z, const uint16_t* gamma, uint16_t* y,
                            int64_t T, int heads, int head_dim, float eps, float w_offset, int gate_mode,
                            wzyb_stream_t stream);
/* fp32 o/z/gamma in, fp16 y out: pf_gdn_rmsnorm_gate_parallel's own types. */
int wzyb_gdn_gated_norm_f32_f16(const float* o, const float* z, const float* gamma, uint16_t* y, int64_t T,
                                int heads, int head_dim, float eps, float w_offset, int gate_mode,
                                wzyb_stream_t stream);

/* ============================================================================================
 * SwiGLU activation  out = (g / (1 + exp(-g))) * u.
 * Separate layout: gate, up, out [n], n % 8 == 0 -- silu_mul_multi (src/wzy_kernels_v2.cuh:1240-1244,
 * launched at src/wzy_stage_v2.cuh:733).
 * Interleaved layout: gu [T, 2*nff] = [gate | up] per row -> out [T, nff], nff % 8 == 0 --
 * pf_silu_mul_interleaved_to_fp16 (src/wzy_prefill_tc.cuh:69-80, launched at :942).
 * ========================================================================================== */
int wzyb_swiglu_f16(const uint16_t* gate, const uint16_t* up, uint16_t* out, int64_t n, wzyb_stream_t stream);
int wzyb_swiglu_f32(const float* gate, const float* up, float* out, int64_t n, wzyb_stream_t stream);
/* SwiGLU fused with Q8_0 quantisation and no activation output: silu_mul_quant32_multi
 * (src/wzy_kernels_v2.cuh:1247-1279, launched at src/wzy_stage_v2.cuh:713). q32 [n] int8, s32 [n/32]
 * fp32, n % 32 == 0; the activation uses the reference's expression (IEEE divide). */
int wzyb_swiglu_q8_f32(const float* gate, const float* up, int8_t* q32, float* s32, int64_t n, wzyb_stream_t stream);

/* ============================================================================================
 * fp32 activation rows x [T, cols] to int8 GEMM inputs in one pass: per 32-element group q32 [T, cols]
 * int8 + s32 [T, cols/32] fp32, and/or per 16-element group q16 + s16 [T, cols/16]; each group
 * d = amax/127, q = rint(x * 127/amax) clamped to [-127, 127]. Either pair may be NULL (not both);
 * cols % 32 == 0 with q32, % 16 == 0 otherwise. Replaces quant_act_multi (src/wzy_kernels_v2.cuh:58-111;
 * launched at src/wzy_stage_v2.cuh:449/468/609/630/697 and src/wzy_mtp.cuh:652-700).
 * ========================================================================================== */
int wzyb_quant_act_f32(const float* x, int8_t* q32, float* s32, int8_t* q16, float* s16, int64_t T, int cols,
                       wzyb_stream_t stream);

/* ============================================================================================
 * Block-scaled GEMM inputs for sm_100's tensor cores, in the same passes: the B200 form of the
 * quantisation epilogue that the reference writes as int8 (quant_act_multi, the xq8 path of
 * fused_gr_norm_multi, silu_mul_quant32_multi). Codes and scales are row-major over the flat
 * element order; scale bytes need no alignment, codes 16-byte aligned.
 *  MXFP8 (E4M3 elements, E8M0 scale, block 32): q [n] e4m3 bytes, s [n/32] E8M0 bytes. Per block:
 *    X = 2^ceil(log2(amax / 448)) -- the smallest power of two keeping the block within +-448, so
 *    nothing clips (OCP's floor(log2 amax) - 8 clips the block maximum by up to 12.5 %) -- s = log2(X)
 *    + 127 (0 for an all-zero block), q = e4m3(x / X) round-to-nearest-even; inf/NaN: s = 0xFF.
 *  NVFP4 (block 16, per-tensor scale gs): q [n/2] bytes (element 2i in the low nibble), s [n/16] e4m3
 *    bytes. Per block: s = e4m3((amax * gs) / 6); q = e2m1(x * (gs / float(s))) round-to-nearest-even,
 *    saturating at +-6 (0 when float(s) == 0). x ~= e2m1 * float(s) / gs.
 * ========================================================================================== */
int wzyb_quant_act_mxfp8_f32(const float* x, uint8_t* q, uint8_t* s, int64_t T, int cols, wzyb_stream_t stream);
int wzyb_quant_act_nvfp4_f32(const float* x, uint8_t* q, uint8_t* s, float global_scale, int64_t T, int cols,
                             wzyb_stream_t stream);
/* Either format with a choice of scale-factor layout, for a GEMM that takes the codes as its A (or B)
 * operand [rows, cols] (rows = T here, T * hc for the norm):
 *  format     WZYB_BLOCK_MXFP8 (global_scale unused) or WZYB_BLOCK_NVFP4;
 *  sf_layout  WZYB_SF_ROW_MAJOR: s [rows, cols/G] bytes (G = 32 MXFP8, 16 NVFP4), as the entry points
 *               above;
 *             WZYB_SF_TILED_128X4: the scale layout of sm_100's block-scaled MMA operands (what a
 *               tcgen05 GEMM copies to tensor memory, and cuBLASLt's block-scaled GEMMs read): the
 *               [rows, cols/G] scale matrix in tiles of 128 rows x 4 scale columns, 512 bytes each;
 *               the ceil(cols/G/4) tiles of one 128-row band are consecutive, and inside a tile
 *               scale (r, c) sits at byte (r % 32) * 16 + (r / 32) * 4 + c. s must hold
 *               ceil(rows/128) * 128 * ceil(cols/G/4) * 4 bytes; bytes of padding rows and columns are
 *               not written.
 * Codes are row-major [rows, cols] in both cases. */
#define WZYB_BLOCK_MXFP8 0
#define WZYB_BLOCK_NVFP4 1
#define WZYB_SF_ROW_MAJOR 0
#define WZYB_SF_TILED_128X4 1
int wzyb_quant_act_block_f32(const float* x, uint8_t* q, uint8_t* s, int format, int sf_layout, float global_scale,
                             int64_t T, int cols, wzyb_stream_t stream);
int wzyb_gr_norm_block_f32(float* R, const float* w_norm, const float* bo_prev, const float* inj_prev, float* xn,
                           uint8_t* xq, uint8_t* xs, int format, int sf_layout, float global_scale, int64_t T,
                           int n_embd, int hc, float eps, wzyb_stream_t stream);
/* SwiGLU straight to a block format with a choice of scale layout: gate, up and the codes [rows, cols]
 * (cols % 32 == 0), format and sf_layout as above. */
int wzyb_swiglu_block_f32(const float* gate, const float* up, uint8_t* q, uint8_t* s, int format, int sf_layout,
                          float global_scale, int64_t rows, int cols, wzyb_stream_t stream);
/* SwiGLU (the reference's expression) straight to the block formats; n % 32 == 0. */
int wzyb_swiglu_mxfp8_f32(const float* gate, const float* up, uint8_t* q, uint8_t* s, int64_t n,
                          wzyb_stream_t stream);
int wzyb_swiglu_nvfp4_f32(const float* gate, const float* up, uint8_t* q, uint8_t* s, float global_scale, int64_t n,
                          wzyb_stream_t stream);
/* wzyb_gr_norm_f32 with xn also written in a block format (as wzyb_gr_norm_q8_f32 writes Q8_0). */
int wzyb_gr_norm_mxfp8_f32(float* R, const float* w_norm, const float* bo_prev, const float* inj_prev, float* xn,
                           uint8_t* xq, uint8_t* xs, int64_t T, int n_embd, int hc, float eps, wzyb_stream_t stream);
int wzyb_gr_norm_nvfp4_f32(float* R, const float* w_norm, const float* bo_prev, const float* inj_prev, float* xn,
                           uint8_t* xq, uint8_t* xs, float global_scale, int64_t T, int n_embd, int hc, float eps,
                           wzyb_stream_t stream);
int wzyb_swiglu_interleaved_f16(const uint16_t* gu, uint16_t* out, int64_t T, int nff, wzyb_stream_t stream);
int wzyb_swiglu_interleaved_f32_f16(const float* gu, uint16_t* out, int64_t T, int nff, wzyb_stream_t stream);

/* ============================================================================================
 * Token-embedding gather: out[t, :] = table[id(t), :], bit-exact row copy.
 * id(t) = ids[t] when 0 <= ids[t] < vocab; otherwise clamp to [0, vocab-1] (WZYB_OOB_CLAMP, as the
 * device gather mtp_gather_bf16_emb, src/wzy_kernels_v2.cuh:27-36) or 0 (WZYB_OOB_ZERO_ID, as the
 * host gather stage_one_emb, src/wzy_engine_v2.cu:862-875). If d_oob_count != NULL the number of
 * out-of-range ids is ADDED to *d_oob_count (a device uint32).
 * _rows: any element type, row_bytes % 16 == 0.  _f16: row_bytes = 2*hidden.
 * _bf16_f32: bf16 table -> fp32 rows, exactly mtp_gather_bf16_emb's conversion.
 * ========================================================================================== */
int wzyb_embed_gather_rows(const void* table, int64_t vocab, int64_t row_bytes, const int32_t* ids, int64_t T,
                           void* out, int oob_policy, uint32_t* d_oob_count, wzyb_stream_t stream);
int wzyb_embed_gather_f16(const uint16_t* table, int64_t vocab, int hidden, const int32_t* ids, int64_t T,
                          uint16_t* out, int oob_policy, uint32_t* d_oob_count, wzyb_stream_t stream);
int wzyb_embed_gather_bf16_f32(const uint16_t* table, int64_t vocab, int hidden, const int32_t* ids, int64_t T,
                               float* out, int oob_policy, uint32_t* d_oob_count, wzyb_stream_t stream);

/* ============================================================================================
 * 16-head 3-gram PLE gather (fp16 tables).
 *   For token i with history (t0, t1, t2) = (ids[i], ids[i-1], ids[i-2]):
 *     history ids before the first token come from prev_ids = {id[-2], id[-1]} (host array, copied
 *     into the launch; NULL = no history). A history id that is negative or == eos_id cuts the
 *     context: it and every older id become eos_id (the reference's rule, src/wzy_engine_v2.cu:946-953).
 *     a = t0*0x9E3779B1, b = t1*0x85EBCA77, c = t2*0xC2B2AE3D  (uint32 wrap-around)
 *     row_h = (a ^ b ^ (c + h)) mod rows_per_table   (WZYB_PLE_HASH_C_PRECEDENCE)
 *           = ((a ^ b ^ c) + h) mod rows_per_table   (WZYB_PLE_HASH_XOR_THEN_ADD)
 *     out[i, h*head_dim : (h+1)*head_dim] = tables[h][row_h, :]
 * tables: HOST array of `heads` device pointers (heads <= 32), each [rows_per_table, head_dim];
 * out [T, heads*head_dim]; head_dim % 8 == 0. Bit-exact copy.
 * Replaces the host staging loops stage_ple_window / stage_emb_ple_pf (src/wzy_engine_v2.cu:943-978,
 * :1210-1265) with the table format and hash of the fp16 synthetic configuration.
 * ========================================================================================== */
int wzyb_ple_gather_f16(const uint16_t* const* tables, int heads, int64_t rows_per_table, int head_dim,
                        const int32_t* ids, int64_t T, const int32_t* prev_ids, int32_t eos_id, int hash_variant,
                        uint16_t* out, wzyb_stream_t stream);

/* ============================================================================================
 * PLE in the reference model's own format and its downstream block.
 * ========================================================================================== */
/* 2-gram / 3-gram u64 hash: for token t with history cut as above (c0 = id[t], c1, c2):
 *   m2 = c0*mult[0] ^ c1*mult[1];  m3 = m2 ^ c2*mult[2]       (u64 wrap; c0 sign-extended)
 *   head h < 8: row = (uint32)(m2 % vocab[h] + off[h]);  h >= 8: (uint32)(m3 % vocab[h] + off[h]) */
typedef struct {
    uint64_t mult[3];
    uint64_t vocab[16];
    uint64_t off[16];
} wzyb_ple_fp8_hash;
/* The reference's constants (stage_ple_window, src/wzy_engine_v2.cu:909-916): 320,001,446 rows. */
int wzyb_ple_fp8_reference_hash(wzyb_ple_fp8_hash* out);
/* out[t, h*row_bytes + i] = e4m3(table[row_h, i]) * scale, fp32 [T, 16*row_bytes]; the e4m3 NaN codes
 * (0x7F, 0xFF) read as signed zero. table [table_rows, row_bytes] fp8 e4m3 bytes, row_bytes % 16 == 0
 * (the reference's 160); every off[h] + vocab[h] <= table_rows; prev_ids as wzyb_ple_gather_f16.
 * Replaces stage_ple_window / stage_emb_ple_pf (src/wzy_engine_v2.cu:943-978, :1210-1265) with
 * PleSrc's row decode (src/wzy_stage_v2.cuh:215-324) and the H2D copy of the staged rows. */
int wzyb_ple_gather_fp8_f32(const uint8_t* table, int64_t table_rows, int row_bytes, float scale,
                            const wzyb_ple_fp8_hash* hash, const int32_t* ids, int64_t T, const int32_t* prev_ids,
                            int32_t eos_id, float* out, wzyb_stream_t stream);
/* gv[t,c,:] = value[t,:] * 1/(1 + exp(-s * sqrt(max(|d|, 1e-6)))), d = dot(key[t,c,:], query[t,c,:]) /
 * sqrt(n_embd), s = sign(d) (+1 at 0). key, query, gv [T, hc, n_embd]; value [T, n_embd]; fp32.
 * ple_gate_gv_multi (src/wzy_kernels_v2.cuh:1321-1346, launched at src/wzy_stage_v2.cuh:592). */
int wzyb_ple_gate_f32(const float* key, const float* query, const float* value, float* gv, int64_t T, int n_embd,
                      int hc, wzyb_stream_t stream);
/* Causal 4-tap conv of dilation 3 per channel c < hcd over x(s) = norm[s, c] (s >= 0) or
 * hist[c, 9 + s] (-9 <= s < 0):  acc = cw[c,0]*x(t-9) + cw[c,1]*x(t-6) + cw[c,2]*x(t-3) + cw[c,3]*x(t);
 * R[t,c] += gv[t,c] + acc / (1 + exp(-acc)); afterwards hist[c, i] = x(T - 9 + i). With hist_snaps
 * (or NULL), hist_snaps[t, c, 0..8] = x(t-8..t). norm, gv, R [T, hcd]; cw [hcd, 4]; hist [hcd, 9].
 * ple_conv_multi (src/wzy_kernels_v2.cuh:1348-1373, launched at src/wzy_stage_v2.cuh:594). */
int wzyb_ple_conv_f32(const float* norm, const float* cw, float* hist, const float* gv, float* R, int64_t T, int hcd,
                      float* hist_snaps, wzyb_stream_t stream);

/* Host restatement of the row index (for halos, tests and callers that stage on the host). */
uint32_t wzyb_ple_row_index(int32_t t0, int32_t t1, int32_t t2, int head, int64_t rows_per_table,
                            int32_t eos_id, int hash_variant);

/* ============================================================================================
 * Layer bundles: the ops that the reference's prefill executor launches one after another inside a
 * layer (src/wzy_prefill_tc.cuh:697 residual norm and :862-867 q/k norm+RoPE; :942 SwiGLU and :845
 * GDN gated norm) and the rows its engine stages in one host routine (stage_emb_ple_pf,
 * src/wzy_engine_v2.cu:1210-1265). A bundle up to a measured size (algorithmic bytes: 1.25 GiB for
 * attn_prep, about 37,000 tokens of the benchmark's layer; 1 GiB for act, about 18,000 tokens; 96 MiB
 * for embed_ple, about 6,000 tokens) is ONE kernel launch: the ops share no tensor, and every CTA of
 * the persistent grid runs both ops' code in turn, the larger items first (the same device code as
 * the ops' own entry points, so results are bit-identical to the separate calls). Larger bundles are
 * issued as the two ops' own launches, which measure as fast or faster once a launch's fixed costs
 * are small against its traffic. The tensors of the two ops must not overlap; if they do, or if a shape is outside the one-launch
 * kernels' range (attn_prep: fp16 hidden <= 2560 and head_dim 64/128/256; act: head_dim 64/128/256;
 * embed_ple: PLE head_dim 64/128/256), or a non-default design was chosen with
 * wzyb_set_kernel_variant, the entry point issues the ops as separate launches in the order above.
 * Arguments are validated exactly as by the per-op entry points.
 * ========================================================================================== */
typedef struct {
    /* residual add + RMSNorm, [T, hidden] */
    const uint16_t* x;
    uint16_t* residual;
    const uint16_t* norm_weight;
    uint16_t* normed;
    int hidden;
    /* q/k norm + RoPE, in place */
    wzyb_head_tensor q;
    wzyb_head_tensor k;
    int head_dim;
    int rot_dims;
    const float* cos_tab;
    const float* sin_tab;
    int64_t table_rows;
    const int32_t* d_base_pos;
    int64_t pos_offset;
    float eps;
    float w_offset; /* applied to norm_weight and the q/k gammas */
} wzyb_attn_prep_args;

typedef struct {
    /* SwiGLU over act_rows rows of ffn elements (routed + shared expert rows) */
    const uint16_t* gate;
    const uint16_t* up;
    uint16_t* act;
    int64_t act_rows;
    int ffn;
    /* GDN gated norm over T tokens of gdn_heads x gdn_head_dim */
    const uint16_t* o;
    const uint16_t* z;
    const uint16_t* gdn_gamma;
    uint16_t* gdn_out;
    int gdn_heads;
    int gdn_head_dim;
    float eps;
    float gdn_w_offset;
    int gate_mode;
} wzyb_act_args;

int wzyb_attn_prep_f16(const wzyb_attn_prep_args* a, int64_t T, wzyb_stream_t stream);
int wzyb_act_f16(const wzyb_act_args* a, int64_t T, wzyb_stream_t stream);

/* Token-embedding rows and 3-gram PLE rows of the same T ids, in one launch: what stage_emb_ple_pf
 * (src/wzy_engine_v2.cu:1210-1265) stages on the host for a prefill chunk (one stage_one_emb row and
 * 16 PLE rows per token). Fields as wzyb_embed_gather_f16 and wzyb_ple_gather_f16. */
typedef struct {
    const int32_t* ids; /* [T] device token ids, read by both gathers                           */
    /* token embedding: emb_out[t] = table[id(t)] */
    const uint16_t* table;
    int64_t vocab;
    int hidden;
    int oob_policy;
    uint32_t* d_oob_count; /* or NULL                                                           */
    uint16_t* emb_out;     /* [T, hidden]                                                       */
    /* PLE: ple_out[t, h*head_dim ...] = ple_tables[h][row_h(t)] */
    const uint16_t* const* ple_tables; /* HOST array of ple_heads device pointers               */
    int ple_heads;
    int64_t ple_rows; /* rows per table                                                         */
    int ple_head_dim;
    const int32_t* prev_ids; /* HOST {id[-2], id[-1]} or NULL                                   */
    int32_t eos_id;
    int hash_variant;
    uint16_t* ple_out; /* [T, ple_heads * ple_head_dim]                                        */
} wzyb_embed_ple_args;

int wzyb_embed_ple_f16(const wzyb_embed_ple_args* a, int64_t T, wzyb_stream_t stream);

/* Token-row sharding for G independent GPUs (no collective): rank r gets rows
 * [row0, row0 + rows) of a contiguous ceil(total/G) split. */
int wzyb_shard_rows(int64_t total, int world, int rank, int64_t* row0, int64_t* rows);
/* PLE history halo for a shard starting at row0 of host ids[]: out_prev = {id[row0-2], id[row0-1]},
 * taking ids before the sequence from seq_prev (2 ids, or NULL = none = -1). */
int wzyb_ple_halo(const int32_t* ids, int64_t row0, const int32_t* seq_prev, int32_t out_prev[2]);

/* ============================================================================================
 * Runtime helpers.
 * ========================================================================================== */
/* Launch semantics: every kernel is launched with programmatic stream serialization (programmatic
 * dependent launch) and begins by waiting for the previous grid in the stream to complete, before
 * any memory access, so stream order holds exactly as for plain launches (also when captured into
 * a CUDA graph), while the launch itself overlaps the previous kernel's tail. WZYB_PDL=0 in the
 * environment launches without the attribute.
 * One-time per-device set-up (device check, SM count, shared-memory opt-in). Launchers call it
 * lazily; call it explicitly before capturing a stream into a CUDA graph. */
int wzyb_prepare_device(void);
/* Read the current device's fault bits (synchronous); clears them when clear != 0. */
int wzyb_read_faults(uint32_t* faults, int clear);
/* Launch-shape tuning per kernel family (process-wide), for A/B measurement (ctas_per_sm 1..16,
 * stages 0..64; what they mean per family): gathers' bulk design: CTAs per SM (1..4, default 2) and
 * slots per warp (0 = as many as the shared-memory budget allows); add+RMSNorm: stages 1 turns off
 * the L2 look-ahead of the quantising norm; SwiGLU: CTAs per SM of its grid (default 4), stages 1 / 2
 * force the scalar / packed math; head
 * norm+RoPE: ctas_per_sm 2 selects the other instantiation of its design; layer bundles: stages picks the
 * schedule (0 by size as above, 1 the persistent grid split between the ops, 2 one item per warp on a
 * grid sized to the work, 3 both ops on every CTA, 4 the ops' own launches). KV append: stages
 * is the rounds of heads per warp item (0 by size, 1 or 2), ctas_per_sm caps the grid of 128-thread CTAs
 * (default 16).
 * Families: 0 add+RMSNorm, 1 head norm+RoPE, 2 GDN gated norm, 3 SwiGLU, 4 gathers, 5 layer bundles,
 * 6 KV append. */
#define WZYB_FAM_NORM 0
#define WZYB_FAM_HEAD_ROPE 1
#define WZYB_FAM_GDN 2
#define WZYB_FAM_SWIGLU 3
#define WZYB_FAM_GATHER 4
#define WZYB_FAM_BUNDLE 5
#define WZYB_FAM_KV 6
int wzyb_set_launch_tuning(int family, int ctas_per_sm, int stages);
/* Kernel design per family (process-wide), for A/B measurement:
 *   WZYB_VARIANT_AUTO   the library's choice for the shape (default)
 *   WZYB_VARIANT_RING   (gathers) TMA bulk copies global -> shared -> global, a ring of slots per warp
 *   WZYB_VARIANT_DIRECT warp-owned units, 16-byte loads prefetched into registers, no CTA barrier
 *   WZYB_VARIANT_ASYNC  warp-owned units staged in a lane-private shared-memory ring by cp.async
 *   WZYB_VARIANT_WIDE   CTA-owned rows (4-16 warps), registers, one CTA barrier per row
 *   WZYB_VARIANT_PAIR   (head norm+RoPE) two chunks per lane holding each rotation pair, no shuffle
 *   WZYB_VARIANT_SPLIT  (layer bundles) each op of a bundle as its own launch, in the reference's order
 * Families 0 (add+RMSNorm), 1 (head norm+RoPE) and 2 (GDN gated norm) have the DIRECT and ASYNC
 * designs; family 0 also WIDE, which AUTO picks for rows past one warp's register budget; family 1
 * also PAIR; family 4 (gathers) RING, for output rows up to 16 KiB; family 5 AUTO (one launch per
 * bundle) and SPLIT (a family without a design falls back to AUTO; DIRECT and ASYNC do so for rows
 * too wide). */
#define WZYB_VARIANT_AUTO 0
#define WZYB_VARIANT_RING 1
#define WZYB_VARIANT_DIRECT 2
#define WZYB_VARIANT_ASYNC 3
#define WZYB_VARIANT_WIDE 4
#define WZYB_VARIANT_PAIR 5
#define WZYB_VARIANT_SPLIT 6
int wzyb_set_kernel_variant(int family, int variant);
const char* wzyb_status_string(int status);
int wzyb_version(void);

#ifdef __cplusplus
}
#endif

#endif /* WZYB200_H */
