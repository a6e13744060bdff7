/*
 * wzyb_oracle.c -- CPU restatement of wzy-flash-serve's per-layer elementwise math.
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker and the timed CPU baseline. Nothing in the product
 * library links or loads it. Each function names the reference lines it restates.
 *
 * Build: gcc -O3 -march=x86-64-v2 -ffp-contract=off -fopenmp -shared -fPIC (oracle/Makefile).
 */
#define _POSIX_C_SOURCE 200112L /* clock_gettime under -std=c11 */
#include "wzyb_oracle.h"

#include <math.h>
#include <omp.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

/* ------------------------------------------------------------------------------------------- */
/* IEEE binary16 <-> binary32                                                                  */
/* ------------------------------------------------------------------------------------------- */
float or_h2f(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1Fu;
    const uint32_t m = h & 0x3FFu;
    uint32_t bits;
    if (e == 0x1F) {
        bits = sign | 0x7F800000u | (m << 13);
    } else if (e != 0) {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    } else if (m == 0) {
        bits = sign;
    } else { /* subnormal: m * 2^-24, exact in float */
        const float v = (float)m * 5.9604644775390625e-08f;
        float out = (sign ? -v : v);
        return out;
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* round-to-nearest-even, overflow to inf, NaN kept quiet */
uint16_t or_f2h(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
    if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* >= 65520 rounds to inf */
    if (ax < 0x38800000u) {                                  /* below 2^-14: subnormal or zero */
        float a;
        memcpy(&a, &ax, 4);
        const float s = a * 16777216.0f; /* exact: scaling by 2^24 */
        return (uint16_t)(sign | (uint16_t)rintf(s));
    }
    const uint32_t e = (ax >> 23) - 112u;
    const uint32_t mant = ax & 0x7FFFFFu;
    uint32_t h = (e << 10) | (mant >> 13);
    const uint32_t rem = mant & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1u;
    return (uint16_t)(sign | h);
}

void or_h2f_array(const uint16_t* in, float* out, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) out[i] = or_h2f(in[i]);
}

void or_f2h_array(const float* in, uint16_t* out, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) out[i] = or_f2h(in[i]);
}

void or_set_threads(int n) { omp_set_num_threads(n > 0 ? n : 1); }
int or_get_threads(void) { return omp_get_max_threads(); }

static inline float sigmoid_den(float z) { return 1.0f + expf(-z); }

/* ------------------------------------------------------------------------------------------- */
/* residual add + RMSNorm                                                                      */
/* fused_gr_norm_multi (src/wzy_kernels_v2.cuh:409-456) / pf_gr_norm_fp16                      */
/* (src/wzy_qsa_wmma.cuh:197-232): v = R + bo*gw; R <- v; xn = (v * rsqrt(sum(v^2)/n + eps)) * g */
/* with gw = 2*sigmoid(inj/hc) (:419), == 1.0 for the single-stream add.                        */
/* ------------------------------------------------------------------------------------------- */
/* one row t; v is n floats of scratch */
static void add_rmsnorm_row_f16(const uint16_t* x, uint16_t* res, const uint16_t* w, uint16_t* y, int64_t t, int n,
                                float eps, float w_offset, float* v) {
    uint16_t* r = res + t * n;
    double ss = 0.0;
    for (int d = 0; d < n; ++d) {
        float val = or_h2f(r[d]);
        if (x) val = val + or_h2f(x[t * n + d]);
        v[d] = val;
        ss += (double)val * (double)val;
    }
    const float sc = 1.0f / sqrtf((float)ss / (float)n + eps);
    for (int d = 0; d < n; ++d) {
        const float g = w_offset + or_h2f(w[d]);
        y[t * n + d] = or_f2h((v[d] * sc) * g);
        if (x) r[d] = or_f2h(v[d]);
    }
}

void or_add_rmsnorm_f16(const uint16_t* x, uint16_t* res, const uint16_t* w, uint16_t* y, int64_t T, int n,
                        float eps, float w_offset) {
#pragma omp parallel
    {
        float* v = (float*)malloc(sizeof(float) * (size_t)n);
#pragma omp for schedule(static)
        for (int64_t t = 0; t < T; ++t) add_rmsnorm_row_f16(x, res, w, y, t, n, eps, w_offset, v);
        free(v);
    }
}

/* Timing loop of the CPU baseline for the decode-step add + RMSNorm (one token): `reps` calls of the
 * scalar row code on the same buffers, on the calling thread (the residual keeps accumulating x), each
 * call's wall time in ns (CLOCK_MONOTONIC) written to samples_ns. */
void or_time_add_rmsnorm_f16(const uint16_t* x, uint16_t* res, const uint16_t* w, uint16_t* y, int64_t T, int n,
                             float eps, float w_offset, int reps, double* samples_ns) {
    float* v = (float*)malloc(sizeof(float) * (size_t)n);
    for (int i = 0; i < reps; ++i) {
        struct timespec a, b;
        clock_gettime(CLOCK_MONOTONIC, &a);
        for (int64_t t = 0; t < T; ++t) add_rmsnorm_row_f16(x, res, w, y, t, n, eps, w_offset, v);
        clock_gettime(CLOCK_MONOTONIC, &b);
        samples_ns[i] = (double)(b.tv_sec - a.tv_sec) * 1e9 + (double)(b.tv_nsec - a.tv_nsec);
    }
    free(v);
}

void or_gr_norm_f32(float* R, const float* w, const float* bo, const float* inj, float* xn, uint16_t* xn_h16,
                    int64_t T, int n, int hc, float eps) {
#pragma omp parallel for schedule(static)
    for (int64_t u = 0; u < T * hc; ++u) {
        const int64_t t = u / hc;
        const int c = (int)(u % hc);
        float* rc = R + u * n;
        const float* gc = w + (int64_t)c * n;
        const float gw = bo ? (inj ? 2.0f / (1.0f + expf(-inj[u] / (float)hc)) : 1.0f) : 0.0f;
        double ss = 0.0;
        for (int d = 0; d < n; ++d) {
            float val = rc[d];
            if (bo) {
                val = val + bo[t * n + d] * gw;
                rc[d] = val;
            }
            ss += (double)val * (double)val;
        }
        const float sc = 1.0f / sqrtf((float)ss / (float)n + eps);
        for (int d = 0; d < n; ++d) {
            const float yn = (rc[d] * sc) * gc[d];
            if (xn) xn[u * n + d] = yn;
            if (xn_h16) xn_h16[u * n + d] = or_f2h(yn);
        }
    }
}

/* Q8_0 of one 32-element group: the xq8 path of fused_gr_norm_multi (src/wzy_kernels_v2.cuh:440-454)  */
/* and silu_mul_quant32_multi (:1247-1279): d = amax/127; q = rint(v * 127/amax) in [-127, 127].     */
static void q8_group_n(const float* v, int n, int8_t* q, float* s) {
    float am = 0.f;
    for (int i = 0; i < n; ++i) am = fmaxf(am, fabsf(v[i]));
    const float d = am / 127.0f;
    const float inv = d > 0.f ? 127.0f / am : 0.f;
    for (int i = 0; i < n; ++i) {
        const float t = v[i] * inv;
        /* __float2int_rn maps NaN (a NaN or infinite input) to 0 and saturates: t = +-inf (a tiny    */
        /* nonzero amax, where 127/amax overflows) clamps to +-127                                    */
        int qi = isnan(t) ? 0 : t >= 127.f ? 127 : t <= -127.f ? -127 : (int)rintf(t);
        q[i] = (int8_t)(qi < -127 ? -127 : (qi > 127 ? 127 : qi));
    }
    *s = d;
}

static void q8_group(const float* v, int8_t* q, float* s) { q8_group_n(v, 32, q, s); }

/* quant_act_multi (src/wzy_kernels_v2.cuh:58-111): the same rule per 32 (q32) and per 16 (q16) */
void or_quant_act_f32(const float* x, int8_t* q32, float* s32, int8_t* q16, float* s16, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t g = 0; g < n / 16; ++g) {
        if (q16) q8_group_n(x + g * 16, 16, q16 + g * 16, s16 + g);
        if (q32 && (g & 1) == 0) q8_group_n(x + g * 16, 32, q32 + g * 16, s32 + g / 2);
    }
}

void or_gr_norm_q8_f32(float* R, const float* w, const float* bo, const float* inj, float* xn, int8_t* q8,
                       float* s8, int64_t T, int n, int hc, float eps) {
    or_gr_norm_f32(R, w, bo, inj, xn, NULL, T, n, hc, eps);
#pragma omp parallel for schedule(static)
    for (int64_t g = 0; g < T * hc * (int64_t)n / 32; ++g) q8_group(xn + g * 32, q8 + g * 32, s8 + g);
}

void or_swiglu_q8_f32(const float* g, const float* u, int8_t* q, float* s, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t grp = 0; grp < n / 32; ++grp) {
        float v[32];
        for (int i = 0; i < 32; ++i) v[i] = (g[grp * 32 + i] / sigmoid_den(g[grp * 32 + i])) * u[grp * 32 + i];
        q8_group(v, q + grp * 32, s + grp);
    }
}

/* ------------------------------------------------------------------------------------------- */
/* multi-stream residual outside the norm                                                      */
/* gr_write_multi (src/wzy_kernels_v2.cuh:813-828): R[t,c,:] += blk[t,:] * 2/(1+exp(-inj/hc))  */
/* ------------------------------------------------------------------------------------------- */
void or_gr_write_f32(float* R, const float* blk, const float* inj, int64_t T, int n, int hc) {
#pragma omp parallel for schedule(static)
    for (int64_t u = 0; u < T * hc; ++u) {
        const float gw = inj ? 2.0f / sigmoid_den(inj[u] / (float)hc) : 1.0f;
        const float* b = blk + (u / hc) * n;
        float* r = R + u * n;
        for (int d = 0; d < n; ++d) r[d] = r[d] + b[d] * gw;
    }
}

/* pf_gr_up_mean_fp16 (src/wzy_qsa_wmma.cuh:234-253) / gr_up_gate_mean_pf_kernel                */
/* (src/wzy_prefill_tc.cuh:37-51): mixed[t,d] = (sum_c xn[t,c,d] / (1 + exp(-gg[t,c,d]))) / hc,  */
/* streams summed in order c = 0..hc-1; the reference's 4 streams scale by 0.25.                 */
static void hc_mix_row(const float* x, const float* g, int64_t n, int hc, int64_t d, float* out) {
    float acc = 0.f;
    for (int c = 0; c < hc; ++c) acc += x[c * n + d] / sigmoid_den(g[c * n + d]);
    *out = acc * (1.0f / (float)hc);
}

void or_hc_mix_f16(const uint16_t* xn, const uint16_t* gg, float* mixed, uint16_t* mixed_h16, int64_t T, int n,
                   int hc) {
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < T; ++t) {
        float* x = (float*)malloc(sizeof(float) * 2 * (size_t)hc * n);
        float* g = x + (size_t)hc * n;
        or_h2f_array(xn + t * hc * n, x, (int64_t)hc * n);
        or_h2f_array(gg + t * hc * n, g, (int64_t)hc * n);
        for (int64_t d = 0; d < n; ++d) {
            float m;
            hc_mix_row(x, g, n, hc, d, &m);
            if (mixed) mixed[t * n + d] = m;
            if (mixed_h16) mixed_h16[t * n + d] = or_f2h(m);
        }
        free(x);
    }
}

void or_hc_mix_f32(const float* xn, const float* gg, float* mixed, int64_t T, int n, int hc) {
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < T; ++t)
        for (int64_t d = 0; d < n; ++d) hc_mix_row(xn + t * hc * n, gg + t * hc * n, n, hc, d, mixed + t * n + d);
}

/* silu_div_hc_to_fp16_kernel (src/wzy_prefill_tc.cuh:24-35): v = lo * scale; out = fp16(v / (1 + exp(-v))) */
void or_silu_scale_f16(const float* lo, uint16_t* out, int64_t n, float scale) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        const float v = lo[i] * scale;
        out[i] = or_f2h(v / sigmoid_den(v));
    }
}

/* ------------------------------------------------------------------------------------------- */
/* per-head RMSNorm + partial NeoX RoPE: fused_head_norm_rope_multi (src/wzy_qsa_256k.cuh:50-84) */
/*   p *= rsqrt(sum(p^2)/hd + eps) * gamma;  (a, d) = (p[i], p[i+R/2])                          */
/*   p[i] = a*cos - d*sin;  p[i+R/2] = a*sin + d*cos, cos/sin = tab[pos*(R/2) + i]              */
/* A position outside the table leaves the head un-rotated (the CUDA path flags it).            */
/* ------------------------------------------------------------------------------------------- */
static void head_norm_rope_row(float* p, const float* g, const float* cos_tab, const float* sin_tab,
                               int64_t table_rows, int64_t pos, int hd, int rot, float eps) {
    double ss = 0.0;
    for (int i = 0; i < hd; ++i) ss += (double)p[i] * (double)p[i];
    const float sc = 1.0f / sqrtf((float)ss / (float)hd + eps);
    for (int i = 0; i < hd; ++i) p[i] *= sc * g[i];
    const int half = rot / 2;
    if (half == 0 || pos < 0 || pos >= table_rows) return;
    for (int i = 0; i < half; ++i) {
        const float cs = cos_tab[pos * half + i], sn = sin_tab[pos * half + i];
        const float a = p[i], d = p[i + half];
        p[i] = a * cs - d * sn;
        p[i + half] = a * sn + d * cs;
    }
}

void or_head_norm_rope_f16(uint16_t* data, const uint16_t* gamma, const float* cos_tab, const float* sin_tab,
                           int64_t table_rows, int64_t base_pos, int64_t T, int heads, int hd, int64_t head_stride,
                           int64_t row_stride, int rot, float eps, float w_offset) {
    float g[1024];
    for (int i = 0; i < hd; ++i) g[i] = w_offset + or_h2f(gamma[i]);
#pragma omp parallel for schedule(static)
    for (int64_t th = 0; th < T * heads; ++th) {
        const int64_t t = th / heads;
        const int h = (int)(th % heads);
        uint16_t* p = data + t * row_stride + (int64_t)h * head_stride;
        float buf[1024];
        for (int i = 0; i < hd; ++i) buf[i] = or_h2f(p[i]);
        head_norm_rope_row(buf, g, cos_tab, sin_tab, table_rows, base_pos + t, hd, rot, eps);
        for (int i = 0; i < hd; ++i) p[i] = or_f2h(buf[i]);
    }
}

void or_head_norm_rope_f32(float* data, const float* gamma, const float* cos_tab, const float* sin_tab,
                           int64_t table_rows, int64_t base_pos, int64_t T, int heads, int hd, int64_t head_stride,
                           int64_t row_stride, int rot, float eps, float w_offset) {
    float g[1024];
    for (int i = 0; i < hd; ++i) g[i] = w_offset + gamma[i];
#pragma omp parallel for schedule(static)
    for (int64_t th = 0; th < T * heads; ++th) {
        const int64_t t = th / heads;
        const int h = (int)(th % heads);
        head_norm_rope_row(data + t * row_stride + (int64_t)h * head_stride, g, cos_tab, sin_tab, table_rows,
                           base_pos + t, hd, rot, eps);
    }
}

/* ------------------------------------------------------------------------------------------- */
/* INT8 KV append: kv_append_int8_multi (src/wzy_qsa_256k.cuh:86-145), cells per kv_is_in_vram /  */
/* kv_vram_slot (:17-29) with the mirror pointer the reference passes as non-NULL. Per 64 group:  */
/* sh = fp16(max|x|/127), d = float(sh), q = d > 0 ? rint(x/d) : 0 clamped to [-127, 127].        */
/* ------------------------------------------------------------------------------------------- */
static int kv_in_ring(int64_t p, int64_t end, int64_t cap) {
    if (cap <= 2 * 4096) return p >= (end - cap > 0 ? end - cap : 0);
    if (p < 4096) return 1;
    const int64_t lo = end - (cap - 4096);
    return p >= (lo > 4096 ? lo : 4096);
}

static int64_t kv_ring_cell(int64_t p, int64_t cap) {
    if (cap <= 2 * 4096) return p % cap;
    if (p < 4096) return p;
    return 4096 + (p - 4096) % (cap - 4096);
}

static void kv_q8_group(const float* x, int8_t* q, uint16_t* s) {
    float am = 0.f;
    for (int i = 0; i < 64; ++i) am = fmaxf(am, fabsf(x[i]));
    const uint16_t sh = or_f2h(am / 127.0f);
    const float d = or_h2f(sh);
    for (int i = 0; i < 64; ++i) {
        /* __float2int_rn (src/wzy_qsa_256k.cuh:121) maps NaN (a NaN input, or inf / inf) to 0 */
        const float t = d > 0.f ? x[i] / d : 0.f;
        long qi = isnan(t) ? 0 : lrintf(t);
        q[i] = (int8_t)(qi < -127 ? -127 : qi > 127 ? 127 : qi);
    }
    *s = sh;
}

/* one token's fp32 k and v rows [kvd] into its cells */
static void kv_append_token(const float* k, const float* v, int kvd, int64_t pos, int64_t end, int8_t* rkq,
                            uint16_t* rks, int8_t* rvq, uint16_t* rvs, int8_t* fkq, uint16_t* fks, int8_t* fvq,
                            uint16_t* fvs, int64_t ring_cap, int64_t max_ctx) {
    if (pos < 0 || pos >= max_ctx) return;
    const int spc = kvd / 64;
    for (int g = 0; g < spc; ++g) {
        int8_t qk[64], qv[64];
        uint16_t sk, sv;
        kv_q8_group(k + g * 64, qk, &sk);
        kv_q8_group(v + g * 64, qv, &sv);
        if (kv_in_ring(pos, end, ring_cap)) {
            const int64_t c = kv_ring_cell(pos, ring_cap);
            memcpy(rkq + c * kvd + g * 64, qk, 64);
            memcpy(rvq + c * kvd + g * 64, qv, 64);
            rks[c * spc + g] = sk;
            rvs[c * spc + g] = sv;
        }
        if (fkq) {
            memcpy(fkq + pos * kvd + g * 64, qk, 64);
            memcpy(fvq + pos * kvd + g * 64, qv, 64);
            fks[pos * spc + g] = sk;
            fvs[pos * spc + g] = sv;
        }
    }
}

/* Tokens are visited in order, so a ring cell shared by two tokens keeps the later one (the      */
/* in-window rule makes that impossible within one call).                                        */
void or_kv_append_int8_f32(const float* k, const float* v, int64_t T, int kvd, int64_t base_pos, int8_t* rkq,
                           uint16_t* rks, int8_t* rvq, uint16_t* rvs, int8_t* fkq, uint16_t* fks, int8_t* fvq,
                           uint16_t* fvs, int64_t ring_cap, int64_t max_ctx) {
    for (int64_t t = 0; t < T; ++t)
        kv_append_token(k + t * kvd, v + t * kvd, kvd, base_pos + t, base_pos + T, rkq, rks, rvq, rvs, fkq, fks, fvq,
                        fvs, ring_cap, max_ctx);
}

/* fp16 k and v: k normalised and rotated in fp32 (as or_head_norm_rope_f16), quantised from those  */
/* fp32 values, and written back rounded to fp16; v widened exactly.                              */
void or_k_rope_kv_append_f16(uint16_t* k, const uint16_t* gamma, const uint16_t* v, const float* cos_tab,
                             const float* sin_tab, int64_t table_rows, int64_t base_pos, int64_t T, int kv_heads, int hd,
                             int rot, float eps, float w_offset, int8_t* rkq, uint16_t* rks, int8_t* rvq, uint16_t* rvs,
                             int8_t* fkq, uint16_t* fks, int8_t* fvq, uint16_t* fvs, int64_t ring_cap, int64_t max_ctx) {
    const int kvd = kv_heads * hd;
    float g[1024];
    for (int i = 0; i < hd; ++i) g[i] = w_offset + or_h2f(gamma[i]);
    float* kb = (float*)malloc(sizeof(float) * 2 * (size_t)kvd);
    float* vb = kb + kvd;
    for (int64_t t = 0; t < T; ++t) {
        or_h2f_array(k + t * kvd, kb, kvd);
        or_h2f_array(v + t * kvd, vb, kvd);
        for (int h = 0; h < kv_heads; ++h)
            head_norm_rope_row(kb + h * hd, g, cos_tab, sin_tab, table_rows, base_pos + t, hd, rot, eps);
        for (int i = 0; i < kvd; ++i) k[t * kvd + i] = or_f2h(kb[i]);
        kv_append_token(kb, vb, kvd, base_pos + t, base_pos + T, rkq, rks, rvq, rvs, fkq, fks, fvq, fvs, ring_cap,
                        max_ctx);
    }
    free(kb);
}

/* build_rope_cos_sin_host (src/wzy_qsa_256k.cuh:33-46): inv_i = theta^(-2i/R) in fp64,        */
/* angle = p * inv_i in fp64, cos/sin in fp64 rounded to fp32; layout [p][R/2].                 */
void or_rope_table(float* cos_tab, float* sin_tab, int64_t rows, int rot, double theta) {
    const int half = rot / 2;
    double inv[512];
    for (int i = 0; i < half; ++i) inv[i] = pow(theta, -2.0 * (double)i / (double)rot);
#pragma omp parallel for schedule(static)
    for (int64_t p = 0; p < rows; ++p) {
        for (int i = 0; i < half; ++i) {
            const double ang = (double)p * inv[i];
            cos_tab[p * half + i] = (float)cos(ang);
            sin_tab[p * half + i] = (float)sin(ang);
        }
    }
}

/* ------------------------------------------------------------------------------------------- */
/* GDN gated RMSNorm: pf_gdn_rmsnorm_gate_parallel (src/wzy_qsa_wmma.cuh:178-195)               */
/*   y = o * rsqrt(sum(o^2) * (1/hd) + eps) * gamma[col] / (1 + exp(-z))                        */
/* ------------------------------------------------------------------------------------------- */
static inline float gdn_out(float o, float sc, float g, float z, int gate_mode) {
    const float den = sigmoid_den(z);
    return gate_mode == 1 ? (o * sc * g) * (z / den) : o * sc * g / den;
}

void or_gdn_gated_norm_f16(const uint16_t* o, const uint16_t* z, const uint16_t* gamma, uint16_t* y, int64_t T,
                           int heads, int hd, float eps, float w_offset, int gate_mode) {
    float g[1024];
    for (int i = 0; i < hd; ++i) g[i] = w_offset + or_h2f(gamma[i]);
#pragma omp parallel for schedule(static)
    for (int64_t th = 0; th < T * heads; ++th) {
        const int64_t base = th * hd;
        double ss = 0.0;
        for (int i = 0; i < hd; ++i) {
            const double v = (double)or_h2f(o[base + i]);
            ss += v * v;
        }
        const float sc = 1.0f / sqrtf((float)ss * (1.0f / (float)hd) + eps);
        for (int i = 0; i < hd; ++i)
            y[base + i] = or_f2h(gdn_out(or_h2f(o[base + i]), sc, g[i], or_h2f(z[base + i]), gate_mode));
    }
}

void or_gdn_gated_norm_f32(const float* o, const float* z, const float* gamma, float* y, int64_t T, int heads, int hd,
                           float eps, float w_offset, int gate_mode) {
#pragma omp parallel for schedule(static)
    for (int64_t th = 0; th < T * heads; ++th) {
        const int64_t base = th * hd;
        double ss = 0.0;
        for (int i = 0; i < hd; ++i) ss += (double)o[base + i] * (double)o[base + i];
        const float sc = 1.0f / sqrtf((float)ss * (1.0f / (float)hd) + eps);
        for (int i = 0; i < hd; ++i)
            y[base + i] = gdn_out(o[base + i], sc, w_offset + gamma[i], z[base + i], gate_mode);
    }
}

/* ------------------------------------------------------------------------------------------- */
/* SwiGLU: silu_mul_multi (src/wzy_kernels_v2.cuh:1240-1244) (g / (1 + exp(-g))) * u;           */
/* interleaved rows [gate | up]: pf_silu_mul_interleaved_to_fp16 (src/wzy_prefill_tc.cuh:69-80)  */
/* ------------------------------------------------------------------------------------------- */
static inline float swiglu1(float g, float u) { return (g / sigmoid_den(g)) * u; }

void or_swiglu_f16(const uint16_t* g, const uint16_t* u, uint16_t* out, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) out[i] = or_f2h(swiglu1(or_h2f(g[i]), or_h2f(u[i])));
}

void or_swiglu_f32(const float* g, const float* u, float* out, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) out[i] = swiglu1(g[i], u[i]);
}

void or_swiglu_interleaved_f16(const uint16_t* gu, uint16_t* out, int64_t T, int nff) {
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < T; ++t)
        for (int c = 0; c < nff; ++c)
            out[t * nff + c] = or_f2h(swiglu1(or_h2f(gu[t * 2 * nff + c]), or_h2f(gu[t * 2 * nff + nff + c])));
}

void or_swiglu_interleaved_f32(const float* gu, float* out, int64_t T, int nff) {
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < T; ++t)
        for (int c = 0; c < nff; ++c) out[t * nff + c] = swiglu1(gu[t * 2 * nff + c], gu[t * 2 * nff + nff + c]);
}

/* ------------------------------------------------------------------------------------------- */
/* token-embedding gather: out-of-range id -> 0 as stage_one_emb (src/wzy_engine_v2.cu:863) or  */
/* clamped as mtp_gather_bf16_emb (src/wzy_kernels_v2.cuh:30)                                   */
/* ------------------------------------------------------------------------------------------- */
static inline int64_t resolve_id(int32_t id, int64_t vocab, int policy) {
    if (id >= 0 && id < vocab) return id;
    if (policy == 1) return 0;
    return id < 0 ? 0 : vocab - 1;
}

uint32_t or_embed_gather_rows(const void* table, int64_t vocab, int64_t row_bytes, const int32_t* ids, int64_t T,
                              void* out, int oob_policy) {
    uint32_t bad = 0;
#pragma omp parallel for schedule(static) reduction(+ : bad)
    for (int64_t t = 0; t < T; ++t) {
        if (!(ids[t] >= 0 && ids[t] < vocab)) ++bad;
        const int64_t id = resolve_id(ids[t], vocab, oob_policy);
        memcpy((char*)out + t * row_bytes, (const char*)table + id * row_bytes, (size_t)row_bytes);
    }
    return bad;
}

/* bf16 -> fp32 by placing the 16 bits in the high half: db2f (src/wzy_kernels_v2.cuh:23) */
uint32_t or_embed_gather_bf16_f32(const uint16_t* table, int64_t vocab, int hidden, const int32_t* ids, int64_t T,
                                  float* out, int oob_policy) {
    uint32_t bad = 0;
#pragma omp parallel for schedule(static) reduction(+ : bad)
    for (int64_t t = 0; t < T; ++t) {
        if (!(ids[t] >= 0 && ids[t] < vocab)) ++bad;
        const int64_t id = resolve_id(ids[t], vocab, oob_policy);
        for (int d = 0; d < hidden; ++d) {
            const uint32_t bits = (uint32_t)table[id * hidden + d] << 16;
            memcpy(&out[t * hidden + d], &bits, 4);
        }
    }
    return bad;
}

/* ------------------------------------------------------------------------------------------- */
/* 3-gram PLE row index. History cut as stage_ple_window builds ctx[1..2]                        */
/* (src/wzy_engine_v2.cu:946-953): an id < 0 or == EOS cuts, and it and all older ids become EOS. */
/* Mix: a = t0*0x9E3779B1, b = t1*0x85EBCA77, c = t2*0xC2B2AE3D (uint32),                         */
/* row = (a ^ b ^ (c + head)) mod rows [variant 0] or ((a ^ b ^ c) + head) mod rows [variant 1]. */
/* ------------------------------------------------------------------------------------------- */
uint32_t or_ple_row(int32_t t0, int32_t t1, int32_t t2, int head, int64_t rows, int32_t eos, int variant) {
    int32_t ctx1, ctx2;
    int cut = (t1 < 0 || t1 == eos);
    ctx1 = cut ? eos : t1;
    cut = cut || (t2 < 0 || t2 == eos);
    ctx2 = cut ? eos : t2;
    const uint32_t a = (uint32_t)t0 * 0x9E3779B1u;
    const uint32_t b = (uint32_t)ctx1 * 0x85EBCA77u;
    const uint32_t c = (uint32_t)ctx2 * 0xC2B2AE3Du;
    const uint32_t h = variant == 1 ? ((a ^ b ^ c) + (uint32_t)head) : (a ^ b ^ (c + (uint32_t)head));
    return (uint32_t)((uint64_t)h % (uint64_t)rows);
}

void or_ple_gather_f16(const uint16_t* const* tables, int heads, int64_t rows, int hd, const int32_t* ids, int64_t T,
                       const int32_t* prev_ids, int32_t eos, int variant, uint16_t* out) {
    const int32_t prev2 = prev_ids ? prev_ids[0] : -1;
    const int32_t prev1 = prev_ids ? prev_ids[1] : -1;
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < T; ++t) {
        const int32_t t1 = t >= 1 ? ids[t - 1] : prev1;
        const int32_t t2 = t >= 2 ? ids[t - 2] : (t == 1 ? prev1 : prev2);
        for (int h = 0; h < heads; ++h) {
            const uint32_t r = or_ple_row(ids[t], t1, t2, h, rows, eos, variant);
            memcpy(out + (t * heads + h) * (int64_t)hd, tables[h] + (int64_t)r * hd, sizeof(uint16_t) * (size_t)hd);
        }
    }
}

/* ------------------------------------------------------------------------------------------- */
/* PLE in the reference model's own format                                                     */
/* stage_ple_window (src/wzy_engine_v2.cu:943-978): context [cur, prev1, prev2] with the EOS cut; */
/* for n in {2, 3}: mixed = xor_j ctx[j] * mult[j] (u64); 8 heads per n:                        */
/* row = (uint32)(mixed % vocab[h] + off[h]). PleSrc (src/wzy_stage_v2.cuh:278-285): e4m3 byte   */
/* decoded by a 256-entry table (subnormal mm*2^-9, NaN codes -> 0) times the global scale.      */
/* ------------------------------------------------------------------------------------------- */
uint32_t or_ple_fp8_row(int32_t cur, int32_t p1, int32_t p0, int h, const uint64_t* mult, const uint64_t* vocab,
                        const uint64_t* off, int32_t eos) {
    const int32_t t3[3] = {p0, p1, cur};
    int64_t ctx[3];
    ctx[0] = cur;
    int cut = 0;
    for (int s = 1; s < 3; ++s) {
        const int32_t v = cut ? -1 : t3[2 - s];
        cut = cut || v < 0 || v == eos;
        ctx[s] = cut ? eos : v;
    }
    const int n = h < 8 ? 2 : 3;
    uint64_t mixed = (uint64_t)ctx[0] * mult[0];
    for (int j = 1; j < n; ++j) mixed ^= (uint64_t)ctx[j] * mult[j];
    return (uint32_t)(mixed % vocab[h] + off[h]);
}

void or_ple_gather_fp8_f32(const uint8_t* table, int row_bytes, float scale, const uint64_t* mult,
                           const uint64_t* vocab, const uint64_t* off, const int32_t* ids, int64_t T,
                           const int32_t* prev_ids, int32_t eos, float* out) {
    float lut[256];
    for (int v = 0; v < 256; ++v) {
        const int sg = (v >> 7) & 1, e = (v >> 3) & 0xF, mm = v & 7;
        float f;
        if (e == 0) f = ldexpf((float)mm, -9);
        else if (e == 15 && mm == 7) f = 0.f;
        else f = ldexpf(1.f + (float)mm / 8.f, e - 7);
        lut[v] = (sg ? -f : f) * scale;
    }
    const int32_t prev2 = prev_ids ? prev_ids[0] : -1;
    const int32_t prev1 = prev_ids ? prev_ids[1] : -1;
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < T; ++t) {
        const int32_t p1 = t >= 1 ? ids[t - 1] : prev1;
        const int32_t p0 = t >= 2 ? ids[t - 2] : (t == 1 ? prev1 : prev2);
        for (int h = 0; h < 16; ++h) {
            const uint32_t r = or_ple_fp8_row(ids[t], p1, p0, h, mult, vocab, off, eos);
            const uint8_t* src = table + (uint64_t)r * (uint64_t)row_bytes;
            float* dst = out + (t * 16 + h) * (int64_t)row_bytes;
            for (int i = 0; i < row_bytes; ++i) dst[i] = lut[src[i]];
        }
    }
}

/* ple_gate_gv_multi (src/wzy_kernels_v2.cuh:1321-1346): d = dot(key, query) / sqrt(n) (double sum); */
/* g = 1/(1 + exp(-sign(d) * sqrt(max(|d|, 1e-6)))); gv = value[t] * g.                           */
void or_ple_gate_f32(const float* key, const float* query, const float* value, float* gv, int64_t T, int n, int hc) {
#pragma omp parallel for schedule(static)
    for (int64_t u = 0; u < T * hc; ++u) {
        const float* k = key + u * n;
        const float* q = query + u * n;
        const float* v = value + (u / hc) * n;
        double acc = 0.0;
        for (int d = 0; d < n; ++d) acc += (double)k[d] * (double)q[d];
        float tot = (float)acc / sqrtf((float)n);
        const float sg = tot < 0.f ? -1.f : 1.f;
        const float g = 1.f / (1.f + expf(-sg * sqrtf(fmaxf(fabsf(tot), 1e-6f))));
        for (int d = 0; d < n; ++d) gv[u * n + d] = v[d] * g;
    }
}

/* ple_conv_multi (src/wzy_kernels_v2.cuh:1348-1373), sequential over T per channel as there:      */
/* h = hist[c, 0..8]; acc = w0*h0 + w1*h3 + w2*h6 + w3*cur; shift in cur; R += gv + silu(acc).      */
void or_ple_conv_f32(const float* norm, const float* cw, float* hist, const float* gv, float* R, int64_t T, int hcd,
                     float* snaps) {
#pragma omp parallel for schedule(static)
    for (int c = 0; c < hcd; ++c) {
        float h[9];
        for (int i = 0; i < 9; ++i) h[i] = hist[(int64_t)9 * c + i];
        const float w0 = cw[4 * c], w1 = cw[4 * c + 1], w2 = cw[4 * c + 2], w3 = cw[4 * c + 3];
        for (int64_t t = 0; t < T; ++t) {
            const float cur = norm[t * hcd + c];
            const float acc = w0 * h[0] + w1 * h[3] + w2 * h[6] + w3 * cur;
            for (int i = 0; i < 8; ++i) h[i] = h[i + 1];
            h[8] = cur;
            R[t * hcd + c] += gv[t * hcd + c] + acc / (1.0f + expf(-acc));
            if (snaps)
                for (int i = 0; i < 9; ++i) snaps[(t * hcd + c) * 9 + i] = h[i];
        }
        for (int i = 0; i < 9; ++i) hist[(int64_t)9 * c + i] = h[i];
    }
}

/* ------------------------------------------------------------------------------------------- */
/* Block-scaled GEMM-input formats (no reference counterpart: the B200 form of the int8 epilogue) */
/* e4m3 = OCP FP8 E4M3 (bias 7, max 448, NaN 0x7F), e2m1 = FP4 E2M1 {0, .5, 1, 1.5, 2, 3, 4, 6};   */
/* both round-to-nearest-even and saturate finite overflow to the largest magnitude.             */
/* ------------------------------------------------------------------------------------------- */
uint8_t or_f2e4m3(float f) {
    const uint8_t sign = signbit(f) ? 0x80 : 0x00;
    if (isnan(f)) return 0x7F;
    const float a = fabsf(f);
    if (a >= 448.0f) return (uint8_t)(sign | 0x7E);
    if (a < 0.015625f) /* below 2^-6: subnormal steps of 2^-9 (q == 8 is the first normal) */
        return (uint8_t)(sign | (uint8_t)rintf(a * 512.0f));
    int e;
    frexpf(a, &e); /* a in [2^(e-1), 2^e) */
    const int E = e - 1;
    const float q = rintf(ldexpf(a, 3 - E)); /* 8..16 steps of 2^(E-3); 16 carries into the next binade */
    return (uint8_t)(sign | (uint8_t)(((E + 7) << 3) + (int)q - 8));
}

float or_e4m32f(uint8_t b) {
    const int sg = (b >> 7) & 1, e = (b >> 3) & 0xF, m = b & 7;
    float f;
    if (e == 15 && m == 7) return NAN;
    if (e == 0) f = ldexpf((float)m, -9);
    else f = ldexpf(1.f + (float)m / 8.f, e - 7);
    return sg ? -f : f;
}

uint8_t or_f2e2m1(float f) {
    const uint8_t sign = signbit(f) ? 0x8 : 0x0;
    const float a = fabsf(f);
    if (isnan(f)) return 0x7; /* the hardware's choice: positive largest */
    if (a >= 6.0f) return (uint8_t)(sign | 0x7);
    if (a < 2.0f) return (uint8_t)(sign | (uint8_t)rintf(a * 2.0f));     /* 0, .5, 1, 1.5, (2) */
    if (a < 4.0f) return (uint8_t)(sign | (uint8_t)(rintf(a) + 2.0f));  /* 2, 3, (4) */
    return (uint8_t)(sign | (uint8_t)(rintf(a * 0.5f) + 4.0f));        /* 4, 6 */
}

/* MXFP8: per 32, scale X = 2^ceil(log2(amax / 448)) (the smallest power of two keeping the block   */
/* within +-448) as the E8M0 byte log2(X) + 127; codes e4m3(x / X). amax == 0 -> byte 0; inf/NaN -> 0xFF */
static uint32_t mxfp8_scale_byte(float amax) {
    const float t = amax / 448.0f;
    uint32_t tb;
    memcpy(&tb, &t, 4);
    const uint32_t et = tb >> 23;
    if (et == 0xFFu) return 0xFFu;
    if (et == 0u) return tb <= 0x00400000u ? 0u : 1u;
    return et + ((tb & 0x7FFFFFu) != 0u ? 1u : 0u);
}

void or_quant_mxfp8(const float* x, uint8_t* q, uint8_t* s, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t g = 0; g < n / 32; ++g) {
        float am = 0.f;
        for (int i = 0; i < 32; ++i) am = fmaxf(am, fabsf(x[g * 32 + i]));
        const uint32_t e8 = mxfp8_scale_byte(am);
        float inv = 0.f;
        if (e8 != 0xFFu) {
            const uint32_t ib = (254u - e8) << 23;
            memcpy(&inv, &ib, 4);
        }
        for (int i = 0; i < 32; ++i) q[g * 32 + i] = or_f2e4m3(x[g * 32 + i] * inv);
        s[g] = (uint8_t)e8;
    }
}

/* NVFP4: per 16, scale byte e4m3((amax * gs) / 6), codes e2m1(x * (gs / float(scale))) */
void or_quant_nvfp4(const float* x, uint8_t* q, uint8_t* s, float gs, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t g = 0; g < n / 16; ++g) {
        float am = 0.f;
        for (int i = 0; i < 16; ++i) am = fmaxf(am, fabsf(x[g * 16 + i]));
        const uint8_t sc = or_f2e4m3((am * gs) / 6.0f);
        const float sf = or_e4m32f(sc);
        const float r = sf > 0.f ? gs / sf : 0.f;
        for (int i = 0; i < 8; ++i) {
            const uint8_t lo = or_f2e2m1(x[g * 16 + 2 * i] * r), hi = or_f2e2m1(x[g * 16 + 2 * i + 1] * r);
            q[g * 8 + i] = (uint8_t)(lo | (hi << 4));
        }
        s[g] = sc;
    }
}
