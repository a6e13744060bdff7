// kv_append.cu -- k per-head RMSNorm + partial NeoX RoPE fused with the INT8 KV-cache append.
//
// The reference appends in three launches per layer: fused_head_norm_rope_multi on k
// (src/wzy_stage_v2.cuh:640-641, src/wzy_prefill_tc.cuh:864-865), then kv_append_int8_multi
// (src/wzy_qsa_256k.cuh:86-145, launched at src/wzy_stage_v2.cuh:655 and src/wzy_prefill_tc.cuh:878),
// which re-reads k and v, one 64-thread block per (64-element group, token). Here one warp owns a
// (token, round of heads): it loads those k and v heads once, normalises and rotates k (written back
// in place), and quantises both into the cache:
//   per 64-element group  sh = fp16(max|x| / 127),  d = float(sh),  q = d > 0 ? rint(x / d) : 0,
//   q clamped to [-127, 127]; codes [cell, kvd] int8, scales [cell, kvd/64] fp16.
// A 64-element group is 8 consecutive lanes (8 elements each); its max is three xor shuffles.
// Cells (restating kv_is_in_vram / kv_vram_slot, src/wzy_qsa_256k.cuh:17-29, with the mirror pointer
// the reference always passes as non-NULL):
//   pos = base_pos + pos_offset + t; tokens with pos outside [0, max_ctx) are not appended;
//   ring (device) cell: ring_cap <= 2*4096: pos % ring_cap, written when pos >= end - ring_cap;
//                       else pos < 4096 (pinned sink): pos, always written;
//                            else 4096 + (pos - 4096) % (ring_cap - 4096), written when
//                            pos >= max(4096, end - (ring_cap - 4096));
//   end = base_pos + pos_offset + T (one past this call's last position), so a call never writes two
//   of its own tokens into one ring cell; full-context mirror cell: pos (when the mirror is given).
#include "launch.hpp"
#include "common.cuh"

namespace wzyb {

constexpr int kKvSinkPin = 4096;
constexpr int kKvGroup = 64;

struct KvAppendArgs {
    void* k;              // [T, kv_heads * HD] (normed + rotated in place when norm_rope)
    const void* k_gamma;  // [HD]
    const void* v;        // [T, kv_heads * HD]
    const float* cos_tab;
    const float* sin_tab;
    int64_t table_rows;
    const int32_t* d_base_pos;
    int64_t pos_offset;
    int64_t T;
    int kv_heads;
    int rot;
    float eps;
    float w_offset;
    int norm_rope;
    wzyb_kv_cache c;
    uint64_t ring_div;    // divisor of the ring cell: ring_cap, or ring_cap - 4096 past the pinned sink
    uint64_t ring_recip;  // floor((2^64 - 1) / ring_div), for mod_u64
    // optional q heads, normed and rotated in place in the same launch (q_heads == 0: none)
    void* q;
    const void* q_gamma;
    int q_heads;
    int64_t q_head_stride;  // elements between heads of a token
    int64_t q_row_stride;   // elements between tokens
};

__device__ __forceinline__ bool kv_in_ring(int64_t p, int64_t end, int64_t cap) {
    if (cap <= 2 * kKvSinkPin) return p >= (end - cap > 0 ? end - cap : 0);
    if (p < kKvSinkPin) return true;
    const int64_t lo = end - (cap - kKvSinkPin);
    return p >= (lo > kKvSinkPin ? lo : kKvSinkPin);
}

// p >= 0; div and recip as KvAppendArgs::ring_div / ring_recip
__device__ __forceinline__ int64_t kv_ring_cell(int64_t p, int64_t cap, uint64_t div, uint64_t recip) {
    if (cap <= 2 * kKvSinkPin) return (int64_t)mod_u64((uint64_t)p, div, recip);
    if (p < kKvSinkPin) return p;
    return kKvSinkPin + (int64_t)mod_u64((uint64_t)(p - kKvSinkPin), div, recip);
}

// This lane's max |x| (NaNs dropped, as the reference's fmaxf) and its max with NaNs kept.
__device__ __forceinline__ void kv_lane_max(const float2 (&x)[4], float& am, float& an) {
    am = 0.f;
    an = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float a = fabsf(x[i].x), b = fabsf(x[i].y);
        am = fmaxf(am, fmaxf(a, b));
        an = fmax_nan(an, fmax_nan(a, b));
    }
}

// The group maxima (lanes 8m..8m+7) of N vectors, their shuffles interleaved.
template <int N>
__device__ __forceinline__ void kv_group_max(float (&am)[N]) {
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
        float t[N];
#pragma unroll
        for (int m = 0; m < N; ++m) t[m] = __shfl_xor_sync(0xffffffffu, am[m], o);
#pragma unroll
        for (int m = 0; m < N; ++m) am[m] = fmaxf(am[m], t[m]);
    }
}

// A group's fp16 scale fp16(RN(am / 127)) for am >= 0, with the quotient by Markstein's sequence
// instead of a divide: r = RN(1/127) (0x3C010204), q0 = RN(am * r), e = am - q0 * 127 (exact under
// FMA), RN(q0 + e * r) is the correctly rounded quotient wherever it is a normal fp32. Quotients below
// 2^-126 give a zero fp16 scale either way, and am = inf keeps inf. Branch-free.
__device__ __forceinline__ __half kv_group_scale(float am) {
    const float r = __int_as_float(0x3C010204);
    const float q0 = __fmul_rn(am, r);
    const float q = fmaf(fmaf(-q0, 127.0f, am), r, q0);
    return __float2half_rn(am <= 3.402823466e38f ? q : am);
}

// RN(1/d) for a scale d = 0 (gives 0) or a finite fp16 scale (a normal fp32 in [2^-24, 65504]), by one
// Newton-Raphson step from the approximate reciprocal: y0 = rcp.approx(d) (within 1 ulp), then
// RN(y0 + y0 * (1 - d * y0)). The residual 1 - d*y0 needs at most 12 significant bits (d has 11), so
// the FMA computes it exactly, and the step leaves a relative error below 2^-44. 1/d = 2^-k / M for an
// odd M < 2^11 lies at least 2^-36 (relative) from every fp32 rounding midpoint, so the final rounding
// is the correct one. Branch-free; d = inf is not an input (those groups take the scalar path).
__device__ __forceinline__ float kv_recip(float d) {
    float y0;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y0) : "f"(d));
    const float y = fmaf(y0, fmaf(-d, y0, 1.0f), y0);
    return d > 0.f ? y : 0.f;
}

// The 8 codes of this lane's elements in a 64-element group with scale d (r = RN(1/d), 0 when d = 0),
// packed little-endian into a uint2. Codes are rint(x / d) clamped to [-127, 127] of the correctly
// rounded quotient, computed without a divide per element (Markstein's theorem: with r = RN(1/d) and
// q0 = RN(x*r) within one ulp of x/d, the residual e = x - q0*d is exact under FMA and RN(q0 + e*r) is
// the correctly rounded quotient; d is 0 or an fp16 value >= 2^-24, so nothing underflows where the
// rounding can change the code), in packed fp32, and rounded to the nearest even integer as the low
// byte of fl(q + 1.5 * 2^23). kClamp = false needs every |x| <= the group max am and d a normal fp16
// (or 0): then d >= (am / 127)(1 - 2^-24)(1 - 2^-11), |x / d| < 127.07 and the clamp cannot act.
// Every x must be finite and d <= 65504.
template <bool kClamp>
__device__ __forceinline__ uint2 kv_q8_pack(const float2 (&x)[4], float d, float r) {
    const float2 nr2 = splat2(-r), r2 = splat2(r), d2 = splat2(d);
    uint32_t b[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 nq0 = fmul2_unfused(x[i], nr2);                         // -RN(x*r)
        const float2 e = ffma2(nq0, d2, x[i]);                               // x - q0*d, exact
        float2 q = ffma2(e, r2, make_float2(-nq0.x, -nq0.y));                // RN(x / d)
        if (kClamp) {
            q.x = fminf(fmaxf(q.x, -127.0f), 127.0f);
            q.y = fminf(fmaxf(q.y, -127.0f), 127.0f);
        }
        const float2 t = fadd2(q, splat2(12582912.0f));                      // rint in the low byte
        b[2 * i] = __float_as_uint(t.x);
        b[2 * i + 1] = __float_as_uint(t.y);
    }
    uint32_t w[2];
#pragma unroll
    for (int k = 0; k < 2; ++k)
        w[k] = __byte_perm(__byte_perm(b[4 * k], b[4 * k + 1], 0x0040),
                           __byte_perm(b[4 * k + 2], b[4 * k + 3], 0x0040), 0x5410);
    return make_uint2(w[0], w[1]);
}

// kv_q8_pack for any group: the packed path while this lane's values are finite (an, the lane's max
// with NaNs kept, is finite) and the scale is finite; otherwise the scalar conversion, so NaN codes are
// 0 (as __float2int_rn) and a finite group whose scale rounds to fp16 infinity (max >= 127 * 65520, fp32
// inputs only) gets x / inf = 0, every code as the reference's expression.
__device__ __forceinline__ uint2 kv_q8_pack_any(const float2 (&x)[4], float an, float d, float r) {
    if (an <= 3.402823466e38f && d <= 65504.0f) return kv_q8_pack<true>(x, d, r);
    uint32_t w[2] = {0u, 0u};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float v = (i & 1) ? x[i >> 1].y : x[i >> 1].x;
        const int qi = d > 0.f ? max(-127, min(127, __float2int_rn(v / d))) : 0;
        w[i >> 2] |= ((uint32_t)(qi & 0xFF)) << ((i & 3) * 8);
    }
    return make_uint2(w[0], w[1]);
}

// Store a lane's packed codes (and, from the group's first lane, the fp16 scale) to up to two cells.
__device__ __forceinline__ void kv_q8_store(uint2 codes, uint16_t sbits, int lane, int8_t* q0, uint16_t* s0,
                                            int8_t* q1, uint16_t* s1) {
    const bool first = (lane & 7) == 0;
    if (q0 != nullptr) {
        *reinterpret_cast<uint2*>(q0) = codes;
        if (first) *s0 = sbits;
    }
    if (q1 != nullptr) {
        *reinterpret_cast<uint2*>(q1) = codes;
        if (first) *s1 = sbits;
    }
}

// One warp per (token, group of kR rounds of heads): HD/8 lanes per head, 32/(HD/8) heads side by
// side per round. kR = 1 (small calls, e.g. decode) spreads a token's heads over warps for the
// shortest chain; kR = 2 (long calls) keeps the reference's 2 heads of 256 on one warp, with the k and
// v vectors of both rounds loaded before any arithmetic and the token's cell and cos/sin work done
// once. The cos/sin slice is loaded behind the head vectors.
// HAS_Q: the launch carries q heads (the q-item code is compiled out otherwise, which keeps the k/v-only
// kernel's registers down).
template <typename T, int HD, int kR, bool HAS_Q>
__global__ void __launch_bounds__(128, HAS_Q && sizeof(T) == 4 ? 3 : 4) kv_append_kernel(const KvAppendArgs a) {
    pdl_begin();
    constexpr int L = HD / 8;
    constexpr int HPW = 32 / L;
    const int lane = threadIdx.x & 31;
    const int li = lane % L, hw = lane / L;
    const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int64_t gwarp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int kvd = a.kv_heads * HD;
    const int spc = kvd / kKvGroup;  // scales per cell
    const int half = a.rot / 2, hl = half / 8;
    const bool rot_lane = li < 2 * hl, first_half = li < hl;
    const int src = rot_lane ? (first_half ? lane + hl : lane - hl) : lane;
    const int ci = (first_half ? li : li - hl) * 8;
    const int64_t base = (a.d_base_pos ? (int64_t)__ldg(a.d_base_pos) : 0) + a.pos_offset;
    const int64_t end = base + a.T;
    const int rounds = (a.kv_heads + HPW - 1) / HPW;
    const int groups = (rounds + kR - 1) / kR;
    const int q_rounds = (a.q_heads + HPW - 1) / HPW;
    const int per_tok = groups + (q_rounds + kR - 1) / kR;  // k/v items, then q items
    const int64_t items = a.T * per_tok;
    T* const kd = static_cast<T*>(a.k);
    const T* const vd = static_cast<const T*>(a.v);

    float2 g[4];  // k gamma (+ offset) of this lane's 8 dims
#pragma unroll
    for (int i = 0; i < 4; ++i) g[i] = splat2(0.f);
    if (a.norm_rope) {
        Vec8<T>::load_ro2(static_cast<const T*>(a.k_gamma) + li * 8, g);
#pragma unroll
        for (int i = 0; i < 4; ++i) g[i] = fadd2(splat2(a.w_offset), g[i]);
    }
    // cos/sin of position pos for this lane's 8 dims (the first rotary half with -sin)
    auto load_cos_sin = [&](int64_t pos, float2 (&c2)[4], float2 (&s2)[4]) {
        Vec8<float>::load_ro2(a.cos_tab + pos * half + ci, c2);
        Vec8<float>::load_ro2(a.sin_tab + pos * half + ci, s2);
        if (first_half) {
#pragma unroll
            for (int i = 0; i < 4; ++i) s2[i] = make_float2(-s2[i].x, -s2[i].y);
        }
    };
    // p[j] *= rsqrt(mean(p[j]^2) + eps) * gamma, then the pair rotation (one shuffle per element), for
    // the N heads in p (float2[N][4]) together, so their dependent chains interleave
    auto norm_rotate = [&](auto& p, const float2 (&gm)[4], bool rot, const float2 (&c2)[4], const float2 (&s2)[4]) {
        constexpr int N = sizeof(p) / sizeof(p[0]);
        float ss[N];
#pragma unroll
        for (int j = 0; j < N; ++j) ss[j] = sumsq8(p[j]);
#pragma unroll
        for (int o = L / 2; o > 0; o >>= 1) {
            float tt[N];
#pragma unroll
            for (int j = 0; j < N; ++j) tt[j] = __shfl_xor_sync(0xffffffffu, ss[j], o);
#pragma unroll
            for (int j = 0; j < N; ++j) ss[j] += tt[j];
        }
        float2 q[N][4];
#pragma unroll
        for (int j = 0; j < N; ++j) {
            const float2 sc = splat2(rsqrt_approx(ss[j] / (float)HD + a.eps));
#pragma unroll
            for (int i = 0; i < 4; ++i) p[j][i] = fmul2(p[j][i], fmul2(sc, gm[i]));
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                q[j][i].x = __shfl_sync(0xffffffffu, p[j][i].x, src);
                q[j][i].y = __shfl_sync(0xffffffffu, p[j][i].y, src);
            }
        }
        if (rot) {
#pragma unroll
            for (int j = 0; j < N; ++j)
#pragma unroll
                for (int i = 0; i < 4; ++i) p[j][i] = ffma2(q[j][i], s2[i], fmul2(p[j][i], c2[i]));
        }
    };

    StridePos ps(gwarp, nwarps, per_tok);  // item = (token q, round group r)
    for (int64_t it = gwarp; it < items; it += nwarps, ps.advance()) {
        const int64_t t = ps.q;
        if (HAS_Q && ps.r >= groups) {  // q heads of this token: norm + rotation in place, nothing appended
            const int q0 = (ps.r - groups) * kR;
            T* const qrow = static_cast<T*>(a.q) + t * a.q_row_stride;
            typename Vec8<T>::Raw qr[kR];
#pragma unroll
            for (int j = 0; j < kR; ++j) {
                const int h = (q0 + j) * HPW + hw;
                if (q0 + j < q_rounds && h < a.q_heads) qr[j] = Vec8<T>::ldcs_raw(qrow + h * a.q_head_stride + li * 8);
            }
            float2 gq[4];
            Vec8<T>::load_ro2(static_cast<const T*>(a.q_gamma) + li * 8, gq);
#pragma unroll
            for (int i = 0; i < 4; ++i) gq[i] = fadd2(splat2(a.w_offset), gq[i]);
            const int64_t pos = base + t;
            const bool pos_ok = half > 0 && pos >= 0 && pos < a.table_rows;
            float2 c2[4], s2[4];
            if (pos_ok && rot_lane) load_cos_sin(pos, c2, s2);
            // one head at a time: interleaving the q heads' chains measured slower (register pressure)
#pragma unroll
            for (int j = 0; j < kR; ++j) {
                if (q0 + j >= q_rounds) break;  // warp-uniform
                const int h = (q0 + j) * HPW + hw;
                const bool act = h < a.q_heads;
                float2 p[1][4];
                if (act) {
                    Vec8<T>::cvt2(qr[j], p[0]);
                } else {
#pragma unroll
                    for (int i = 0; i < 4; ++i) p[0][i] = splat2(0.f);
                }
                norm_rotate(p, gq, pos_ok && rot_lane, c2, s2);
                if (act) Vec8<T>::store2(qrow + h * a.q_head_stride + li * 8, p[0]);
            }
            continue;
        }
        const int r0 = ps.r * kR;
        typename Vec8<T>::Raw kr[kR], vr[kR];
#pragma unroll
        for (int j = 0; j < kR; ++j) {
            const int h = (r0 + j) * HPW + hw;
            if (r0 + j < rounds && h < a.kv_heads) {
                kr[j] = Vec8<T>::ldcs_raw(kd + t * kvd + h * HD + li * 8);
                vr[j] = Vec8<T>::ldcs_raw(vd + t * kvd + h * HD + li * 8);
            }
        }
        const int64_t pos = base + t;
        const bool keep = pos >= 0 && pos < a.c.max_ctx;
        const bool ring = keep && kv_in_ring(pos, end, a.c.ring_cap);
        const int64_t rcell = ring ? kv_ring_cell(pos, a.c.ring_cap, a.ring_div, a.ring_recip) : 0;
        const bool full = keep && a.c.full_k_q != nullptr;
        const bool pos_ok = half > 0 && pos >= 0 && pos < a.table_rows;
        float2 c2[4], s2[4];
        if (a.norm_rope) {
            if (pos_ok && rot_lane) load_cos_sin(pos, c2, s2);
            if (half > 0 && !pos_ok && lane == 0 && r0 == 0) raise_fault(WZYB_FAULT_POS_RANGE);
        }
        // the kR rounds' heads go through each step together, so their dependent chains interleave
        // (a round past the last one runs on zeros and stores nothing)
        bool act[kR];
        int col[kR];
        float2 p[kR][4], v[kR][4];
#pragma unroll
        for (int j = 0; j < kR; ++j) {
            const int h = (r0 + j) * HPW + hw;
            act[j] = r0 + j < rounds && h < a.kv_heads;
            col[j] = h * HD + li * 8;
            if (act[j]) {
                Vec8<T>::cvt2(kr[j], p[j]);
                Vec8<T>::cvt2(vr[j], v[j]);
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i) p[j][i] = v[j][i] = splat2(0.f);
            }
        }
        if (a.norm_rope) {  // warp-uniform
            norm_rotate(p, g, pos_ok && rot_lane, c2, s2);
#pragma unroll
            for (int j = 0; j < kR; ++j)
                if (act[j]) Vec8<T>::store2(kd + t * kvd + col[j], p[j]);
        }
        if (keep) {  // warp-uniform
            constexpr int N = 2 * kR;  // vectors: k and v of each round
            float am[N], an[N], d[N], r[N];
            __half sh[N];
#pragma unroll
            for (int j = 0; j < kR; ++j) {
                kv_lane_max(p[j], am[2 * j], an[2 * j]);
                kv_lane_max(v[j], am[2 * j + 1], an[2 * j + 1]);
            }
            kv_group_max<N>(am);
            bool plain = true;  // every vector finite with a normal (or zero) fp16 scale
#pragma unroll
            for (int m = 0; m < N; ++m) {
                sh[m] = kv_group_scale(am[m]);
                d[m] = __half2float(sh[m]);
                r[m] = kv_recip(d[m]);
                plain = plain && an[m] <= 3.402823466e38f && d[m] <= 65504.0f &&
                        (d[m] >= 6.103515625e-05f || d[m] == 0.f);
            }
            uint2 codes[N];
            if (plain) {
#pragma unroll
                for (int j = 0; j < kR; ++j) {
                    codes[2 * j] = kv_q8_pack<false>(p[j], d[2 * j], r[2 * j]);
                    codes[2 * j + 1] = kv_q8_pack<false>(v[j], d[2 * j + 1], r[2 * j + 1]);
                }
            } else {
#pragma unroll
                for (int j = 0; j < kR; ++j) {
                    codes[2 * j] = kv_q8_pack_any(p[j], an[2 * j], d[2 * j], r[2 * j]);
                    codes[2 * j + 1] = kv_q8_pack_any(v[j], an[2 * j + 1], d[2 * j + 1], r[2 * j + 1]);
                }
            }
#pragma unroll
            for (int j = 0; j < kR; ++j) {
                if (!act[j]) continue;
                const int c = col[j], sc_i = c / kKvGroup;
                kv_q8_store(codes[2 * j], __half_as_ushort(sh[2 * j]), lane,
                            ring ? a.c.ring_k_q + rcell * kvd + c : nullptr, a.c.ring_k_s + rcell * spc + sc_i,
                            full ? a.c.full_k_q + pos * kvd + c : nullptr, full ? a.c.full_k_s + pos * spc + sc_i : nullptr);
                kv_q8_store(codes[2 * j + 1], __half_as_ushort(sh[2 * j + 1]), lane,
                            ring ? a.c.ring_v_q + rcell * kvd + c : nullptr, a.c.ring_v_s + rcell * spc + sc_i,
                            full ? a.c.full_v_q + pos * kvd + c : nullptr, full ? a.c.full_v_s + pos * spc + sc_i : nullptr);
            }
        }
    }
}

template <typename T>
static int launch_kv_append(KvAppendArgs a, int head_dim, cudaStream_t stream) {
    const wzyb_kv_cache& c = a.c;
    if (!a.k || !a.v || !c.ring_k_q || !c.ring_k_s || !c.ring_v_q || !c.ring_v_s) return WZYB_ERR_NULL;
    const bool has_full = c.full_k_q || c.full_k_s || c.full_v_q || c.full_v_s;
    if (has_full && !(c.full_k_q && c.full_k_s && c.full_v_q && c.full_v_s)) return WZYB_ERR_NULL;
    if (a.norm_rope && (!a.k_gamma || (a.rot > 0 && (!a.cos_tab || !a.sin_tab)))) return WZYB_ERR_NULL;
    if (a.T < 0 || a.T > (int64_t(1) << 40) || a.kv_heads < 1 || a.kv_heads > 64 ||
        (head_dim != 64 && head_dim != 128 && head_dim != 256) || c.ring_cap < 1 || c.max_ctx < 0)
        return WZYB_ERR_SHAPE;
    if (a.norm_rope && (a.rot < 0 || a.rot > head_dim || (a.rot % 16) != 0 || a.table_rows < 0)) return WZYB_ERR_SHAPE;
    if (!aligned16(a.k) || !aligned16(a.v) || (a.norm_rope && !aligned16(a.k_gamma)) || !aligned16(c.ring_k_q) ||
        !aligned16(c.ring_v_q) || (has_full && (!aligned16(c.full_k_q) || !aligned16(c.full_v_q))) ||
        (a.norm_rope && a.rot > 0 && (!aligned16(a.cos_tab) || !aligned16(a.sin_tab))))
        return WZYB_ERR_ALIGN;
    if (((uintptr_t)c.ring_k_s | (uintptr_t)c.ring_v_s | (uintptr_t)c.full_k_s | (uintptr_t)c.full_v_s) & 1)
        return WZYB_ERR_ALIGN;
    if (a.q_heads > 0) {  // the fused q heads (norm_rope only)
        if (!a.norm_rope || !a.q || !a.q_gamma) return WZYB_ERR_NULL;
        if (a.q_heads > 256 || (a.q_heads > 1 && a.q_head_stride < head_dim) || a.q_head_stride < 0 ||
            a.q_row_stride < 0)
            return WZYB_ERR_SHAPE;
        // tokens' q heads must not overlap: each is normalised and rotated in place at its own position
        const int64_t q_row_span = (int64_t)(a.q_heads - 1) * a.q_head_stride + head_dim;
        if (a.T > 1 && a.q_row_stride < q_row_span) return WZYB_ERR_SHAPE;
        if (!aligned16(a.q) || !aligned16(a.q_gamma) || ((a.q_head_stride * (int64_t)sizeof(T)) % 16) != 0 ||
            ((a.q_row_stride * (int64_t)sizeof(T)) % 16) != 0)
            return WZYB_ERR_ALIGN;
        // q is rewritten in place while k and v are read: the three must not share bytes
        if (a.T > 0) {
            const uintptr_t q0 = (uintptr_t)a.q;
            const uintptr_t q1 = q0 + (uintptr_t)(((a.T - 1) * a.q_row_stride + q_row_span) * (int64_t)sizeof(T));
            const uintptr_t kv_bytes = (uintptr_t)(a.T * (int64_t)a.kv_heads * head_dim * (int64_t)sizeof(T));
            const uintptr_t k0 = (uintptr_t)a.k, v0 = (uintptr_t)a.v;
            if ((q0 < k0 + kv_bytes && k0 < q1) || (q0 < v0 + kv_bytes && v0 < q1)) return WZYB_ERR_SHAPE;
        }
    } else if (a.q_heads < 0) {
        return WZYB_ERR_SHAPE;
    }
    if (a.T == 0) return WZYB_OK;
    DeviceInfo di;
    const int rc = device_info(&di);
    if (rc != WZYB_OK) return rc;
    a.ring_div = (uint64_t)(c.ring_cap <= 2 * kKvSinkPin ? c.ring_cap : c.ring_cap - kKvSinkPin);
    a.ring_recip = ~0ull / a.ring_div;
    const int hpw = 32 / (head_dim / 8);
    const int64_t rounds = (a.kv_heads + hpw - 1) / hpw;
    const int64_t q_rounds = (a.q_heads + hpw - 1) / hpw;
    // one round per warp while the call is smaller than a few warps per SM, else two
    const Tuning tu = tuning(kFamKv);
    const bool split = tu.stages == 1 || (tu.stages != 2 && a.T * (rounds + q_rounds) <= (int64_t)di.sms * 32);
    const int64_t items = split ? a.T * (rounds + q_rounds) : a.T * ((rounds + 1) / 2 + (q_rounds + 1) / 2);
    // 128-thread CTAs: the same warps per SM as 256-thread ones at these registers, in finer CTAs
    // (4096 / 65,536 / 262,144 tokens: 14.3 -> 14.1, 105.8 -> 101.4, 390 -> 381 us)
    constexpr int thr = 128;
    const int grid = persistent_grid(di, tu.ctas_per_sm, (items + thr / 32 - 1) / (thr / 32));
#define WZYB_KV(HDV)                                                                              \
    if (a.q_heads > 0) {                                                                          \
        if (split) launch_k(kv_append_kernel<T, HDV, 1, true>, grid, thr, 0, stream, a);                \
        else launch_k(kv_append_kernel<T, HDV, 2, true>, grid, thr, 0, stream, a);                      \
    } else {                                                                                      \
        if (split) launch_k(kv_append_kernel<T, HDV, 1, false>, grid, thr, 0, stream, a);               \
        else launch_k(kv_append_kernel<T, HDV, 2, false>, grid, thr, 0, stream, a);                     \
    }
    switch (head_dim) {
        case 64: { WZYB_KV(64) break; }
        case 128: { WZYB_KV(128) break; }
        default: { WZYB_KV(256) break; }
    }
#undef WZYB_KV
    return launch_status();
}

template <typename T>
static int kv_append_entry(T* k, const T* k_gamma, const T* v, const float* cos_tab, const float* sin_tab,
                           int64_t table_rows, const int32_t* d_base_pos, int64_t pos_offset, int64_t T_, int kv_heads,
                           int head_dim, int rot_dims, float eps, float w_offset, int norm_rope,
                           const wzyb_kv_cache* cache, cudaStream_t stream, const wzyb_head_tensor* q = nullptr) {
    if (cache == nullptr) return WZYB_ERR_NULL;
    KvAppendArgs a;
    a.q = q ? q->data : nullptr;
    a.q_gamma = q ? q->gamma : nullptr;
    a.q_heads = q ? q->heads : 0;
    a.q_head_stride = q ? q->head_stride : 0;
    a.q_row_stride = q ? q->row_stride : 0;
    a.k = k;
    a.k_gamma = k_gamma;
    a.v = v;
    a.cos_tab = cos_tab;
    a.sin_tab = sin_tab;
    a.table_rows = table_rows;
    a.d_base_pos = d_base_pos;
    a.pos_offset = pos_offset;
    a.T = T_;
    a.kv_heads = kv_heads;
    a.rot = norm_rope ? rot_dims : 0;
    a.eps = eps;
    a.w_offset = w_offset;
    a.norm_rope = norm_rope;
    a.c = *cache;
    return launch_kv_append<T>(a, head_dim, stream);
}

}  // namespace wzyb

extern "C" {

int wzyb_kv_append_int8_f32(const float* k, const float* v, int64_t T, int kv_heads, int head_dim,
                            const int32_t* d_base_pos, int64_t pos_offset, const wzyb_kv_cache* cache,
                            wzyb_stream_t stream) {
    return wzyb::kv_append_entry<float>(const_cast<float*>(k), nullptr, v, nullptr, nullptr, 0, d_base_pos, pos_offset,
                                        T, kv_heads, head_dim, 0, 0.f, 0.f, 0, cache, (cudaStream_t)stream);
}

int wzyb_k_rope_kv_append_f32(float* k, const float* k_gamma, const float* v, const float* cos_tab,
                              const float* sin_tab, int64_t table_rows, const int32_t* d_base_pos, int64_t pos_offset,
                              int64_t T, int kv_heads, int head_dim, int rot_dims, float eps, float w_offset,
                              const wzyb_kv_cache* cache, wzyb_stream_t stream) {
    return wzyb::kv_append_entry<float>(k, k_gamma, v, cos_tab, sin_tab, table_rows, d_base_pos, pos_offset, T,
                                        kv_heads, head_dim, rot_dims, eps, w_offset, 1, cache, (cudaStream_t)stream);
}

int wzyb_qk_rope_kv_append_f32(const wzyb_head_tensor* q, float* k, const float* k_gamma, const float* v,
                               const float* cos_tab, const float* sin_tab, int64_t table_rows,
                               const int32_t* d_base_pos, int64_t pos_offset, int64_t T, int kv_heads, int head_dim,
                               int rot_dims, float eps, float w_offset, const wzyb_kv_cache* cache,
                               wzyb_stream_t stream) {
    if (q == nullptr) return WZYB_ERR_NULL;
    return wzyb::kv_append_entry<float>(k, k_gamma, v, cos_tab, sin_tab, table_rows, d_base_pos, pos_offset, T,
                                        kv_heads, head_dim, rot_dims, eps, w_offset, 1, cache, (cudaStream_t)stream, q);
}

int wzyb_qk_rope_kv_append_f16(const wzyb_head_tensor* q, uint16_t* k, const uint16_t* k_gamma, const uint16_t* v,
                               const float* cos_tab, const float* sin_tab, int64_t table_rows,
                               const int32_t* d_base_pos, int64_t pos_offset, int64_t T, int kv_heads, int head_dim,
                               int rot_dims, float eps, float w_offset, const wzyb_kv_cache* cache,
                               wzyb_stream_t stream) {
    if (q == nullptr) return WZYB_ERR_NULL;
    return wzyb::kv_append_entry<__half>((__half*)k, (const __half*)k_gamma, (const __half*)v, cos_tab, sin_tab,
                                         table_rows, d_base_pos, pos_offset, T, kv_heads, head_dim, rot_dims, eps,
                                         w_offset, 1, cache, (cudaStream_t)stream, q);
}

int wzyb_k_rope_kv_append_f16(uint16_t* k, const uint16_t* k_gamma, const uint16_t* v, const float* cos_tab,
                              const float* sin_tab, int64_t table_rows, const int32_t* d_base_pos, int64_t pos_offset,
                              int64_t T, int kv_heads, int head_dim, int rot_dims, float eps, float w_offset,
                              const wzyb_kv_cache* cache, wzyb_stream_t stream) {
    return wzyb::kv_append_entry<__half>((__half*)k, (const __half*)k_gamma, (const __half*)v, cos_tab, sin_tab,
                                         table_rows, d_base_pos, pos_offset, T, kv_heads, head_dim, rot_dims, eps,
                                         w_offset, 1, cache, (cudaStream_t)stream);
}

}  // extern "C"
