// head_rope.cu -- per-head RMSNorm + partial NeoX RoPE, in place; q and k of a token in one unit.
//
// Math follows fused_head_norm_rope_multi (src/wzy_qsa_256k.cuh:50-84):
//   p *= rsqrt(sum(p^2)/hd + eps) * gamma
//   (a, d) = (p[i], p[i+R/2]), i < R/2:  p[i] = a*cos - d*sin;  p[i+R/2] = a*sin + d*cos
// with cos/sin from a [pos][R/2] fp32 table built in fp64 (build_rope_cos_sin_host,
// src/wzy_qsa_256k.cuh:33-46). The reference runs one 128-thread block per (head, token) with three
// __syncthreads and rotates on 32 of the 128 threads. Here no design uses a shared-memory reduction:
//   pair   (default): hd/16 lanes per head, each holding the two 8-element chunks of a rotation pair
//          (or two plain chunks), so the rotation needs no shuffle; heads reduced with xor shuffles;
//          6 heads per warp item, or a whole token for long calls;
//   direct: hd/8 lanes per head, the rotation partner fetched from the lane R/16 away by shuffles;
//   async (on request): the direct design's units staged in shared memory by cp.async.
#include <cmath>

#include "launch.hpp"

namespace wzyb {

struct HeadSection {
    void* data;
    const void* gamma;
    int heads;
    int64_t head_stride;
    int64_t row_stride;
};

struct HeadRopeArgs {
    HeadSection sec[2];  // q, k (k.heads may be 0)
    const float* cos_tab;
    const float* sin_tab;
    int64_t table_rows;
    const int32_t* d_base_pos;
    int64_t pos_offset;
    int64_t T;
    int rot;  // rot_dims
    float eps;
    float w_offset;
};

// ---- per-head math shared by the direct and async designs (packed fp32) ------------------------
// gamma of this lane's 8 dims for the q (g[0]) and k (g[1]) sections, with the weight offset added
template <typename T>
__device__ __forceinline__ void load_head_gammas(const HeadRopeArgs& a, int li, float2 (&g)[2][4]) {
#pragma unroll
    for (int s = 0; s < 2; ++s) {
#pragma unroll
        for (int i = 0; i < 4; ++i) g[s][i] = splat2(0.f);
        if (a.sec[s].heads > 0) {
            Vec8<T>::load_ro2(static_cast<const T*>(a.sec[s].gamma) + li * 8, g[s]);
#pragma unroll
            for (int i = 0; i < 4; ++i) g[s][i] = fadd2(splat2(a.w_offset), g[s][i]);
        }
    }
}

// cos and a signed sin, so that both halves rotate with out = own*cos + partner*ssin:
// first half a*cos - d*sin (ssin = -sin), second half d*cos + a*sin (ssin = +sin).
__device__ __forceinline__ void sign_sin(bool first_half, float2 (&s2)[4]) {
    if (first_half) {
#pragma unroll
        for (int i = 0; i < 4; ++i) s2[i] = make_float2(-s2[i].x, -s2[i].y);
    }
}

// One head's 8-element slice in this lane: p *= rsqrt(mean(p^2) + eps) * gamma over the head's L
// lanes, then (rotate) the NeoX pair rotation with the partner slice fetched from lane `src`.
template <int L, int HD>
__device__ __forceinline__ void norm_rope_head(float2 (&p)[4], bool q_gamma, const float2 (&g)[2][4], float eps,
                                               int src, bool rotate, const float2 (&c2)[4], const float2 (&s2)[4]) {
    const float ss = group_sum<L>(sumsq8(p));
    const float2 sc = splat2(rsqrt_approx(ss / (float)HD + eps));
    if (q_gamma) {  // warp-uniform when a warp holds one head
#pragma unroll
        for (int i = 0; i < 4; ++i) p[i] = fmul2(p[i], fmul2(sc, g[0][i]));
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) p[i] = fmul2(p[i], fmul2(sc, g[1][i]));
    }
    float2 q[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        q[i].x = __shfl_sync(0xffffffffu, p[i].x, src);
        q[i].y = __shfl_sync(0xffffffffu, p[i].y, src);
    }
    if (rotate) {
#pragma unroll
        for (int i = 0; i < 4; ++i) p[i] = ffma2(q[i], s2[i], fmul2(p[i], c2[i]));
    }
}

// The same per-head math with the lane's 8 gammas given as two float4 (read from a lane-major table
// in shared memory), which keeps 16 registers per thread free for more resident warps.
template <int L, int HD>
__device__ __forceinline__ void norm_rope_head_sg(float2 (&p)[4], const float4 ga, const float4 gb, float eps, int src,
                                                  bool rotate, const float2 (&c2)[4], const float2 (&s2)[4]) {
    const float ss = group_sum<L>(sumsq8(p));
    const float2 sc = splat2(rsqrt_approx(ss / (float)HD + eps));
    p[0] = fmul2(p[0], fmul2(sc, make_float2(ga.x, ga.y)));
    p[1] = fmul2(p[1], fmul2(sc, make_float2(ga.z, ga.w)));
    p[2] = fmul2(p[2], fmul2(sc, make_float2(gb.x, gb.y)));
    p[3] = fmul2(p[3], fmul2(sc, make_float2(gb.z, gb.w)));
    float2 q[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        q[i].x = __shfl_sync(0xffffffffu, p[i].x, src);
        q[i].y = __shfl_sync(0xffffffffu, p[i].y, src);
    }
    if (rotate) {
#pragma unroll
        for (int i = 0; i < 4; ++i) p[i] = ffma2(q[i], s2[i], fmul2(p[i], c2[i]));
    }
}

// Direct design: a warp owns a chunk of kNH*(32/L) consecutive heads of ONE token (q heads first,
// then k heads), so the token's cos/sin row is fetched once per chunk. All heads of the chunk are
// loaded as raw 16-byte registers before any arithmetic; each head is then normalised inside its
// lane group and rotated with one shuffle per element, and written back in place. The only shared
// memory holds the two gammas (2 KB, written once before the single CTA barrier at kernel start);
// 128-thread CTAs and ~90 registers give ~20 resident warps per SM.
template <typename T, int HD, int kNH>
__global__ void __launch_bounds__(128) head_rope_direct_kernel(const HeadRopeArgs a) {
    pdl_begin();
    constexpr int L = HD / 8;
    constexpr int HPW = 32 / L;         // heads side by side in one warp
    constexpr int CH = kNH * HPW;       // heads per chunk
    const int lane = threadIdx.x & 31;
    const int li = lane % L;            // lane inside its head
    const int hw = lane / L;            // head slot inside the warp
    const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int64_t gwarp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int hq = a.sec[0].heads, htot = hq + a.sec[1].heads;
    const int chunks = (htot + CH - 1) / CH;
    const int64_t items = a.T * chunks;
    const int half = a.rot / 2, hl = half / 8;
    const bool rot_lane = li < 2 * hl, first_half = li < hl;
    const int src = rot_lane ? (first_half ? lane + hl : lane - hl) : lane;
    const int ci = (first_half ? li : li - hl) * 8;
    const int64_t base_pos = (a.d_base_pos ? (int64_t)__ldg(a.d_base_pos) : 0) + a.pos_offset;

    // gammas (+ weight offset) of both sections as fp32 in shared memory, lane-major: sgl[s][k][l] holds
    // dims 8l + 4k .. +3, so each of a head's two 16-byte gamma loads reads one contiguous span (no
    // bank conflicts; lanes of other heads of the same section in the warp read the same words)
    __shared__ __align__(16) float4 sgl[2][2][L];
    for (int i = threadIdx.x; i < 4 * L; i += blockDim.x) {
        const int s = i / (2 * L), k = (i / L) % 2, l = i % L;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (a.sec[s].heads > 0) {
            const T* gm = static_cast<const T*>(a.sec[s].gamma) + l * 8 + k * 4;
            v = make_float4(a.w_offset + (float)gm[0], a.w_offset + (float)gm[1], a.w_offset + (float)gm[2],
                            a.w_offset + (float)gm[3]);
        }
        sgl[s][k][l] = v;
    }
    __syncthreads();

    // Section row bases are formed once per token; a head is then one 64-bit multiply-add away.
    T* const qdata = static_cast<T*>(a.sec[0].data);
    T* const kdata = static_cast<T*>(a.sec[1].heads > 0 ? a.sec[1].data : a.sec[0].data);
    const int64_t qrs = a.sec[0].row_stride, qhs = a.sec[0].head_stride;
    const int64_t krs = a.sec[1].row_stride, khs = a.sec[1].head_stride;

    StridePos ps(gwarp, nwarps, chunks);  // item it = (token q, chunk r)
    for (int64_t it = gwarp; it < items; it += nwarps, ps.advance()) {
        const int64_t t = ps.q;
        const int h0 = ps.r * CH;
        T* const qrow = qdata + t * qrs + li * 8;
        T* const krow = kdata + t * krs + li * 8;
        auto head_ptr = [&](int h) -> T* { return h < hq ? qrow + h * qhs : krow + (h - hq) * khs; };
        typename Vec8<T>::Raw rp[kNH];
#pragma unroll
        for (int j = 0; j < kNH; ++j) {
            const int h = h0 + j * HPW + hw;
            if (h < htot) rp[j] = Vec8<T>::ldcs_raw(head_ptr(h));
        }
        const int64_t pos = base_pos + t;
        const bool pos_ok = half > 0 && pos >= 0 && pos < a.table_rows;
        float2 c2[4], s2[4];
        if (pos_ok && rot_lane) {
            Vec8<float>::load_ro2(a.cos_tab + pos * half + ci, c2);
            Vec8<float>::load_ro2(a.sin_tab + pos * half + ci, s2);
            sign_sin(first_half, s2);
        }
        if (half > 0 && !pos_ok && lane == 0 && h0 == 0) raise_fault(WZYB_FAULT_POS_RANGE);
#pragma unroll
        for (int j = 0; j < kNH; ++j) {
            if (h0 + j * HPW >= htot) break;  // warp-uniform: no head of this round exists
            const int h = h0 + j * HPW + hw;
            float2 p[4];
            if (h < htot) {
                Vec8<T>::cvt2(rp[j], p);
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i) p[i] = splat2(0.f);
            }
            const int sec = h < hq ? 0 : 1;
            norm_rope_head_sg<L, HD>(p, sgl[sec][0][li], sgl[sec][1][li], a.eps, src, pos_ok && rot_lane, c2, s2);
            if (h < htot) Vec8<T>::store2(head_ptr(h), p);
        }
    }
}

// Pair design: the direct design's per-token head chunks with L2 = HD/16 lanes per head, each lane
// holding two 8-element chunks. With P = rot/16 rotary chunk pairs (c, c + P), lane m < P holds exactly
// the pair (m, m + P), so the NeoX rotation is done inside the lane with no shuffle; lanes m >= P hold
// chunks m + P and m + L2 of the rest of the head, so the first load instruction of a head covers
// chunks [0, P) and [2P, L2 + P) and the second [P, 2P) and [L2 + P, 2 L2): every 32-byte sector is
// read whole by one instruction (16 sectors per head, not 28). The norm reduces over L2 lanes. The
// rotation expressions are the direct design's (own*cos + partner*(+-sin), fused), so results match it
// bit for bit. With 3 rounds per item, five CTAs per SM (<= 102 registers, 96 used with no spill)
// instead of the four that an unbounded allocation (106) leaves: 82 -> 86 % of HBM peak at 262K
// tokens on the same box. With 9 rounds, three (156 registers).
// The body takes its CTA's index among `nctas` CTAs that share the items (a fused bundle kernel runs it
// on a subset of its grid); every thread of the CTA must call it (one barrier after the gamma table).
// parts: 1 fills the CTA's gamma table (ending with a CTA barrier), 2 runs the items, 3 both. A kernel
// that runs other work first fills the table at its start and runs the items later (the table is one
// shared array per CTA).
template <typename T, int HD, int kNH>
__device__ __forceinline__ void head_rope_pair_body(const HeadRopeArgs& a, int cta, int nctas, int parts = 3) {
    constexpr int L2 = HD / 16;   // lanes per head
    constexpr int HPW = 32 / L2;  // heads side by side in one warp
    constexpr int CH = kNH * HPW; // heads per chunk item
    const int lane = threadIdx.x & 31;
    const int li = lane % L2;
    const int hw = lane / L2;
    const int64_t nwarps = (int64_t)nctas * (blockDim.x >> 5);
    const int64_t gwarp = (int64_t)cta * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int hq = a.sec[0].heads, htot = hq + a.sec[1].heads;
    const int chunks = (htot + CH - 1) / CH;
    const int64_t items = a.T * chunks;
    const int half = a.rot / 2, P = half / 8;
    const bool rot_lane = li < P;
    const int c0 = rot_lane ? li : li + P;       // first chunk of this lane
    const int c1 = rot_lane ? li + P : li + L2;  // second chunk
    const int64_t base_pos = (a.d_base_pos ? (int64_t)__ldg(a.d_base_pos) : 0) + a.pos_offset;

    // gammas (+ weight offset) as a lane-major table: sgl[s][k][l] = dims 4(k&1).. of chunk c0 (k < 2)
    // or c1 (k >= 2) of lane l, so each 16-byte gamma load of a head reads one contiguous span
    __shared__ __align__(16) float4 sgl[2][4][L2];
    if (parts & 1) {
    for (int i = threadIdx.x; i < 8 * L2; i += blockDim.x) {
        const int s = i / (4 * L2), k = (i / L2) % 4, l = i % L2;
        const int c = k < 2 ? (l < P ? l : l + P) : (l < P ? l + P : l + L2);
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (a.sec[s].heads > 0) {
            const T* gm = static_cast<const T*>(a.sec[s].gamma) + c * 8 + (k & 1) * 4;
            v = make_float4(a.w_offset + (float)gm[0], a.w_offset + (float)gm[1], a.w_offset + (float)gm[2],
                            a.w_offset + (float)gm[3]);
        }
        sgl[s][k][l] = v;
    }
    __syncthreads();
    }
    if (!(parts & 2)) return;

    T* const qdata = static_cast<T*>(a.sec[0].data);
    T* const kdata = static_cast<T*>(a.sec[1].heads > 0 ? a.sec[1].data : a.sec[0].data);
    const int64_t qrs = a.sec[0].row_stride, qhs = a.sec[0].head_stride;
    const int64_t krs = a.sec[1].row_stride, khs = a.sec[1].head_stride;

    StridePos ps(gwarp, nwarps, chunks);  // item it = (token q, chunk r)
    for (int64_t it = gwarp; it < items; it += nwarps, ps.advance()) {
        const int64_t t = ps.q;
        const int h0 = ps.r * CH;
        T* const qrow = qdata + t * qrs;
        T* const krow = kdata + t * krs;
        auto head_ptr = [&](int h) -> T* { return h < hq ? qrow + h * qhs : krow + (h - hq) * khs; };
        typename Vec8<T>::Raw ra[kNH], rb[kNH];
#pragma unroll
        for (int j = 0; j < kNH; ++j) {
            const int h = h0 + j * HPW + hw;
            if (h < htot) {
                T* hp = head_ptr(h);
                ra[j] = Vec8<T>::ldcs_raw(hp + c0 * 8);
                rb[j] = Vec8<T>::ldcs_raw(hp + c1 * 8);
            }
        }
        const int64_t pos = base_pos + t;
        const bool pos_ok = half > 0 && pos >= 0 && pos < a.table_rows;
        float2 c2[4], s2[4];
        if (pos_ok && rot_lane) {
            Vec8<float>::load_ro2(a.cos_tab + pos * half + li * 8, c2);
            Vec8<float>::load_ro2(a.sin_tab + pos * half + li * 8, s2);
        }
        if (half > 0 && !pos_ok && lane == 0 && h0 == 0) raise_fault(WZYB_FAULT_POS_RANGE);
#pragma unroll
        for (int j = 0; j < kNH; ++j) {
            if (h0 + j * HPW >= htot) break;  // warp-uniform: no head of this round exists
            const int h = h0 + j * HPW + hw;
            const bool act = h < htot;
            float2 pa[4], pb[4];
            if (act) {
                Vec8<T>::cvt2(ra[j], pa);
                Vec8<T>::cvt2(rb[j], pb);
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i) pa[i] = pb[i] = splat2(0.f);
            }
            const float ss = group_sum<L2>(sumsq8(pa) + sumsq8(pb));
            const float2 sc = splat2(rsqrt_approx(ss / (float)HD + a.eps));
            const int sec = h < hq ? 0 : 1;
            const float4 ga0 = sgl[sec][0][li], ga1 = sgl[sec][1][li], gb0 = sgl[sec][2][li], gb1 = sgl[sec][3][li];
            pa[0] = fmul2(pa[0], fmul2(sc, make_float2(ga0.x, ga0.y)));
            pa[1] = fmul2(pa[1], fmul2(sc, make_float2(ga0.z, ga0.w)));
            pa[2] = fmul2(pa[2], fmul2(sc, make_float2(ga1.x, ga1.y)));
            pa[3] = fmul2(pa[3], fmul2(sc, make_float2(ga1.z, ga1.w)));
            pb[0] = fmul2(pb[0], fmul2(sc, make_float2(gb0.x, gb0.y)));
            pb[1] = fmul2(pb[1], fmul2(sc, make_float2(gb0.z, gb0.w)));
            pb[2] = fmul2(pb[2], fmul2(sc, make_float2(gb1.x, gb1.y)));
            pb[3] = fmul2(pb[3], fmul2(sc, make_float2(gb1.z, gb1.w)));
            if (pos_ok && rot_lane) {
                // first half a*cos - d*sin, second half d*cos + a*sin, as own*cos + partner*(+-sin)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float2 a_ = pa[i], d_ = pb[i];
                    pa[i] = ffma2(d_, make_float2(-s2[i].x, -s2[i].y), fmul2(a_, c2[i]));
                    pb[i] = ffma2(a_, s2[i], fmul2(d_, c2[i]));
                }
            }
            if (act) {
                T* hp = head_ptr(h);
                // write-back stores: each of the two instructions covers half of every line of the head
                // (streaming stores here cost 86 -> 68 % of peak)
                Vec8<T>::store2_wb(hp + c0 * 8, pa);
                Vec8<T>::store2_wb(hp + c1 * 8, pb);
            }
        }
    }
}

template <typename T, int HD, int kNH>
__global__ void __launch_bounds__(128, kNH >= 9 ? 3 : 5) head_rope_pair_kernel(const HeadRopeArgs a) {
    pdl_begin();
    head_rope_pair_body<T, HD, kNH>(a, blockIdx.x, gridDim.x);
}

// Async design: the direct design's per-token head chunks, but the kP chunks in flight per warp sit
// in a shared-memory ring filled by cp.async (16 bytes per lane per head) together with the token's
// cos/sin row, instead of in registers. Head vectors are lane-private; the cos/sin row is copied by
// the first-half rotary lanes and read by both halves, so each slot is bracketed by __syncwarp.
template <typename T, int HD, int kNH, int kP>
__global__ void __launch_bounds__(128, 6) head_rope_async_kernel(const HeadRopeArgs a) {
    pdl_begin();
    constexpr int L = HD / 8;
    constexpr int HPW = 32 / L;
    constexpr int CH = kNH * HPW;
    constexpr int C = Vec8<T>::kChunks;
    extern __shared__ __align__(16) uint4 sm_hr[];
    const int lane = threadIdx.x & 31;
    const int li = lane % L, hw = lane / L;
    const int half = a.rot / 2, hl = half / 8;
    const int slot_u4 = kNH * C * 32 + 4 * hl;  // head vectors + cos/sin row (hl x 32 B each)
    uint4* ring = sm_hr + (size_t)(threadIdx.x >> 5) * kP * slot_u4;
    const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int64_t gwarp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int hq = a.sec[0].heads, htot = hq + a.sec[1].heads;
    const int chunks = (htot + CH - 1) / CH;
    const int64_t items = a.T * chunks;
    const bool rot_lane = li < 2 * hl, first_half = li < hl;
    const int src = rot_lane ? (first_half ? lane + hl : lane - hl) : lane;
    const int c8i = first_half ? li : li - hl;  // which 8 cos/sin values this lane uses
    const int64_t base_pos = (a.d_base_pos ? (int64_t)__ldg(a.d_base_pos) : 0) + a.pos_offset;

    float2 g[2][4];
    load_head_gammas<T>(a, li, g);
    auto head_ptr = [&](int64_t t, int h) -> T* {
        const int s = h < hq ? 0 : 1;
        const HeadSection& sc = a.sec[s];
        return static_cast<T*>(sc.data) + t * sc.row_stride + (int64_t)(s == 0 ? h : h - hq) * sc.head_stride + li * 8;
    };
    auto pos_in_table = [&](int64_t pos) { return half > 0 && pos >= 0 && pos < a.table_rows; };
    StridePos ipos(gwarp, nwarps, chunks);  // next item to issue
    StridePos cpos(gwarp, nwarps, chunks);  // next item to consume
    auto issue = [&](int64_t it, int slot) {
        const int64_t t = ipos.q;
        const int h0 = ipos.r * CH;
        ipos.advance();
        if (it < items) {
            uint4* sl = ring + slot * slot_u4;
#pragma unroll
            for (int j = 0; j < kNH; ++j) {
                const int h = h0 + j * HPW + hw;
                if (h < htot) Vec8<T>::stage_async(sl + j * C * 32, lane, head_ptr(t, h));
            }
            const int64_t pos = base_pos + t;
            if (pos_in_table(pos) && hw == 0 && li < hl) {
                uint4* tab = sl + kNH * C * 32;
                cp_async16(tab + li * 2, a.cos_tab + pos * half + li * 8);
                cp_async16(tab + li * 2 + 1, a.cos_tab + pos * half + li * 8 + 4);
                cp_async16(tab + (hl + li) * 2, a.sin_tab + pos * half + li * 8);
                cp_async16(tab + (hl + li) * 2 + 1, a.sin_tab + pos * half + li * 8 + 4);
            }
        }
        cp_async_commit();
    };
#pragma unroll
    for (int j = 0; j < kP; ++j) issue(gwarp + j * nwarps, j);

    for (int64_t jj = 0;; ++jj) {
        const int64_t it = gwarp + jj * nwarps;
        if (it >= items) break;  // warp-uniform
        const int slot = (int)(jj % kP);
        const int64_t t = cpos.q;
        const int h0 = cpos.r * CH;
        cpos.advance();
        const int64_t pos = base_pos + t;
        const bool pos_ok = pos_in_table(pos);
        if (half > 0 && !pos_ok && lane == 0 && h0 == 0) raise_fault(WZYB_FAULT_POS_RANGE);
        cp_async_wait<kP - 1>();
        __syncwarp();  // the cos/sin row copied by other lanes is visible
        const uint4* sl = ring + slot * slot_u4;
        float2 c2[4], s2[4];
        if (pos_ok && rot_lane) {
            // cos chunk k at tab[2k], tab[2k+1]; sin chunk k at tab[2(hl+k)], tab[2(hl+k)+1]
            const float4* tab = reinterpret_cast<const float4*>(sl + kNH * C * 32);
            const float4 ca = tab[c8i * 2], cb = tab[c8i * 2 + 1];
            const float4 sa = tab[(hl + c8i) * 2], sb = tab[(hl + c8i) * 2 + 1];
            c2[0] = make_float2(ca.x, ca.y);
            c2[1] = make_float2(ca.z, ca.w);
            c2[2] = make_float2(cb.x, cb.y);
            c2[3] = make_float2(cb.z, cb.w);
            s2[0] = make_float2(sa.x, sa.y);
            s2[1] = make_float2(sa.z, sa.w);
            s2[2] = make_float2(sb.x, sb.y);
            s2[3] = make_float2(sb.z, sb.w);
            sign_sin(first_half, s2);
        }
        // Heads are unstaged one at a time (8 live registers per head, not kNH*8); the other kP-1
        // slots stay in flight meanwhile, and this slot is refilled once all its heads are done.
#pragma unroll
        for (int j = 0; j < kNH; ++j) {
            if (h0 + j * HPW >= htot) break;  // warp-uniform
            const int h = h0 + j * HPW + hw;
            float2 p[4];
            if (h < htot) {
                Vec8<T>::unstage2(sl + j * C * 32, lane, p);
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i) p[i] = splat2(0.f);
            }
            norm_rope_head<L, HD>(p, h < hq, g, a.eps, src, pos_ok && rot_lane, c2, s2);
            if (h < htot) Vec8<T>::store2(head_ptr(t, h), p);
        }
        __syncwarp();  // every lane has read the slot: it may be refilled
        issue(it + kP * nwarps, slot);
    }
    cp_async_wait<0>();
}

template <typename T, int kNH>
static int launch_head_rope_direct(const HeadRopeArgs& a, int hd, int htot, const DeviceInfo& di,
                                   cudaStream_t stream) {
    const void* kern = hd == 64    ? (const void*)head_rope_direct_kernel<T, 64, kNH>
                       : hd == 128 ? (const void*)head_rope_direct_kernel<T, 128, kNH>
                                   : (const void*)head_rope_direct_kernel<T, 256, kNH>;
    const int ch = kNH * (256 / hd);
    const int64_t warp_items = a.T * ((htot + ch - 1) / ch);
    const int grid = persistent_grid(di, resident_ctas(kern, 128, 0), (warp_items + 3) / 4);
    if (hd == 64) launch_k(head_rope_direct_kernel<T, 64, kNH>, grid, 128, 0, stream, a);
    else if (hd == 128) launch_k(head_rope_direct_kernel<T, 128, kNH>, grid, 128, 0, stream, a);
    else launch_k(head_rope_direct_kernel<T, 256, kNH>, grid, 128, 0, stream, a);
    return launch_status();
}

template <typename T, int kNH>
static int launch_head_rope_pair(const HeadRopeArgs& a, int hd, int htot, const DeviceInfo& di, cudaStream_t stream) {
    const void* kern = hd == 64    ? (const void*)head_rope_pair_kernel<T, 64, kNH>
                       : hd == 128 ? (const void*)head_rope_pair_kernel<T, 128, kNH>
                                   : (const void*)head_rope_pair_kernel<T, 256, kNH>;
    const int ch = kNH * (512 / hd);
    const int64_t warp_items = a.T * ((htot + ch - 1) / ch);
    const int grid = persistent_grid(di, resident_ctas(kern, 128, 0), (warp_items + 3) / 4);
    if (hd == 64) launch_k(head_rope_pair_kernel<T, 64, kNH>, grid, 128, 0, stream, a);
    else if (hd == 128) launch_k(head_rope_pair_kernel<T, 128, kNH>, grid, 128, 0, stream, a);
    else launch_k(head_rope_pair_kernel<T, 256, kNH>, grid, 128, 0, stream, a);
    return launch_status();
}

// Validates a head norm+RoPE call on the host and fills `a`. Returns WZYB_OK or the WZYB_ERR_* of the
// first bad argument; nothing is enqueued.
template <typename T>
static int head_rope_prepare(const HeadSection& q, const HeadSection& k, const float* cos_tab, const float* sin_tab,
                             int64_t table_rows, const int32_t* d_base_pos, int64_t pos_offset, int64_t T_, int hd,
                             int rot, float eps, float w_offset, HeadRopeArgs& a) {
    if (q.data == nullptr || q.gamma == nullptr) return WZYB_ERR_NULL;
    if (k.heads > 0 && (k.data == nullptr || k.gamma == nullptr)) return WZYB_ERR_NULL;
    if (rot > 0 && (cos_tab == nullptr || sin_tab == nullptr)) return WZYB_ERR_NULL;
    if (hd != 64 && hd != 128 && hd != 256) return WZYB_ERR_SHAPE;
    if (rot < 0 || rot > hd || (rot % 16) != 0) return WZYB_ERR_SHAPE;
    if (T_ < 0 || T_ > (int64_t(1) << 40) || q.heads < 1 || k.heads < 0 || q.heads + k.heads > 256)
        return WZYB_ERR_SHAPE;
    if (rot > 0 && table_rows < 1) return WZYB_ERR_SHAPE;
    const HeadSection* secs[2] = {&q, &k};
    for (int s = 0; s < 2; ++s) {
        const HeadSection& c = *secs[s];
        if (c.heads == 0) continue;
        if (c.head_stride < hd && c.heads > 1) return WZYB_ERR_SHAPE;
        if (c.row_stride < 0 || c.head_stride < 0) return WZYB_ERR_SHAPE;
        if (!aligned16(c.data) || !aligned16(c.gamma) || ((c.head_stride * (int64_t)sizeof(T)) % 16) != 0 ||
            ((c.row_stride * (int64_t)sizeof(T)) % 16) != 0)
            return WZYB_ERR_ALIGN;
    }
    if (rot > 0 && (!aligned16(cos_tab) || !aligned16(sin_tab))) return WZYB_ERR_ALIGN;
    a.sec[0] = q;
    a.sec[1] = k;
    if (k.heads == 0) a.sec[1] = HeadSection{nullptr, nullptr, 0, 0, 0};
    a.cos_tab = cos_tab;
    a.sin_tab = sin_tab;
    a.table_rows = rot > 0 ? table_rows : 0;
    a.d_base_pos = d_base_pos;
    a.pos_offset = pos_offset;
    a.T = T_;
    a.rot = rot;
    a.eps = eps;
    a.w_offset = w_offset;
    return WZYB_OK;
}

template <typename T>
static int launch_head_rope(const HeadSection& q, const HeadSection& k, const float* cos_tab, const float* sin_tab,
                            int64_t table_rows, const int32_t* d_base_pos, int64_t pos_offset, int64_t T_, int hd,
                            int rot, float eps, float w_offset, cudaStream_t stream) {
    HeadRopeArgs a;
    int rc = head_rope_prepare<T>(q, k, cos_tab, sin_tab, table_rows, d_base_pos, pos_offset, T_, hd, rot, eps,
                                  w_offset, a);
    if (rc != WZYB_OK || T_ == 0) return rc;
    DeviceInfo di;
    rc = device_info(&di);
    if (rc != WZYB_OK) return rc;
    const int htot = q.heads + k.heads;

    if (variant(kFamHeadRope) == WZYB_VARIANT_ASYNC) {
        constexpr int kNH = 4, kP = 4;
        const void* kern = hd == 64    ? (const void*)head_rope_async_kernel<T, 64, kNH, kP>
                           : hd == 128 ? (const void*)head_rope_async_kernel<T, 128, kNH, kP>
                                       : (const void*)head_rope_async_kernel<T, 256, kNH, kP>;
        const int slot_u4 = kNH * Vec8<T>::kChunks * 32 + 4 * (rot / 16);
        const int smem = 4 * kP * slot_u4 * 16;
        rc = ensure_smem(kern, smem);
        if (rc != WZYB_OK) return rc;
        const int ch = kNH * (256 / hd);
        const int64_t warp_items = T_ * ((htot + ch - 1) / ch);
        const int grid = persistent_grid(di, resident_ctas(kern, 128, smem), (warp_items + 3) / 4);
        if (hd == 64) launch_k(head_rope_async_kernel<T, 64, kNH, kP>, grid, 128, smem, stream, a);
        else if (hd == 128) launch_k(head_rope_async_kernel<T, 128, kNH, kP>, grid, 128, smem, stream, a);
        else launch_k(head_rope_async_kernel<T, 256, kNH, kP>, grid, 128, smem, stream, a);
        return launch_status();
    }
    {
        // Pair design by default, 3 rounds of 2 heads per item (6 heads; the 18 heads of the benchmark's
        // q+k are 3 whole items): 83 % of peak at 262K tokens vs 76 % for the direct design, whose rotation
        // shuffles and two gamma loads per head kept the shared-memory pipe ~70 % busy. A ctas_per_sm
        // tuning of 2 selects the other instantiation of either design (pair 2 rounds, direct 6 heads).
        const bool alt = tuning(kFamHeadRope).ctas_per_sm == 2;
        if (variant(kFamHeadRope) == WZYB_VARIANT_DIRECT) {
            if (alt) return launch_head_rope_direct<T, 6>(a, hd, htot, di, stream);
            return launch_head_rope_direct<T, 4>(a, hd, htot, di, stream);
        }
        if (alt) return launch_head_rope_pair<T, 2>(a, hd, htot, di, stream);
        // Long calls: 9 rounds per item (the benchmark's 18 heads are one item per token; 3 CTAs per
        // SM, 9 KB in flight per warp): 90 -> 91 % of peak at 262K tokens. Short calls keep 3 rounds,
        // whose 3x more items fill the GPU better (56 vs 51 % at 4096 tokens).
        const int ch9 = 9 * (512 / hd);
        const int64_t per_tok9 = (htot + ch9 - 1) / ch9;
        const bool fill9 = 3 * htot >= 2 * per_tok9 * ch9;
        if (fill9 && a.T * per_tok9 >= (int64_t)di.sms * 12 * 8) return launch_head_rope_pair<T, 9>(a, hd, htot, di, stream);
        return launch_head_rope_pair<T, 3>(a, hd, htot, di, stream);
    }
}

// ---------------------------------------------------------------------------------------------
// RoPE cos/sin table on the device: one thread per (pos, i), fp64 pow and sincos, rounded to fp32.
// ---------------------------------------------------------------------------------------------
__global__ void rope_table_kernel(float* cos_tab, float* sin_tab, int64_t rows, int half, double theta, int rot) {
    pdl_begin();
    const int64_t n = rows * half;
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < n;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t p = idx / half;
        const int i = (int)(idx - p * half);
        const double inv = pow(theta, -2.0 * (double)i / (double)rot);
        const double ang = (double)p * inv;
        double sv, cv;
        sincos(ang, &sv, &cv);
        cos_tab[idx] = (float)cv;
        sin_tab[idx] = (float)sv;
    }
}

}  // namespace wzyb

extern "C" {

int wzyb_head_norm_rope_f16(uint16_t* data, const uint16_t* gamma, const float* cos_tab, const float* sin_tab,
                            int64_t table_rows, const int32_t* d_base_pos, int64_t pos_offset, int64_t T, int heads,
                            int head_dim, int64_t head_stride, int64_t row_stride, int rot_dims, float eps,
                            float w_offset, wzyb_stream_t stream) {
    const wzyb::HeadSection q{data, gamma, heads, head_stride, row_stride};
    const wzyb::HeadSection k{nullptr, nullptr, 0, 0, 0};
    return wzyb::launch_head_rope<__half>(q, k, cos_tab, sin_tab, table_rows, d_base_pos, pos_offset, T, head_dim,
                                          rot_dims, eps, w_offset, (cudaStream_t)stream);
}

int wzyb_head_norm_rope_f32(float* data, const float* gamma, const float* cos_tab, const float* sin_tab,
                            int64_t table_rows, const int32_t* d_base_pos, int64_t pos_offset, int64_t T, int heads,
                            int head_dim, int64_t head_stride, int64_t row_stride, int rot_dims, float eps,
                            float w_offset, wzyb_stream_t stream) {
    const wzyb::HeadSection q{data, gamma, heads, head_stride, row_stride};
    const wzyb::HeadSection k{nullptr, nullptr, 0, 0, 0};
    return wzyb::launch_head_rope<float>(q, k, cos_tab, sin_tab, table_rows, d_base_pos, pos_offset, T, head_dim,
                                         rot_dims, eps, w_offset, (cudaStream_t)stream);
}

int wzyb_qk_norm_rope_f16(const wzyb_head_tensor* q, const wzyb_head_tensor* k, const float* cos_tab,
                          const float* sin_tab, int64_t table_rows, const int32_t* d_base_pos, int64_t pos_offset,
                          int64_t T, int head_dim, int rot_dims, float eps, float w_offset, wzyb_stream_t stream) {
    if (q == nullptr) return WZYB_ERR_NULL;
    const wzyb::HeadSection qs{q->data, q->gamma, q->heads, q->head_stride, q->row_stride};
    wzyb::HeadSection ks{nullptr, nullptr, 0, 0, 0};
    if (k != nullptr && k->heads > 0) ks = wzyb::HeadSection{k->data, k->gamma, k->heads, k->head_stride, k->row_stride};
    return wzyb::launch_head_rope<__half>(qs, ks, cos_tab, sin_tab, table_rows, d_base_pos, pos_offset, T, head_dim,
                                          rot_dims, eps, w_offset, (cudaStream_t)stream);
}

int wzyb_rope_table_host_f32(float* h_cos, float* h_sin, int64_t rows, int rot_dims, double theta) {
    if (h_cos == nullptr || h_sin == nullptr) return WZYB_ERR_NULL;
    if (rows < 0 || rot_dims < 2 || (rot_dims % 2) != 0) return WZYB_ERR_SHAPE;
    const int half = rot_dims / 2;
    for (int i = 0; i < half; ++i) {
        const double inv = std::pow(theta, -2.0 * (double)i / (double)rot_dims);
        for (int64_t p = 0; p < rows; ++p) {
            const double ang = (double)p * inv;
            h_cos[p * half + i] = (float)std::cos(ang);
            h_sin[p * half + i] = (float)std::sin(ang);
        }
    }
    return WZYB_OK;
}

int wzyb_rope_table_f32(float* d_cos, float* d_sin, int64_t rows, int rot_dims, double theta, wzyb_stream_t stream) {
    if (d_cos == nullptr || d_sin == nullptr) return WZYB_ERR_NULL;
    if (rows < 0 || rot_dims < 2 || (rot_dims % 2) != 0) return WZYB_ERR_SHAPE;
    if (rows == 0) return WZYB_OK;
    wzyb::DeviceInfo di;
    const int rc = wzyb::device_info(&di);
    if (rc != WZYB_OK) return rc;
    const int half = rot_dims / 2;
    const int64_t n = rows * half;
    int64_t blocks = (n + 255) / 256;
    if (blocks > (int64_t)di.sms * 16) blocks = (int64_t)di.sms * 16;
    wzyb::launch_k(wzyb::rope_table_kernel, (int)blocks, 256, 0, (cudaStream_t)stream, d_cos, d_sin, rows, half, theta, rot_dims);
    return wzyb::launch_status();
}

}  // extern "C"
