// norm_rows.cu -- residual add + RMSNorm over rows, one HBM pass.
//
// Math follows fused_gr_norm_multi (src/wzy_kernels_v2.cuh:409-456) and its prefill twin
// pf_gr_norm_fp16 (src/wzy_qsa_wmma.cuh:197-232):
//   v = R + bo * gw          gw = 2*sigmoid(inj/hc) (exactly 1.0 for the single-stream add)
//   R <- v;  xn = (v * rsqrt(sum(v^2)/n + eps)) * g
// The reference runs one 256-thread block per (stream, token) row, reads R twice (the second pass
// re-reads it from cache) with scalar 4-byte accesses. Here every design reads each input once with
// 16-byte accesses and writes both outputs with 16-byte streaming stores:
//   direct (default while a row fits a warp's registers): a warp per row, all its vectors loaded
//          before any arithmetic, xor-shuffle reduction, no shared memory;
//   wide   (longer rows): a CTA per row, per-warp partial sums meeting behind one barrier; with 4
//          streams and bo_prev, a CTA per token (its 4 rows share one bo_prev read);
//   async  (on request): warp-owned rows staged in lane-private shared memory by cp.async;
#include "launch.hpp"

namespace wzyb {

struct NormRowsArgs {
    const void* x;     // bo_prev [T, n] (NULL: plain RMSNorm of res, res not written)
    void* res;         // R [T*hc, n]
    const void* w;     // gamma [hc, n]
    const float* inj;  // [T*hc] inject logits (NULL: gate 1.0)
    void* y;           // xn [T*hc, n]
    int64_t units;     // T * hc
    int n;
    int hc;
    float eps;
    float w_offset;
    void* qout;  // optional quantised xn (wide design only): codes in the QuantFormat of the launch
    void* sout;  // and its group scales
    float gs;    // NVFP4 per-tensor scale
    int lookahead;  // wide design with a quantised output: prefetch the CTA's next row into L2 (0/1)
    int sf_layout;  // block formats: kSfRowMajor or kSfTiled128x4 scale bytes
    int sf_ncb;     // tiled layout: 4-column scale tiles per 128-row band
};

// The quantised output of row u's 8 elements at e (every lane calls it; `e < n` lanes store).
template <int QF>
__device__ __forceinline__ void norm_quant_store(const NormRowsArgs& a, const float (&yo)[8], int64_t u, int e,
                                                 int lane) {
    const int n = a.n;
    if constexpr (QF == kQfMxfp8 || QF == kQfNvfp4) {
        if (a.sf_layout == kSfTiled128x4) {
            constexpr int kG = QF == kQfNvfp4 ? 16 : 32;
            block_group_store_at<QF>(yo, e < n, a.qout,
                                     static_cast<uint8_t*>(a.sout) + sf_tiled_offset(u, e / kG, a.sf_ncb), a.gs,
                                     (u * n + e) >> 3, lane);
            return;
        }
    }
    quant_group_store<QF>(yo, e < n, a.qout, a.sout, a.gs, (u * n + e) >> 3, lane);
}

// Direct design: one warp per row. Lane l owns the 8-element vectors l, l+32, ... of the row, so each
// warp-wide 16-byte load covers 512 contiguous bytes. All VPL vectors of residual and x are loaded
// before any arithmetic (VPL*2 loads in flight per lane); the sum of squares is reduced with five
// xor shuffles; v is recomputed from the raw registers in the second pass instead of being kept in
// fp32, which keeps a row of 2048 at ~100 registers. No shared memory, no CTA barrier.
// The body takes its CTA's index among `nctas` CTAs that share the rows, so a fused bundle kernel can
// run it on a subset of its grid.
template <typename TI, typename TO, int VPL>
__device__ __forceinline__ void norm_rows_direct_body(const NormRowsArgs& a, int cta, int nctas) {
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = (int64_t)nctas * (blockDim.x >> 5);
    const int64_t gwarp = (int64_t)cta * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const TI* __restrict__ x = static_cast<const TI*>(a.x);
    TI* __restrict__ res = static_cast<TI*>(a.res);
    const TI* __restrict__ w = static_cast<const TI*>(a.w);
    TO* __restrict__ y = static_cast<TO*>(a.y);
    const bool has_x = x != nullptr;
    const int n = a.n;
    // One weight row shared by every row (hc == 1): (w_offset + w) in fp32 once per CTA in shared
    // memory, so a row reads it with two 16-byte shared loads per vector instead of a global load,
    // eight conversions and four adds.
    __shared__ __align__(16) float wsm[VPL * 256];
    const bool wtab = a.hc == 1;
    if (wtab) {
        for (int e = threadIdx.x * 8; e < VPL * 256; e += blockDim.x * 8) {
            float2 g[4];
            if (e < n) {
                Vec8<TI>::load_ro2(w + e, g);
#pragma unroll
                for (int i = 0; i < 4; ++i) g[i] = fadd2(splat2(a.w_offset), g[i]);
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i) g[i] = splat2(0.f);
            }
            *reinterpret_cast<float4*>(wsm + e) = make_float4(g[0].x, g[0].y, g[1].x, g[1].y);
            *reinterpret_cast<float4*>(wsm + e + 4) = make_float4(g[2].x, g[2].y, g[3].x, g[3].y);
        }
        __syncthreads();
    }

    for (int64_t u = gwarp; u < a.units; u += nwarps) {
        typename Vec8<TI>::Raw rr[VPL], rx[VPL];
        const TI* rrow = res + u * n;
        const int64_t t = a.hc == 1 ? u : u / a.hc;  // token of this (token, stream) row
        const TI* xrow = has_x ? x + t * n : nullptr;
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            const int e = (k * 32 + lane) * 8;
            if (e < n) {
                rr[k] = Vec8<TI>::ldcs_raw(rrow + e);
                if (has_x) rx[k] = Vec8<TI>::ldcs_raw(xrow + e);
            }
        }
        const float2 gate = splat2((has_x && a.inj != nullptr) ? 2.0f / (1.0f + __expf(-a.inj[u] / (float)a.hc))
                                                                : 1.0f);
        // v = residual + x * gate (packed FFMA2, the same rounding as the reference's scalar fma); with
        // a unit gate and fp16 inputs, v = fp32(residual) + fp32(x) as one mixed-precision add per
        // element (add.rn.f32.f16: the fp16 operand widened exactly, one rounding -- the same bits)
        const bool unit_gate = !(has_x && a.inj != nullptr);
        auto residual_sum = [&](int k, float2 (&v)[4]) {
            if constexpr (sizeof(TI) == 2) {
                if (has_x && unit_gate) {
                    float2 xv[4];
                    Vec8<TI>::cvt2(rx[k], xv);
                    const uint32_t* rw = reinterpret_cast<const uint32_t*>(&rr[k]);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const unsigned short lo = (unsigned short)(rw[i] & 0xFFFFu), hi = (unsigned short)(rw[i] >> 16);
                        asm("add.rn.f32.f16 %0, %1, %2;" : "=f"(v[i].x) : "h"(lo), "f"(xv[i].x));
                        asm("add.rn.f32.f16 %0, %1, %2;" : "=f"(v[i].y) : "h"(hi), "f"(xv[i].y));
                    }
                    return;
                }
            }
            Vec8<TI>::cvt2(rr[k], v);
            if (has_x) {
                float2 xv[4];
                Vec8<TI>::cvt2(rx[k], xv);
#pragma unroll
                for (int i = 0; i < 4; ++i) v[i] = ffma2(xv[i], gate, v[i]);
            }
        };
        float ss = 0.f;
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            if ((k * 32 + lane) * 8 < n) {
                float2 v[4];
                residual_sum(k, v);
                ss += sumsq8(v);
            }
        }
        ss = group_sum<32>(ss);
        const float2 sc = splat2(rsqrt_approx(ss / (float)n + a.eps));
        const float2 woff = splat2(a.w_offset);
        const TI* wrow = w + (u - t * a.hc) * n;
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            const int e = (k * 32 + lane) * 8;
            if (e < n) {
                float2 v[4], g[4], o[4];
                residual_sum(k, v);
                if (wtab) {
                    const float4 g0 = *reinterpret_cast<const float4*>(wsm + e);
                    const float4 g1 = *reinterpret_cast<const float4*>(wsm + e + 4);
                    g[0] = make_float2(g0.x, g0.y);
                    g[1] = make_float2(g0.z, g0.w);
                    g[2] = make_float2(g1.x, g1.y);
                    g[3] = make_float2(g1.z, g1.w);
                } else {
                    Vec8<TI>::load_ro2(wrow + e, g);
#pragma unroll
                    for (int i = 0; i < 4; ++i) g[i] = fadd2(woff, g[i]);
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) o[i] = fmul2(fmul2(v[i], sc), g[i]);  // (v*sc)*g
                Vec8<TO>::store2(y + u * n + e, o);
                if (has_x) Vec8<TI>::store2(res + u * n + e, v);
            }
        }
    }
}

template <typename TI, typename TO, int VPL>
__global__ void __launch_bounds__(256, 2) norm_rows_direct_kernel(const NormRowsArgs a) {
    pdl_begin();
    norm_rows_direct_body<TI, TO, VPL>(a, blockIdx.x, gridDim.x);
}

// Async design: one warp per row as in the direct design, but the row's residual and x vectors are
// staged in a lane-private shared-memory slot by cp.async (each lane copies and later reads back only
// its own 16-byte chunks, so no barrier is needed) and read from there twice -- once for the sum of
// squares, once for the outputs. Registers stay low, so at layer-sized T every row of the call is in
// flight at once (kP = 1); kP = 2 double-buffers rows for long streams.
template <typename TI, typename TO, int VPL, int kP>
__global__ void __launch_bounds__(128) norm_rows_async_kernel(const NormRowsArgs a) {
    pdl_begin();
    constexpr int C = Vec8<TI>::kChunks;
    constexpr int SLOT = 2 * VPL * C * 32;  // uint4: residual vectors, then x vectors
    extern __shared__ __align__(16) uint4 sm_nr[];
    const int lane = threadIdx.x & 31;
    uint4* ring = sm_nr + (size_t)(threadIdx.x >> 5) * kP * SLOT;
    const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int64_t gwarp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const TI* __restrict__ x = static_cast<const TI*>(a.x);
    TI* __restrict__ res = static_cast<TI*>(a.res);
    const TI* __restrict__ w = static_cast<const TI*>(a.w);
    TO* __restrict__ y = static_cast<TO*>(a.y);
    const bool has_x = x != nullptr;
    const int n = a.n;

    auto issue = [&](int64_t u, int slot) {
        if (u < a.units) {
            const int64_t t = a.hc == 1 ? u : u / a.hc;
            uint4* sl = ring + slot * SLOT;
#pragma unroll
            for (int k = 0; k < VPL; ++k) {
                const int e = (k * 32 + lane) * 8;
                if (e < n) {
                    Vec8<TI>::stage_async(sl + k * C * 32, lane, res + u * n + e);
                    if (has_x) Vec8<TI>::stage_async(sl + (VPL + k) * C * 32, lane, x + t * n + e);
                }
            }
        }
        cp_async_commit();  // one group per row, empty or not
    };
#pragma unroll
    for (int j = 0; j < kP; ++j) issue(gwarp + j * nwarps, j);

    for (int64_t j = 0;; ++j) {
        const int64_t u = gwarp + j * nwarps;
        if (u >= a.units) break;  // warp-uniform
        const int slot = (int)(j % kP);
        const uint4* sl = ring + slot * SLOT;
        cp_async_wait<kP - 1>();
        const int64_t t = a.hc == 1 ? u : u / a.hc;
        const float2 gate = splat2((has_x && a.inj != nullptr) ? 2.0f / (1.0f + __expf(-a.inj[u] / (float)a.hc))
                                                                : 1.0f);
        auto residual_sum = [&](int k, float2 (&v)[4]) {  // v = residual + x * gate, from the slot
            Vec8<TI>::unstage2(sl + k * C * 32, lane, v);
            if (has_x) {
                float2 xv[4];
                Vec8<TI>::unstage2(sl + (VPL + k) * C * 32, lane, xv);
#pragma unroll
                for (int i = 0; i < 4; ++i) v[i] = ffma2(xv[i], gate, v[i]);
            }
        };
        float ss = 0.f;
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            if ((k * 32 + lane) * 8 < n) {
                float2 v[4];
                residual_sum(k, v);
                ss += sumsq8(v);
            }
        }
        ss = group_sum<32>(ss);
        const float2 sc = splat2(rsqrt_approx(ss / (float)n + a.eps));
        const float2 woff = splat2(a.w_offset);
        const TI* wrow = w + (u - t * a.hc) * n;
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            const int e = (k * 32 + lane) * 8;
            float2 o[4] = {};
            if (e < n) {
                float2 v[4], g[4];
                residual_sum(k, v);
                Vec8<TI>::load_ro2(wrow + e, g);
#pragma unroll
                for (int i = 0; i < 4; ++i) o[i] = fmul2(fmul2(v[i], sc), fadd2(woff, g[i]));  // (v*sc)*g
                Vec8<TO>::store2(y + u * n + e, o);
                if (has_x) Vec8<TI>::store2(res + u * n + e, v);
            }
        }
        // Refill the slot: only this lane touches its chunks, and its reads precede the new copy.
        issue(u + kP * nwarps, slot);
    }
    cp_async_wait<0>();
}

// Wide design, for rows past one warp's register budget (fp32 rows past 1536, fp16 past 3072 -- the
// reference model's 2560-wide fp32 streams among them): a CTA of NW = blockDim/32 warps (4, 8 or 16)
// owns one row at a time. Thread i of the CTA holds the 8-element vectors k*blockDim + i (k < VPL),
// so each warp-wide load still covers 512 contiguous bytes and every 32-element group sits in 4
// consecutive lanes of one warp (the quantised side output -- Q8_0, MXFP8 or NVFP4 -- takes its
// group max with one or two shuffles). The warps'
// partial sums of squares meet in shared memory behind ONE barrier per row: the partials are
// double-buffered by row parity, and a warp can only come back to a slot after passing the next
// row's barrier, which the slowest warp reaches only once it has read the slot. Rows are spread
// over a persistent grid; several CTAs per SM keep rows in flight across the barriers.
template <typename TI, typename TO, int VPL, int QF>
__global__ void __launch_bounds__(512) norm_rows_wide_kernel(const NormRowsArgs a) {
    pdl_begin();
    __shared__ float part[2][16];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int nw = blockDim.x >> 5;
    const int span = blockDim.x * 8;
    const TI* __restrict__ x = static_cast<const TI*>(a.x);
    TI* __restrict__ res = static_cast<TI*>(a.res);
    const TI* __restrict__ w = static_cast<const TI*>(a.w);
    TO* __restrict__ y = static_cast<TO*>(a.y);
    const bool has_x = x != nullptr;
    const int n = a.n;
    int par = 0;

    for (int64_t u = blockIdx.x; u < a.units; u += gridDim.x, par ^= 1) {
        typename Vec8<TI>::Raw rr[VPL], rx[VPL];
        const int64_t t = a.hc == 1 ? u : u / a.hc;
        const TI* rrow = res + u * n;
        const TI* xrow = has_x ? x + t * n : nullptr;
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            const int e = k * span + threadIdx.x * 8;
            if (e < n) {
                rr[k] = Vec8<TI>::ldcs_raw(rrow + e);
                if (has_x) rx[k] = Vec8<TI>::ldcs_raw(xrow + e);
            }
        }
        if (QF != kQfNone && a.lookahead && u + gridDim.x < a.units) {  // the CTA's next row, into L2
            const int64_t un = u + gridDim.x;
            const int64_t tn = a.hc == 1 ? un : un / a.hc;
#pragma unroll
            for (int k = 0; k < VPL; ++k) {
                const int e = k * span + threadIdx.x * 8;
                if (e < n) {
                    prefetch_l2(res + un * n + e);
                    if (has_x && tn != t) prefetch_l2(x + tn * n + e);
                }
            }
        }
        const float2 gate = splat2((has_x && a.inj != nullptr) ? 2.0f / (1.0f + __expf(-a.inj[u] / (float)a.hc))
                                                                : 1.0f);
        auto residual_sum = [&](int k, float2 (&v)[4]) {  // v = residual + x * gate
            Vec8<TI>::cvt2(rr[k], v);
            if (has_x) {
                float2 xv[4];
                Vec8<TI>::cvt2(rx[k], xv);
#pragma unroll
                for (int i = 0; i < 4; ++i) v[i] = ffma2(xv[i], gate, v[i]);
            }
        };
        float ss = 0.f;
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            if (k * span + threadIdx.x * 8 < n) {
                float2 v[4];
                residual_sum(k, v);
                ss += sumsq8(v);
            }
        }
        ss = group_sum<32>(ss);
        if (lane == 0) part[par][warp] = ss;
        __syncthreads();
        float tot = 0.f;
        for (int i = 0; i < nw; ++i) tot += part[par][i];  // same order in every thread
        const float2 sc = splat2(rsqrt_approx(tot / (float)n + a.eps));
        const float2 woff = splat2(a.w_offset);
        const TI* wrow = w + (u - t * a.hc) * n;
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            const int e = k * span + threadIdx.x * 8;
            float2 o[4] = {};
            if (e < n) {
                float2 v[4], g[4];
                residual_sum(k, v);
                Vec8<TI>::load_ro2(wrow + e, g);
#pragma unroll
                for (int i = 0; i < 4; ++i) o[i] = fmul2(fmul2(v[i], sc), fadd2(woff, g[i]));  // (v*sc)*g
                Vec8<TO>::store2(y + u * n + e, o);
                if (has_x) Vec8<TI>::store2(res + u * n + e, v);
            }
            if (QF != kQfNone) {  // every lane: the group max is a shuffle
                const float yo[8] = {o[0].x, o[0].y, o[1].x, o[1].y, o[2].x, o[2].y, o[3].x, o[3].y};
                norm_quant_store<QF>(a, yo, u, e, lane);
            }
        }
    }
}

// Token design for 4-stream rows (hc = 4, the reference model's hyper-connection width, with bo_prev):
// a CTA owns a token -- its 4 (token, stream) rows and the one bo_prev row they share. Thread i holds
// vectors k * blockDim + i of bo_prev and of the 4 rows; the 4 partial sums of squares meet in shared
// memory behind ONE barrier per token (double-buffered by token parity, as in the wide design), then
// each row is scaled and written. Against the row-per-CTA wide design, bo_prev is read once per token
// instead of once per row, there is one barrier per 4 rows, and each CTA has 4 rows in flight. The
// arithmetic per element is the wide design's; only the order of the cross-warp partial sums follows
// this CTA's warp count.
// Register caps: unbounded, the compiler hoists all 4 streams' gamma loads and takes 118 registers,
// which leaves one 320-thread CTA per SM. One vector per thread fits 72 with no spill (2 CTAs of 320:
// 79 -> 82 % of HBM peak at 4096 tokens x 4 x 2560 against the wide design); with a quantised output
// 64 and a 32-60 byte spill (3 CTAs: 82 -> 83.5 %, where the 72 cap gives 79 %).
template <typename TI, typename TO, int VPL, int QF>
__global__ void __maxnreg__(VPL == 1 ? (QF == kQfNone ? 72 : 64) : 128) norm_rows_token4_kernel(const NormRowsArgs a) {
    pdl_begin();
    constexpr int HC = 4;
    __shared__ float part[2][HC][16];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int nw = blockDim.x >> 5;
    const int span = blockDim.x * 8;
    const TI* __restrict__ x = static_cast<const TI*>(a.x);
    TI* __restrict__ res = static_cast<TI*>(a.res);
    const TI* __restrict__ w = static_cast<const TI*>(a.w);
    TO* __restrict__ y = static_cast<TO*>(a.y);
    const int n = a.n;
    const int64_t T = a.units / HC;
    int par = 0;

    for (int64_t t = blockIdx.x; t < T; t += gridDim.x, par ^= 1) {
        typename Vec8<TI>::Raw rr[HC][VPL], rx[VPL];
        const int64_t u0 = t * HC;
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            const int e = k * span + threadIdx.x * 8;
            if (e < n) {
                rx[k] = Vec8<TI>::ldcs_raw(x + t * n + e);
#pragma unroll
                for (int c = 0; c < HC; ++c) rr[c][k] = Vec8<TI>::ldcs_raw(res + (u0 + c) * n + e);
            }
        }
        float gate[HC];
#pragma unroll
        for (int c = 0; c < HC; ++c) gate[c] = a.inj != nullptr ? 2.0f / (1.0f + __expf(-a.inj[u0 + c] / (float)HC)) : 1.0f;
        auto residual_sum = [&](int c, int k, float2 (&v)[4]) {  // v = residual + x * gate
            Vec8<TI>::cvt2(rr[c][k], v);
            float2 xv[4];
            Vec8<TI>::cvt2(rx[k], xv);
#pragma unroll
            for (int i = 0; i < 4; ++i) v[i] = ffma2(xv[i], splat2(gate[c]), v[i]);
        };
#pragma unroll
        for (int c = 0; c < HC; ++c) {
            float ss = 0.f;
#pragma unroll
            for (int k = 0; k < VPL; ++k) {
                if (k * span + threadIdx.x * 8 < n) {
                    float2 v[4];
                    residual_sum(c, k, v);
                    ss += sumsq8(v);
                }
            }
            ss = group_sum<32>(ss);
            if (lane == 0) part[par][c][warp] = ss;
        }
        __syncthreads();
        const float2 woff = splat2(a.w_offset);
#pragma unroll
        for (int c = 0; c < HC; ++c) {
            float tot = 0.f;
            for (int i = 0; i < nw; ++i) tot += part[par][c][i];  // same order in every thread
            const float2 sc = splat2(rsqrt_approx(tot / (float)n + a.eps));
            const int64_t u = u0 + c;
#pragma unroll
            for (int k = 0; k < VPL; ++k) {
                const int e = k * span + threadIdx.x * 8;
                float2 o[4] = {};
                if (e < n) {
                    float2 v[4], g[4];
                    residual_sum(c, k, v);
                    Vec8<TI>::load_ro2(w + c * n + e, g);
#pragma unroll
                    for (int i = 0; i < 4; ++i) o[i] = fmul2(fmul2(v[i], sc), fadd2(woff, g[i]));  // (v*sc)*g
                    Vec8<TO>::store2(y + u * n + e, o);
                    Vec8<TI>::store2(res + u * n + e, v);
                }
                if (QF != kQfNone) {  // every lane: the group max is a shuffle
                    const float yo[8] = {o[0].x, o[0].y, o[1].x, o[1].y, o[2].x, o[2].y, o[3].x, o[3].y};
                    norm_quant_store<QF>(a, yo, u, e, lane);
                }
            }
        }
    }
}

// Shape of the token design for a row of `vecs` vectors: VPL vectors per thread (1 or 2; 0 = the
// design does not apply) over the fewest warps that hold the row.
static void token4_shape(int vecs, int& nw, int& vpl) {
    vpl = vecs <= 512 ? 1 : vecs <= 1024 ? 2 : 0;
    nw = vpl ? (vecs + 32 * vpl - 1) / (32 * vpl) : 0;
}

template <typename TI, typename TO, int QF>
static int launch_norm_rows_token4(const NormRowsArgs& a, int nw, int vpl, const DeviceInfo& di,
                                   cudaStream_t stream) {
    const int threads = nw * 32;
    const void* kern = vpl == 1 ? (const void*)norm_rows_token4_kernel<TI, TO, 1, QF>
                                : (const void*)norm_rows_token4_kernel<TI, TO, 2, QF>;
    const int grid = persistent_grid(di, resident_ctas(kern, threads, 0), a.units / 4);
    if (vpl == 1) launch_k(norm_rows_token4_kernel<TI, TO, 1, QF>, grid, threads, 0, stream, a);
    else launch_k(norm_rows_token4_kernel<TI, TO, 2, QF>, grid, threads, 0, stream, a);
    return launch_status();
}

// Warps per CTA and vectors per thread of the wide design for a row of `vecs` 8-element vectors:
// the fewest warps (4, 8, 16) that keep VPL within the register budget, VPL rounded up to an
// instantiated count.
template <typename TI>
static void wide_shape(int vecs, int& nw, int& vpl) {
    const int vmax = sizeof(TI) == 2 ? 8 : 4;
    nw = 4;
    while (nw < 16 && (vecs + nw * 32 - 1) / (nw * 32) > vmax) nw *= 2;
    const int need = (vecs + nw * 32 - 1) / (nw * 32);
    vpl = need <= 1 ? 1 : need <= 2 ? 2 : need <= 3 ? 3 : need <= 4 ? 4 : need <= 6 ? 6 : 8;
}

template <typename TI, typename TO, int QF>
static int launch_norm_rows_wide(const NormRowsArgs& a, const DeviceInfo& di, cudaStream_t stream) {
    int nw = 0, vpl = 0;
    if constexpr (sizeof(TI) == 4) {
        // 4 streams sharing a bo_prev row: the token design (fp32 rows, up to 8192 wide), for calls of
        // at least 4 tokens per SM. Shorter calls (decode) keep a CTA per row: 4x the CTAs, and a
        // 1-token call takes 3.2 us there against 6.4 us with its 4 rows in one CTA.
        if (a.hc == 4 && a.x != nullptr && variant(kFamNorm) != WZYB_VARIANT_WIDE &&
            a.units / 4 >= (int64_t)di.sms * 4) {
            token4_shape(a.n / 8, nw, vpl);
            if (vpl) return launch_norm_rows_token4<TI, TO, QF>(a, nw, vpl, di, stream);
        }
    }
    wide_shape<TI>(a.n / 8, nw, vpl);
    const int threads = nw * 32;
    const void* kern = nullptr;
#define WZYB_NRW(V) \
    if (vpl == V) kern = (const void*)norm_rows_wide_kernel<TI, TO, V, QF>;
    WZYB_NRW(1) WZYB_NRW(2) WZYB_NRW(3) WZYB_NRW(4)
    if constexpr (sizeof(TI) == 2) { WZYB_NRW(6) WZYB_NRW(8) }
#undef WZYB_NRW
    if (kern == nullptr) return WZYB_ERR_SHAPE;
    const int grid = persistent_grid(di, resident_ctas(kern, threads, 0), a.units);
#define WZYB_NRW(V) \
    if (vpl == V) launch_k(norm_rows_wide_kernel<TI, TO, V, QF>, grid, threads, 0, stream, a);
    WZYB_NRW(1) WZYB_NRW(2) WZYB_NRW(3) WZYB_NRW(4)
    if constexpr (sizeof(TI) == 2) { WZYB_NRW(6) WZYB_NRW(8) }
#undef WZYB_NRW
    return launch_status();
}

// Validates a row-norm call on the host and fills `a` (every field but the launch shape's). Returns
// WZYB_OK or the WZYB_ERR_* of the first bad argument; nothing is enqueued.
template <typename TI>
static int norm_rows_prepare(const void* x, void* res, const void* w, const float* inj, void* y, int64_t T, int n,
                             int hc, float eps, float w_offset, NormRowsArgs& a) {
    if (res == nullptr || w == nullptr || y == nullptr) return WZYB_ERR_NULL;
    if (T < 0 || T > (int64_t(1) << 40) || n < 8 || n > 16384 || (n % 8) != 0 || hc < 1 || hc > 64)
        return WZYB_ERR_SHAPE;
    if (!aligned16(res) || !aligned16(w) || !aligned16(y) || (x && !aligned16(x))) return WZYB_ERR_ALIGN;
    a.x = x;
    a.res = res;
    a.w = w;
    a.inj = x ? inj : nullptr;
    a.y = y;
    a.units = T * hc;
    a.n = n;
    a.hc = hc;
    a.eps = eps;
    a.w_offset = w_offset;
    a.qout = a.sout = nullptr;
    a.gs = 1.0f;
    a.sf_layout = kSfRowMajor;
    a.sf_ncb = 0;
    a.lookahead = 0;  // without a quantised output it did not pay (76 vs 76 % at 4096 x 4 x 2560)
    return WZYB_OK;
}

template <typename TI, typename TO>
static int launch_norm_rows(const void* x, void* res, const void* w, const float* inj, void* y, int64_t T, int n,
                            int hc, float eps, float w_offset, cudaStream_t stream) {
    NormRowsArgs a;
    int rc = norm_rows_prepare<TI>(x, res, w, inj, y, T, n, hc, eps, w_offset, a);
    if (rc != WZYB_OK || T == 0) return rc;
    DeviceInfo di;
    rc = device_info(&di);
    if (rc != WZYB_OK) return rc;

    // Direct design while a row fits one warp's register budget (<= 12 fp16 or 4 fp32 vectors per
    // lane), the wide design (CTA-owned rows) past it.
    const int vpl_need = (n + 255) / 256;
    const int vpl_max = sizeof(TI) == 2 ? 12 : 4;
    const int var = variant(kFamNorm);
    if (var == WZYB_VARIANT_WIDE || vpl_need > vpl_max)
        return launch_norm_rows_wide<TI, TO, kQfNone>(a, di, stream);
    if (var == WZYB_VARIANT_ASYNC && vpl_need <= (sizeof(TI) == 2 ? 8 : 4)) {
        const int vpl = vpl_need <= 1 ? 1 : vpl_need <= 2 ? 2 : vpl_need <= 4 ? 4 : 8;
        // one row in flight per warp when every row of the call fits in one round, else two
        const int64_t one_round = (int64_t)di.sms * 28;
        const int kp = a.units <= one_round ? 1 : 2;
        const int smem = 4 * kp * 2 * vpl * Vec8<TI>::kChunks * 32 * 16;
        const void* kern = nullptr;
#define WZYB_NRA(V, P) \
    if (vpl == V && kp == P) kern = (const void*)norm_rows_async_kernel<TI, TO, V, P>;
        WZYB_NRA(1, 1) WZYB_NRA(1, 2) WZYB_NRA(2, 1) WZYB_NRA(2, 2)
        WZYB_NRA(4, 1) WZYB_NRA(4, 2) WZYB_NRA(8, 1) WZYB_NRA(8, 2)
#undef WZYB_NRA
        rc = ensure_smem(kern, smem);
        if (rc != WZYB_OK) return rc;
        const int grid = persistent_grid(di, resident_ctas(kern, 128, smem), (a.units + 3) / 4);
#define WZYB_NRA(V, P) \
    if (vpl == V && kp == P) launch_k(norm_rows_async_kernel<TI, TO, V, P>, grid, 128, smem, stream, a);
        WZYB_NRA(1, 1) WZYB_NRA(1, 2) WZYB_NRA(2, 1) WZYB_NRA(2, 2)
        WZYB_NRA(4, 1) WZYB_NRA(4, 2) WZYB_NRA(8, 1) WZYB_NRA(8, 2)
#undef WZYB_NRA
        return launch_status();
    }
    {
        const void* kern = nullptr;
        int vpl = 0;
#define WZYB_NR_PICK(V)                                                  \
    if (!kern && vpl_need <= V) {                                        \
        kern = (const void*)norm_rows_direct_kernel<TI, TO, V>;          \
        vpl = V;                                                         \
    }
        WZYB_NR_PICK(1)
        WZYB_NR_PICK(2)
        WZYB_NR_PICK(4)
        if constexpr (sizeof(TI) == 2) {
            WZYB_NR_PICK(6)
            WZYB_NR_PICK(8)
            WZYB_NR_PICK(10)
            WZYB_NR_PICK(12)
        }
#undef WZYB_NR_PICK
        const int grid = persistent_grid(di, resident_ctas(kern, 256, 0), (a.units + 7) / 8);
        switch (vpl) {
            case 1: launch_k(norm_rows_direct_kernel<TI, TO, 1>, grid, 256, 0, stream, a); break;
            case 2: launch_k(norm_rows_direct_kernel<TI, TO, 2>, grid, 256, 0, stream, a); break;
            case 4: launch_k(norm_rows_direct_kernel<TI, TO, 4>, grid, 256, 0, stream, a); break;
            default:
                // 6-12 vectors per lane only for fp16 rows (fp32 rows that long take the wide design)
                if constexpr (sizeof(TI) == 2) {
                    if (vpl == 6) launch_k(norm_rows_direct_kernel<TI, TO, 6>, grid, 256, 0, stream, a);
                    else if (vpl == 8) launch_k(norm_rows_direct_kernel<TI, TO, 8>, grid, 256, 0, stream, a);
                    else if (vpl == 10) launch_k(norm_rows_direct_kernel<TI, TO, 10>, grid, 256, 0, stream, a);
                    else launch_k(norm_rows_direct_kernel<TI, TO, 12>, grid, 256, 0, stream, a);
                }
                break;
        }
        return launch_status();
    }

    return WZYB_ERR_SHAPE;  // not reached: every row width has the direct or the wide design
}

// Residual fold + norm with a quantised side output of xn (format QF: Q8_0, MXFP8 or NVFP4): the
// wide design at every width (n <= 16384; n % 32 == 0, the largest group).
template <typename TI, typename TO, int QF>
static int launch_norm_rows_quant(const void* x, void* res, const void* w, const float* inj, void* y, void* qout,
                                  void* sout, float gs, int64_t T, int n, int hc, float eps, cudaStream_t stream,
                                  int sf_layout = kSfRowMajor) {
    if (res == nullptr || w == nullptr || y == nullptr || qout == nullptr || sout == nullptr) return WZYB_ERR_NULL;
    if (sf_layout != kSfRowMajor && (QF == kQfQ8 || sf_layout != kSfTiled128x4)) return WZYB_ERR_VALUE;
    if (T < 0 || T > (int64_t(1) << 40) || n < 32 || n > 16384 || (n % 32) != 0 || hc < 1 || hc > 64)
        return WZYB_ERR_SHAPE;
    if (!aligned16(res) || !aligned16(w) || !aligned16(y) || (x && !aligned16(x)) || !aligned16(qout) ||
        (QF == kQfQ8 ? !aligned16(sout) : false))
        return WZYB_ERR_ALIGN;
    if (T == 0) return WZYB_OK;
    DeviceInfo di;
    int rc = device_info(&di);
    if (rc != WZYB_OK) return rc;
    NormRowsArgs a;
    a.x = x;
    a.res = res;
    a.w = w;
    a.inj = x ? inj : nullptr;
    a.y = y;
    a.units = T * hc;
    a.n = n;
    a.hc = hc;
    a.eps = eps;
    a.w_offset = 0.0f;
    a.qout = qout;
    a.sout = sout;
    a.gs = gs;
    a.sf_layout = sf_layout;
    a.sf_ncb = (n / (QF == kQfNvfp4 ? 16 : 32) + 3) / 4;
    // on by default for the quantising rows (76 -> 80 % of peak at 4096 x 4 x 2560): the group
    // quantiser's epilogue is long enough that the next row's reads are worth starting under it
    a.lookahead = tuning(kFamNorm).stages == 1 ? 0 : 1;
    return launch_norm_rows_wide<TI, TO, QF>(a, di, stream);
}

}  // namespace wzyb

extern "C" {

int wzyb_gr_norm_q8_f32(float* R, const float* w_norm, const float* bo_prev, const float* inj_prev, float* xn,
                        int8_t* xq8, float* xs8, int64_t T, int n_embd, int hc, float eps, wzyb_stream_t stream) {
    return wzyb::launch_norm_rows_quant<float, float, wzyb::kQfQ8>(bo_prev, R, w_norm, inj_prev, xn, xq8, xs8, 1.0f, T,
                                                                 n_embd, hc, eps, (cudaStream_t)stream);
}

int wzyb_gr_norm_mxfp8_f32(float* R, const float* w_norm, const float* bo_prev, const float* inj_prev, float* xn,
                           uint8_t* xq, uint8_t* xs, int64_t T, int n_embd, int hc, float eps, wzyb_stream_t stream) {
    return wzyb::launch_norm_rows_quant<float, float, wzyb::kQfMxfp8>(bo_prev, R, w_norm, inj_prev, xn, xq, xs, 1.0f,
                                                                    T, n_embd, hc, eps, (cudaStream_t)stream);
}

int wzyb_gr_norm_nvfp4_f32(float* R, const float* w_norm, const float* bo_prev, const float* inj_prev, float* xn,
                           uint8_t* xq, uint8_t* xs, float global_scale, int64_t T, int n_embd, int hc, float eps,
                           wzyb_stream_t stream) {
    return wzyb::launch_norm_rows_quant<float, float, wzyb::kQfNvfp4>(bo_prev, R, w_norm, inj_prev, xn, xq, xs,
                                                                    global_scale, T, n_embd, hc, eps,
                                                                    (cudaStream_t)stream);
}

int wzyb_gr_norm_block_f32(float* R, const float* w_norm, const float* bo_prev, const float* inj_prev, float* xn,
                           uint8_t* xq, uint8_t* xs, int format, int sf_layout, float global_scale, int64_t T,
                           int n_embd, int hc, float eps, wzyb_stream_t stream) {
    if (format == WZYB_BLOCK_MXFP8)
        return wzyb::launch_norm_rows_quant<float, float, wzyb::kQfMxfp8>(bo_prev, R, w_norm, inj_prev, xn, xq, xs, 1.0f,
                                                                        T, n_embd, hc, eps, (cudaStream_t)stream,
                                                                        sf_layout);
    if (format == WZYB_BLOCK_NVFP4)
        return wzyb::launch_norm_rows_quant<float, float, wzyb::kQfNvfp4>(bo_prev, R, w_norm, inj_prev, xn, xq, xs,
                                                                        global_scale, T, n_embd, hc, eps,
                                                                        (cudaStream_t)stream, sf_layout);
    return WZYB_ERR_VALUE;
}

int wzyb_add_rmsnorm_f16(const uint16_t* x, uint16_t* residual, const uint16_t* weight, uint16_t* y, int64_t T,
                         int hidden, float eps, float w_offset, wzyb_stream_t stream) {
    return wzyb::launch_norm_rows<__half, __half>(x, residual, weight, nullptr, y, T, hidden, 1, eps, w_offset,
                                                  (cudaStream_t)stream);
}

int wzyb_gr_norm_f32(float* R, const float* w_norm, const float* bo_prev, const float* inj_prev, float* xn,
                     int64_t T, int n_embd, int hc, float eps, wzyb_stream_t stream) {
    return wzyb::launch_norm_rows<float, float>(bo_prev, R, w_norm, inj_prev, xn, T, n_embd, hc, eps, 0.0f,
                                                (cudaStream_t)stream);
}

int wzyb_gr_norm_f32_f16(float* R, const float* w_norm, const float* bo_prev, const float* inj_prev, uint16_t* xn,
                         int64_t T, int n_embd, int hc, float eps, wzyb_stream_t stream) {
    return wzyb::launch_norm_rows<float, __half>(bo_prev, R, w_norm, inj_prev, xn, T, n_embd, hc, eps, 0.0f,
                                                 (cudaStream_t)stream);
}

}  // extern "C"
