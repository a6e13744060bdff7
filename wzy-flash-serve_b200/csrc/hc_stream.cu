// hc_stream.cu -- the multi-stream (hyper-connection) residual around the mixing GEMMs.
//
//   gr_write    R[t,c,:] += blk[t,:] * gw[t,c],  gw = 2*sigmoid(inj[t,c]/hc)   (1.0 without inj)
//               gr_write_multi, src/wzy_kernels_v2.cuh:813-828
//   hc_mix      mixed[t,:] = (1/hc) * sum_c xn[t,c,:] * sigmoid(gg[t,c,:])
//               pf_gr_up_mean_fp16, src/wzy_qsa_wmma.cuh:234-253 (fp16 in; fp32 and/or fp16 out)
//               gr_up_gate_mean_pf_kernel, src/wzy_prefill_tc.cuh:37-51 (fp32 in and out)
//   silu_scale  lo16 = silu(lo * scale) rounded to fp16
//               silu_div_hc_to_fp16_kernel, src/wzy_prefill_tc.cuh:24-35
//
// All three are one HBM pass. The reference runs them one scalar element per thread (gr_write on a
// fixed 80-block grid per token, with a 32-bit division per element); here every thread moves
// 16-byte vectors and the per-row gate is computed once per warp.
#include "launch.hpp"
#include "common.cuh"

namespace wzyb {

// --- gr_write ------------------------------------------------------------------------------------
// One warp per (token, stream) row of n floats; the block row blk[t] is read by hc warps and stays in
// L2 between them. R = fma(blk, gw, R), the rounding of the reference's `R += blk * gw`.
constexpr int kGrwThreads = 256;
constexpr int kGrwUnroll = 4;

__global__ void __launch_bounds__(kGrwThreads) gr_write_kernel(float* __restrict__ R, const float* __restrict__ blk,
                                                              const float* __restrict__ inj, int64_t rows, int n,
                                                              int hc) {
    pdl_begin();
    const int lane = threadIdx.x & 31;
    const int vpr = n >> 3;
    const int64_t nwarps = (int64_t)gridDim.x * (kGrwThreads / 32);
    for (int64_t u = (int64_t)blockIdx.x * (kGrwThreads / 32) + (threadIdx.x >> 5); u < rows; u += nwarps) {
        const float2 gw = splat2(inj != nullptr ? 2.0f / (1.0f + __expf(-inj[u] / (float)hc)) : 1.0f);
        float* r = R + u * n;
        const float* b = blk + (u / hc) * n;
        int j = lane;
        for (; j + (kGrwUnroll - 1) * 32 < vpr; j += kGrwUnroll * 32) {
            float2 rv[kGrwUnroll][4], bv[kGrwUnroll][4];
#pragma unroll
            for (int k = 0; k < kGrwUnroll; ++k) {
                Vec8<float>::load2(r + (j + k * 32) * 8, rv[k]);
                Vec8<float>::load_ro2(b + (j + k * 32) * 8, bv[k]);
            }
#pragma unroll
            for (int k = 0; k < kGrwUnroll; ++k) {
#pragma unroll
                for (int i = 0; i < 4; ++i) rv[k][i] = ffma2(bv[k][i], gw, rv[k][i]);
                Vec8<float>::store2(r + (j + k * 32) * 8, rv[k]);
            }
        }
        for (; j < vpr; j += 32) {
            float2 rv[4], bv[4];
            Vec8<float>::load2(r + j * 8, rv);
            Vec8<float>::load_ro2(b + j * 8, bv);
#pragma unroll
            for (int i = 0; i < 4; ++i) rv[i] = ffma2(bv[i], gw, rv[i]);
            Vec8<float>::store2(r + j * 8, rv);
        }
    }
}

// Decode-sized calls (a few rows: T <= 8 tokens x hc streams): one 8-element vector per thread over
// the whole call, so every load is in flight at once instead of a warp walking its row; each thread
// computes its row's gate (same expression).
__global__ void __launch_bounds__(kGrwThreads) gr_write_flat_kernel(float* __restrict__ R,
                                                                   const float* __restrict__ blk,
                                                                   const float* __restrict__ inj, int64_t nvec,
                                                                   int vpr, int hc) {
    pdl_begin();
    const int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (v >= nvec) return;
    const int64_t u = v / vpr;
    const int64_t col = (v - u * vpr) * 8;
    const int64_t n = (int64_t)vpr * 8;
    float2 rv[4], bv[4];
    Vec8<float>::load2(R + u * n + col, rv);
    Vec8<float>::load_ro2(blk + (u / hc) * n + col, bv);
    const float2 gw = splat2(inj != nullptr ? 2.0f / (1.0f + __expf(-inj[u] / (float)hc)) : 1.0f);
#pragma unroll
    for (int i = 0; i < 4; ++i) rv[i] = ffma2(bv[i], gw, rv[i]);
    Vec8<float>::store2(R + u * n + col, rv);
}

// --- hc_mix --------------------------------------------------------------------------------------
// Grid-stride over output vectors (token, 8 columns); each reads the hc stream vectors of xn and gg
// at that position. Streams are summed in order c = 0..hc-1, then scaled by 1/hc (0.25 for the
// reference's 4 streams, exact), as the reference does. The sigmoid uses the base-2 exponential and
// reciprocal approximations (sigmoid2, common.cuh).
constexpr int kMixThreads = 256;

// kHC > 0: the stream count is a compile-time constant and all 2*kHC loads of a vector are issued
// before its math (the reference's 4 streams); kHC == 0: any hc, one stream at a time.
template <typename TI, int kHC>
__global__ void __launch_bounds__(kMixThreads) hc_mix_kernel(const TI* __restrict__ xn, const TI* __restrict__ gg,
                                                            float* __restrict__ mixed, __half* __restrict__ mixed16,
                                                            int64_t nvec, int vpr, int hc_rt, float inv_hc) {
    pdl_begin();
    const int hc = kHC > 0 ? kHC : hc_rt;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t v0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    StridePos p(v0, stride, vpr);
    const int64_t n = (int64_t)vpr * 8;
    for (int64_t v = v0; v < nvec; v += stride, p.advance()) {
        const int64_t base = p.q * hc * n + (int64_t)p.r * 8;
        float2 acc[4] = {};
        if (kHC > 0) {
            typename Vec8<TI>::Raw xr[kHC > 0 ? kHC : 1], gr[kHC > 0 ? kHC : 1];
#pragma unroll
            for (int c = 0; c < kHC; ++c) {
                xr[c] = Vec8<TI>::ldcs_raw(xn + base + c * n);
                gr[c] = Vec8<TI>::ldcs_raw(gg + base + c * n);
            }
#pragma unroll
            for (int c = 0; c < kHC; ++c) {
                float2 x[4], g[4];
                Vec8<TI>::cvt2(xr[c], x);
                Vec8<TI>::cvt2(gr[c], g);
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[i] = ffma2(x[i], sigmoid2(g[i]), acc[i]);
            }
        } else {
            for (int c = 0; c < hc; ++c) {
                float2 x[4], g[4];
                Vec8<TI>::cvt2(Vec8<TI>::ldcs_raw(xn + base + c * n), x);
                Vec8<TI>::cvt2(Vec8<TI>::ldcs_raw(gg + base + c * n), g);
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[i] = ffma2(x[i], sigmoid2(g[i]), acc[i]);
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[i] = fmul2(acc[i], splat2(inv_hc));
        if (mixed != nullptr) Vec8<float>::store2(mixed + v * 8, acc);
        if (mixed16 != nullptr) Vec8<__half>::store2(mixed16 + v * 8, acc);
    }
}

// --- silu_scale ----------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) silu_scale_kernel(const float* __restrict__ lo, __half* __restrict__ out,
                                                         int64_t nvec, float scale) {
    pdl_begin();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nvec; v += stride) {
        float2 x[4];
        Vec8<float>::cvt2(Vec8<float>::ldcs_raw(lo + v * 8), x);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            x[i] = fmul2(x[i], splat2(scale));
            x[i] = fmul2(x[i], sigmoid2(x[i]));
        }
        Vec8<__half>::store2(out + v * 8, x);
    }
}

static int check_hc_shape(int64_t T, int n, int hc) {
    if (T < 0 || T > (int64_t(1) << 40) || n < 8 || (n % 8) != 0 || hc < 1 || hc > 64) return WZYB_ERR_SHAPE;
    return WZYB_OK;
}

template <typename TI>
static int launch_hc_mix(const TI* xn, const TI* gg, float* mixed, __half* mixed16, int64_t T, int n, int hc,
                         cudaStream_t stream) {
    if (!xn || !gg || (!mixed && !mixed16)) return WZYB_ERR_NULL;
    int rc = check_hc_shape(T, n, hc);
    if (rc != WZYB_OK) return rc;
    if (!aligned16(xn) || !aligned16(gg) || (mixed && !aligned16(mixed)) || (mixed16 && !aligned16(mixed16)))
        return WZYB_ERR_ALIGN;
    if (T == 0) return WZYB_OK;
    DeviceInfo di;
    rc = device_info(&di);
    if (rc != WZYB_OK) return rc;
    const int vpr = n / 8;
    const int64_t nvec = T * vpr;
    const int grid = persistent_grid(di, 8, (nvec + kMixThreads - 1) / kMixThreads);
    if (hc == 4)
        launch_k(hc_mix_kernel<TI, 4>, grid, kMixThreads, 0, stream, xn, gg, mixed, mixed16, nvec, vpr, hc, 0.25f);
    else
        launch_k(hc_mix_kernel<TI, 0>, grid, kMixThreads, 0, stream, xn, gg, mixed, mixed16, nvec, vpr, hc, 1.0f / (float)hc);
    return launch_status();
}

}  // namespace wzyb

extern "C" {

int wzyb_gr_write_f32(float* R, const float* blk, const float* inj, int64_t T, int n_embd, int hc,
                      wzyb_stream_t stream) {
    if (!R || !blk) return WZYB_ERR_NULL;
    int rc = wzyb::check_hc_shape(T, n_embd, hc);
    if (rc != WZYB_OK) return rc;
    if (!wzyb::aligned16(R) || !wzyb::aligned16(blk)) return WZYB_ERR_ALIGN;
    if (T == 0) return WZYB_OK;
    wzyb::DeviceInfo di;
    rc = wzyb::device_info(&di);
    if (rc != WZYB_OK) return rc;
    const int64_t rows = T * hc;
    const int64_t nvec = rows * (n_embd / 8);
    if (rows < (int64_t)di.sms * 4) {  // fewer rows than a quarter of the warps one wave holds
        const int64_t blocks = (nvec + wzyb::kGrwThreads - 1) / wzyb::kGrwThreads;
        wzyb::launch_k(wzyb::gr_write_flat_kernel, (unsigned)blocks, wzyb::kGrwThreads, 0, (cudaStream_t)stream, 
            R, blk, inj, nvec, n_embd / 8, hc);
        return wzyb::launch_status();
    }
    const int grid = wzyb::persistent_grid(di, 8, (rows + 7) / 8);
    wzyb::launch_k(wzyb::gr_write_kernel, grid, wzyb::kGrwThreads, 0, (cudaStream_t)stream, R, blk, inj, rows, n_embd, hc);
    return wzyb::launch_status();
}

int wzyb_hc_mix_f16(const uint16_t* xn, const uint16_t* gg, float* mixed, uint16_t* mixed_f16, int64_t T,
                    int n_embd, int hc, wzyb_stream_t stream) {
    return wzyb::launch_hc_mix<__half>((const __half*)xn, (const __half*)gg, mixed, (__half*)mixed_f16, T, n_embd, hc,
                                       (cudaStream_t)stream);
}

int wzyb_hc_mix_f32(const float* xn, const float* gg, float* mixed, int64_t T, int n_embd, int hc,
                    wzyb_stream_t stream) {
    return wzyb::launch_hc_mix<float>(xn, gg, mixed, nullptr, T, n_embd, hc, (cudaStream_t)stream);
}

int wzyb_silu_scale_f16(const float* lo, uint16_t* out, int64_t n, float scale, wzyb_stream_t stream) {
    if (!lo || !out) return WZYB_ERR_NULL;
    if (n < 0 || (n % 8) != 0) return WZYB_ERR_SHAPE;
    if (!wzyb::aligned16(lo) || !wzyb::aligned16(out)) return WZYB_ERR_ALIGN;
    if (n == 0) return WZYB_OK;
    wzyb::DeviceInfo di;
    const int rc = wzyb::device_info(&di);
    if (rc != WZYB_OK) return rc;
    const int64_t nvec = n / 8;
    const int grid = wzyb::persistent_grid(di, 8, (nvec + 255) / 256);
    wzyb::launch_k(wzyb::silu_scale_kernel, grid, 256, 0, (cudaStream_t)stream, lo, (__half*)out, nvec, scale);
    return wzyb::launch_status();
}

}  // extern "C"
