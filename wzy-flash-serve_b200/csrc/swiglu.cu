// swiglu.cu -- SwiGLU activation out = (g / (1 + exp(-g))) * u, one HBM pass.
//
// Math follows silu_mul_multi (src/wzy_kernels_v2.cuh:1240-1244) for separate gate/up tensors and
// pf_silu_mul_interleaved_to_fp16 (src/wzy_prefill_tc.cuh:69-80) for rows laid out [gate | up]; the
// routed-expert epilogues (src/wzy_prefill_tc.cuh:346-360) compute the same expression.
// The reference handles one element (or two) per thread with 4-byte accesses. Here a persistent
// grid streams 16-byte vectors: each thread keeps kUnroll vectors of gate and of up in flight
// before computing, so an SM has ~128 KB of loads outstanding, and stores 16 bytes per vector.
#include "launch.hpp"
#include "common.cuh"

namespace wzyb {

constexpr int kSwigluThreads = 256;
constexpr int kUnroll = 4;

// silu(g) * u on a pair: the reference's (g / (1 + exp(-g))) * u as (g * sigmoid(g)) * u, with the
// sigmoid from the base-2 exponential and reciprocal approximations (sigmoid2, common.cuh).
__device__ __forceinline__ float2 silu_mul2(float2 g, float2 u) { return fmul2(fmul2(g, sigmoid2(g)), u); }

// Scalar form with the fast exp and divide intrinsics, in the reference's exact expression order.
__device__ __forceinline__ float silu_mul(float g, float u) { return __fdividef(g, 1.0f + __expf(-g)) * u; }

template <typename TI, typename TO, bool PACKED>
__device__ __forceinline__ void swiglu_vec(const typename Vec8<TI>::Raw& gr, const typename Vec8<TI>::Raw& ur,
                                           TO* dst) {
    if (PACKED) {
        float2 g[4], u[4], o[4];
        Vec8<TI>::cvt2(gr, g);
        Vec8<TI>::cvt2(ur, u);
#pragma unroll
        for (int i = 0; i < 4; ++i) o[i] = silu_mul2(g[i], u[i]);
        Vec8<TO>::store2(dst, o);
    } else {
        float g[8], u[8], o[8];
        Vec8<TI>::cvt(gr, g);
        Vec8<TI>::cvt(ur, u);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = silu_mul(g[e], u[e]);
        Vec8<TO>::store(dst, o);
    }
}

// Vector v of the output; INTERLEAVED: rows of 2*nff inputs [gate | up] -> rows of nff outputs.
template <bool INTERLEAVED>
__device__ __forceinline__ void swiglu_offsets(int64_t v, int64_t vpr, int64_t nff, int64_t& gi, int64_t& ui,
                                               int64_t& oi) {
    if (INTERLEAVED) {
        const int64_t t = v / vpr;
        const int64_t c = (v - t * vpr) * 8;
        gi = t * 2 * nff + c;
        ui = gi + nff;
        oi = t * nff + c;
    } else {
        gi = ui = oi = v * 8;
    }
}

// The body takes its CTA's index among `nctas` CTAs that share the vectors (a fused bundle kernel runs it
// on a subset of its grid).
template <typename TI, typename TO, bool INTERLEAVED, bool PACKED>
__device__ __forceinline__ void swiglu_body(const TI* __restrict__ gate, const TI* __restrict__ up,
                                            TO* __restrict__ out, int64_t nvec, int64_t vpr, int64_t nff, int cta,
                                            int nctas) {
    const int64_t stride = (int64_t)nctas * blockDim.x;
    int64_t v = (int64_t)cta * blockDim.x + threadIdx.x;
    for (; v + (kUnroll - 1) * stride < nvec; v += kUnroll * stride) {
        typename Vec8<TI>::Raw gr[kUnroll], ur[kUnroll];
#pragma unroll
        for (int k = 0; k < kUnroll; ++k) {
            int64_t gi, ui, oi;
            swiglu_offsets<INTERLEAVED>(v + k * stride, vpr, nff, gi, ui, oi);
            gr[k] = Vec8<TI>::ldcs_raw(gate + gi);
            ur[k] = Vec8<TI>::ldcs_raw(up + ui);
        }
#pragma unroll
        for (int k = 0; k < kUnroll; ++k) {
            int64_t gi, ui, oi;
            swiglu_offsets<INTERLEAVED>(v + k * stride, vpr, nff, gi, ui, oi);
            swiglu_vec<TI, TO, PACKED>(gr[k], ur[k], out + oi);
        }
    }
    for (; v < nvec; v += stride) {
        int64_t gi, ui, oi;
        swiglu_offsets<INTERLEAVED>(v, vpr, nff, gi, ui, oi);
        swiglu_vec<TI, TO, PACKED>(Vec8<TI>::ldcs_raw(gate + gi), Vec8<TI>::ldcs_raw(up + ui), out + oi);
    }
}

template <typename TI, typename TO, bool INTERLEAVED, bool PACKED>
__global__ void __launch_bounds__(kSwigluThreads) swiglu_kernel(const TI* __restrict__ gate, const TI* __restrict__ up,
                                                                 TO* __restrict__ out, int64_t nvec, int64_t vpr,
                                                                 int64_t nff) {
    pdl_begin();
    swiglu_body<TI, TO, INTERLEAVED, PACKED>(gate, up, out, nvec, vpr, nff, blockIdx.x, gridDim.x);
}

// Math path of the SwiGLU stream for nvec 8-element vectors. Measured on B200 (same box, same inputs):
// the packed base-2 sigmoid is faster for layer-sized calls (94% vs 86% of HBM peak at 4096 tokens x
// 11 x 512), the scalar exp/divide form for very long streams (96% vs 93% at 262,144 tokens), so the
// length picks, unless a SwiGLU `stages` tuning of 1 (scalar) or 2 (packed) forces one.
static bool swiglu_scalar_math(int64_t nvec) {
    const Tuning tu = tuning(kFamSwiglu);
    return tu.stages == 1 || (tu.stages != 2 && nvec >= (int64_t(1) << 25));
}

// SwiGLU fused with the GEMM-input quantisation, no activation output: silu_mul_quant32_multi
// (src/wzy_kernels_v2.cuh:1247-1279) for Q8_0, and the MXFP8 / NVFP4 block formats of sm_100's
// block-scaled tensor-core GEMMs. A warp covers 32 consecutive 8-element vectors; a group's max is one
// (16-element) or two (32-element) shuffles. The activation uses the reference's own expression,
// (g / (1 + __expf(-g))) * u with the IEEE divide, so on the same inputs the Q8 codes and scales come
// out as the reference kernel's.
template <typename TI, int QF, int SFL>
__global__ void __launch_bounds__(256) swiglu_quant_kernel(const TI* __restrict__ gate, const TI* __restrict__ up,
                                                           void* __restrict__ q, void* __restrict__ s, float gs,
                                                           int64_t nvec, int vpr, int ncb) {
    pdl_begin();
    constexpr int kG = QF == kQfNvfp4 ? 16 : 32;  // elements per scale
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int64_t first = ((int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * 32;
    // tiled scales: vector v = (row q, vector in row r), stepped; row-major scales need neither
    StridePos ps(SFL == kSfTiled128x4 ? first + lane : 0, SFL == kSfTiled128x4 ? nwarps * 32 : 0, vpr);
    for (int64_t base = first; base < nvec; base += nwarps * 32) {
        const int64_t v = base + lane;
        const bool act = v < nvec;
        float o[8] = {};
        if (act) {
            float g[8], u[8];
            Vec8<TI>::load_stream(gate + v * 8, g);
            Vec8<TI>::load_stream(up + v * 8, u);
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = (g[e] / (1.0f + __expf(-g[e]))) * u[e];
        }
        if constexpr (SFL == kSfTiled128x4) {
            block_group_store_at<QF>(o, act, q, static_cast<uint8_t*>(s) + sf_tiled_offset(ps.q, ps.r * 8 / kG, ncb),
                                     gs, v, lane);
            ps.advance();
        } else {
            quant_group_store<QF>(o, act, q, s, gs, v, lane);
        }
    }
}

template <typename TI, typename TO, bool INTERLEAVED>
static int launch_swiglu(const TI* gate, const TI* up, TO* out, int64_t nvec, int64_t vpr, int64_t nff,
                         cudaStream_t stream) {
    if (nvec == 0) return WZYB_OK;
    DeviceInfo di;
    const int rc = device_info(&di);
    if (rc != WZYB_OK) return rc;
    const Tuning tu = tuning(kFamSwiglu);
    const int grid = persistent_grid(di, tu.ctas_per_sm, (nvec + kSwigluThreads - 1) / kSwigluThreads);
    if (swiglu_scalar_math(nvec))
        launch_k(swiglu_kernel<TI, TO, INTERLEAVED, false>, grid, kSwigluThreads, 0, stream, gate, up, out, nvec, vpr, nff);
    else
        launch_k(swiglu_kernel<TI, TO, INTERLEAVED, true>, grid, kSwigluThreads, 0, stream, gate, up, out, nvec, vpr, nff);
    return launch_status();
}

// n % 32 == 0 (the largest group); Q8 scales are fp32 (4-byte aligned), the block formats' are bytes.
// n elements as rows of `cols` (cols == n for the flat forms); sf_layout for the block formats.
template <int QF>
static int launch_swiglu_quant(const float* gate, const float* up, void* q, void* s, float gs, int64_t n,
                               wzyb_stream_t stream, int64_t cols = 0, int sf_layout = kSfRowMajor) {
    if (!gate || !up || !q || !s) return WZYB_ERR_NULL;
    if (sf_layout != kSfRowMajor && (QF == kQfQ8 || sf_layout != kSfTiled128x4)) return WZYB_ERR_VALUE;
    if (n < 0 || (n % 32) != 0) return WZYB_ERR_SHAPE;
    if (cols == 0) cols = n;  // the flat forms: one row
    if (n > 0 && (cols < 32 || (cols % 32) != 0 || (n % cols) != 0 || cols > (int64_t(1) << 30)))
        return WZYB_ERR_SHAPE;
    if (!aligned16(gate) || !aligned16(up) || !aligned16(q) || (QF == kQfQ8 && !aligned16(s))) return WZYB_ERR_ALIGN;
    if (n == 0) return WZYB_OK;
    DeviceInfo di;
    const int rc = device_info(&di);
    if (rc != WZYB_OK) return rc;
    const int64_t nvec = n / 8;
    const int ncb = (int)((cols / (QF == kQfNvfp4 ? 16 : 32) + 3) / 4);
    const int grid = persistent_grid(di, 8, (nvec + 255) / 256);
    if constexpr (QF != kQfQ8) {
        if (sf_layout == kSfTiled128x4) {
            launch_k(swiglu_quant_kernel<float, QF, kSfTiled128x4>, grid, 256, 0, (cudaStream_t)stream, gate, up, q, s,
                     gs, nvec, (int)(cols / 8), ncb);
            return launch_status();
        }
    }
    launch_k(swiglu_quant_kernel<float, QF, kSfRowMajor>, grid, 256, 0, (cudaStream_t)stream, gate, up, q, s, gs, nvec,
             (int)(cols / 8), ncb);
    return launch_status();
}

}  // namespace wzyb

extern "C" {

int wzyb_swiglu_f16(const uint16_t* gate, const uint16_t* up, uint16_t* out, int64_t n, wzyb_stream_t stream) {
    if (!gate || !up || !out) return WZYB_ERR_NULL;
    if (n < 0 || (n % 8) != 0) return WZYB_ERR_SHAPE;
    if (!wzyb::aligned16(gate) || !wzyb::aligned16(up) || !wzyb::aligned16(out)) return WZYB_ERR_ALIGN;
    return wzyb::launch_swiglu<__half, __half, false>((const __half*)gate, (const __half*)up, (__half*)out, n / 8, 0, 0,
                                                      (cudaStream_t)stream);
}

int wzyb_swiglu_f32(const float* gate, const float* up, float* out, int64_t n, wzyb_stream_t stream) {
    if (!gate || !up || !out) return WZYB_ERR_NULL;
    if (n < 0 || (n % 8) != 0) return WZYB_ERR_SHAPE;
    if (!wzyb::aligned16(gate) || !wzyb::aligned16(up) || !wzyb::aligned16(out)) return WZYB_ERR_ALIGN;
    return wzyb::launch_swiglu<float, float, false>(gate, up, out, n / 8, 0, 0, (cudaStream_t)stream);
}

int wzyb_swiglu_q8_f32(const float* gate, const float* up, int8_t* q32, float* s32, int64_t n, wzyb_stream_t stream) {
    return wzyb::launch_swiglu_quant<wzyb::kQfQ8>(gate, up, q32, s32, 1.0f, n, stream);
}

int wzyb_swiglu_mxfp8_f32(const float* gate, const float* up, uint8_t* q, uint8_t* s, int64_t n,
                          wzyb_stream_t stream) {
    return wzyb::launch_swiglu_quant<wzyb::kQfMxfp8>(gate, up, q, s, 1.0f, n, stream);
}

int wzyb_swiglu_nvfp4_f32(const float* gate, const float* up, uint8_t* q, uint8_t* s, float global_scale, int64_t n,
                          wzyb_stream_t stream) {
    return wzyb::launch_swiglu_quant<wzyb::kQfNvfp4>(gate, up, q, s, global_scale, n, stream);
}

int wzyb_swiglu_block_f32(const float* gate, const float* up, uint8_t* q, uint8_t* s, int format, int sf_layout,
                          float global_scale, int64_t rows, int cols, wzyb_stream_t stream) {
    if (rows < 0 || cols < 32 || rows > (int64_t(1) << 40)) return WZYB_ERR_SHAPE;
    if (format == WZYB_BLOCK_MXFP8)
        return wzyb::launch_swiglu_quant<wzyb::kQfMxfp8>(gate, up, q, s, 1.0f, rows * cols, stream, cols, sf_layout);
    if (format == WZYB_BLOCK_NVFP4)
        return wzyb::launch_swiglu_quant<wzyb::kQfNvfp4>(gate, up, q, s, global_scale, rows * cols, stream, cols,
                                                        sf_layout);
    return WZYB_ERR_VALUE;
}

int wzyb_swiglu_interleaved_f16(const uint16_t* gu, uint16_t* out, int64_t T, int nff, wzyb_stream_t stream) {
    if (!gu || !out) return WZYB_ERR_NULL;
    if (T < 0 || nff < 8 || (nff % 8) != 0) return WZYB_ERR_SHAPE;
    if (!wzyb::aligned16(gu) || !wzyb::aligned16(out)) return WZYB_ERR_ALIGN;
    const int64_t vpr = nff / 8;
    return wzyb::launch_swiglu<__half, __half, true>((const __half*)gu, (const __half*)gu, (__half*)out, T * vpr, vpr,
                                                     nff, (cudaStream_t)stream);
}

int wzyb_swiglu_interleaved_f32_f16(const float* gu, uint16_t* out, int64_t T, int nff, wzyb_stream_t stream) {
    if (!gu || !out) return WZYB_ERR_NULL;
    if (T < 0 || nff < 8 || (nff % 8) != 0) return WZYB_ERR_SHAPE;
    if (!wzyb::aligned16(gu) || !wzyb::aligned16(out)) return WZYB_ERR_ALIGN;
    const int64_t vpr = nff / 8;
    return wzyb::launch_swiglu<float, __half, true>(gu, gu, (__half*)out, T * vpr, vpr, nff, (cudaStream_t)stream);
}

}  // extern "C"
