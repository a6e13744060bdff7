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

// (g / (1 + exp(-g))) * u in the reference's order; __fdividef is the fast divide (<= 2 fp32 ulp from
// the IEEE quotient; 0 when g < -87, where the exact value is below 1e-35).
__device__ __forceinline__ float silu_mul(float g, float u) { return __fdividef(g, 1.0f + __expf(-g)) * u; }

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

template <typename TI, typename TO, bool INTERLEAVED>
__global__ void __launch_bounds__(kSwigluThreads) swiglu_kernel(const TI* __restrict__ gate, const TI* __restrict__ up,
                                                                 TO* __restrict__ out, int64_t nvec, int64_t vpr,
                                                                 int64_t nff) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
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
            float g[8], u[8], o[8];
            Vec8<TI>::cvt(gr[k], g);
            Vec8<TI>::cvt(ur[k], u);
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = silu_mul(g[e], u[e]);
            Vec8<TO>::store(out + oi, o);
        }
    }
    for (; v < nvec; v += stride) {
        int64_t gi, ui, oi;
        swiglu_offsets<INTERLEAVED>(v, vpr, nff, gi, ui, oi);
        float g[8], u[8], o[8];
        Vec8<TI>::load_stream(gate + gi, g);
        Vec8<TI>::load_stream(up + ui, u);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = silu_mul(g[e], u[e]);
        Vec8<TO>::store(out + oi, o);
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
    const int64_t per_wave = (int64_t)di.sms * tu.ctas_per_sm;
    const int64_t need = (nvec + kSwigluThreads - 1) / kSwigluThreads;
    const int grid = (int)(need < per_wave ? need : per_wave);
    swiglu_kernel<TI, TO, INTERLEAVED><<<grid, kSwigluThreads, 0, stream>>>(gate, up, out, nvec, vpr, nff);
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
