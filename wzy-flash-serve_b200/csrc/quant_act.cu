// quant_act.cu -- fp32 activation rows to the int8 GEMM inputs, in one HBM pass.
//
// Math follows quant_act_multi (src/wzy_kernels_v2.cuh:58-111): per group of 32 (q32/s32) and, from
// the same read, per group of 16 (q16/s16): d = amax / 127, q = rint(x * (127 / amax)) clamped to
// [-127, 127]. The reference gives each thread one 16-element group (scalar 4-byte re-reads of the
// second half for the 32-wide scale). Here a lane holds 8 elements (two 16-byte loads); a 16-group
// is 2 lanes and a 32-group 4 lanes: one lane max, then one xor shuffle for the 16-group max and one
// more for the 32-group max.
//
// The same pass also writes the block-scaled formats that sm_100's tensor cores take as GEMM
// inputs (tcgen05.mma block scaling): MXFP8 (e4m3 codes, E8M0 scale per 32) and NVFP4 (e2m1 codes
// two per byte, e4m3 scale per 16, a per-tensor scale). Their rules are in common.cuh.
#include "launch.hpp"
#include "common.cuh"

namespace wzyb {

__global__ void __launch_bounds__(256) quant_act_kernel(const float* __restrict__ x, signed char* __restrict__ q32,
                                                        float* __restrict__ s32, signed char* __restrict__ q16,
                                                        float* __restrict__ s16, int64_t nvec) {
    pdl_begin();
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t base = ((int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * 32; base < nvec;
         base += nwarps * 32) {
        const int64_t v = base + lane;
        const bool act = v < nvec;
        float o[8] = {};
        if (act) Vec8<float>::load_stream(x + v * 8, o);
        if (q16 != nullptr && q32 != nullptr) {
            q8_group_store_16_32(o, act, q16 + v * 8, s16 + (v >> 1), q32 + v * 8, s32 + (v >> 2), lane);
        } else {
            if (q16 != nullptr) q8_group_store<2>(o, act, q16 + v * 8, s16 + (v >> 1), lane);
            if (q32 != nullptr) q8_group_store<4>(o, act, q32 + v * 8, s32 + (v >> 2), lane);
        }
    }
}

// Row-major scales index by the flat vector; the tiled 128x4 layout needs the (row, scale column) of
// each lane's vector, stepped per lane with StridePos (no division in the loop).
template <int QF, int SFL>
__global__ void __launch_bounds__(256) quant_act_block_kernel(const float* __restrict__ x, void* __restrict__ q,
                                                              void* __restrict__ s, float gs, int64_t nvec, int vpr,
                                                              int ncb) {
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
        if (act) Vec8<float>::load_stream(x + v * 8, o);
        if constexpr (SFL == kSfTiled128x4) {
            block_group_store_at<QF>(o, act, q, static_cast<uint8_t*>(s) + sf_tiled_offset(ps.q, ps.r * 8 / kG, ncb),
                                     gs, v, lane);
            ps.advance();
        } else {
            quant_group_store<QF>(o, act, q, s, gs, v, lane);
        }
    }
}

template <int QF>
static int launch_quant_act_block(const float* x, void* q, void* s, float gs, int sf_layout, int64_t T, int cols,
                                  wzyb_stream_t stream) {
    if (!x || !q || !s) return WZYB_ERR_NULL;
    const int group = QF == kQfNvfp4 ? 16 : 32;
    if (sf_layout != kSfRowMajor && sf_layout != kSfTiled128x4) return WZYB_ERR_VALUE;
    if (T < 0 || T > (int64_t(1) << 40) || cols < group || (cols % group) != 0) return WZYB_ERR_SHAPE;
    if (!aligned16(x) || !aligned16(q)) return WZYB_ERR_ALIGN;
    if (T == 0) return WZYB_OK;
    DeviceInfo di;
    const int rc = device_info(&di);
    if (rc != WZYB_OK) return rc;
    const int64_t nvec = T * cols / 8;
    const int ncb = (cols / group + 3) / 4;
    const int grid = persistent_grid(di, 8, (nvec + 255) / 256);
    if (sf_layout == kSfTiled128x4)
        launch_k(quant_act_block_kernel<QF, kSfTiled128x4>, grid, 256, 0, (cudaStream_t)stream, x, q, s, gs, nvec,
                 cols / 8, ncb);
    else
        launch_k(quant_act_block_kernel<QF, kSfRowMajor>, grid, 256, 0, (cudaStream_t)stream, x, q, s, gs, nvec,
                 cols / 8, ncb);
    return launch_status();
}

}  // namespace wzyb

extern "C" {

int wzyb_quant_act_f32(const float* x, int8_t* q32, float* s32, int8_t* q16, float* s16, int64_t T, int cols,
                       wzyb_stream_t stream) {
    if (!x || (!q32 && !q16) || (q32 && !s32) || (q16 && !s16)) return WZYB_ERR_NULL;
    if (T < 0 || T > (int64_t(1) << 40) || cols < 16 || (cols % (q32 ? 32 : 16)) != 0) return WZYB_ERR_SHAPE;
    if (!wzyb::aligned16(x) || (q32 && !wzyb::aligned16(q32)) || (q16 && !wzyb::aligned16(q16)) ||
        (s32 && ((uintptr_t)s32 & 3)) || (s16 && ((uintptr_t)s16 & 3)))
        return WZYB_ERR_ALIGN;
    if (T == 0) return WZYB_OK;
    wzyb::DeviceInfo di;
    const int rc = wzyb::device_info(&di);
    if (rc != WZYB_OK) return rc;
    const int64_t nvec = T * cols / 8;
    const int grid = wzyb::persistent_grid(di, 8, (nvec + 255) / 256);
    wzyb::launch_k(wzyb::quant_act_kernel, grid, 256, 0, (cudaStream_t)stream, x, (signed char*)q32, s32, (signed char*)q16, s16,
                                                                    nvec);
    return wzyb::launch_status();
}

int wzyb_quant_act_mxfp8_f32(const float* x, uint8_t* q, uint8_t* s, int64_t T, int cols, wzyb_stream_t stream) {
    return wzyb::launch_quant_act_block<wzyb::kQfMxfp8>(x, q, s, 1.0f, wzyb::kSfRowMajor, T, cols, stream);
}

int wzyb_quant_act_nvfp4_f32(const float* x, uint8_t* q, uint8_t* s, float global_scale, int64_t T, int cols,
                             wzyb_stream_t stream) {
    return wzyb::launch_quant_act_block<wzyb::kQfNvfp4>(x, q, s, global_scale, wzyb::kSfRowMajor, T, cols, stream);
}

int wzyb_quant_act_block_f32(const float* x, uint8_t* q, uint8_t* s, int format, int sf_layout, float global_scale,
                             int64_t T, int cols, wzyb_stream_t stream) {
    if (format == WZYB_BLOCK_MXFP8)
        return wzyb::launch_quant_act_block<wzyb::kQfMxfp8>(x, q, s, 1.0f, sf_layout, T, cols, stream);
    if (format == WZYB_BLOCK_NVFP4)
        return wzyb::launch_quant_act_block<wzyb::kQfNvfp4>(x, q, s, global_scale, sf_layout, T, cols, stream);
    return WZYB_ERR_VALUE;
}

}  // extern "C"
