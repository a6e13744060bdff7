// gdn_norm.cu -- GDN output gated RMSNorm, one HBM pass.
//
// Math follows pf_gdn_rmsnorm_gate_parallel (src/wzy_qsa_wmma.cuh:178-195) and the tail of
// fused_gdn_step_norm_multi (src/wzy_kernels_v2.cuh:966-976):
//   y = o * rsqrt(sum(o^2)/hd + eps) * gamma[col] / (1 + exp(-z))
// i.e. the gate is sigmoid(z) at every reference site; WZYB_GATE_SILU selects z*sigmoid(z).
// The reference runs one 128-thread block per (head, token) with a shared-memory reduction. Here each
// head is owned by hd/8 lanes that reduce with xor shuffles, and y leaves with one 16-byte store per
// lane. Default (direct): a warp per 256-element slab, 4 slabs' loads in flight per warp; on request,
// the slabs staged in shared memory by cp.async (async).
#include "launch.hpp"

namespace wzyb {

// x gated by sigmoid(z) (or z*sigmoid(z)), with x = o * rsqrt(...) * gamma already formed in the
// reference's order. The reference divides x by (1 + exp(-z)); __fdividef is the fast divide
// (<= 2 fp32 ulp apart, far inside an fp16 ulp). When 1 + exp(-z) exceeds 2^126 (z < -87) it
// returns 0, where the exact quotient is below 1e-37.
__device__ __forceinline__ float gdn_gate(float x, float z, bool silu) {
    const float den = 1.0f + __expf(-z);
    const float q = __fdividef(silu ? z : x, den);  // one divide for either gate
    return silu ? x * q : q;
}

// One head's 8-element slice in this lane (packed fp32), the sum of squares reduced over the head's
// L lanes:  x = (o * rsqrt(sum/hd + eps)) * gamma;  out = x * sigmoid(z)  or  x * (z * sigmoid(z)).
// The reference divides x by (1 + exp(-z)); here x is multiplied by the approximate reciprocal of
// 1 + 2^(-z log2 e) (sigmoid2), a few fp32 ulp from the IEEE quotient.
template <int L, int HD, bool SILU>
__device__ __forceinline__ void gdn_vec(const float2 (&o)[4], const float2 (&z)[4], const float2 (&g)[4], float eps,
                                        float2 (&out)[4]) {
    const float ss = group_sum<L>(sumsq8(o));
    const float2 sc = splat2(rsqrt_approx(ss * (1.0f / (float)HD) + eps));
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 x = fmul2(fmul2(o[i], sc), g[i]);
        const float2 s = sigmoid2(z[i]);
        out[i] = SILU ? fmul2(x, fmul2(z[i], s)) : fmul2(x, s);
    }
}

struct GdnArgs {
    const void* o;
    const void* z;
    const void* gamma;
    void* y;
    int64_t T;
    int heads;
    float eps;
    float w_offset;
    int gate_mode;
};

// Direct design: a warp owns one 256-element slab of a token row (32/L whole heads), keeps kU slabs of
// o and z in flight as raw 16-byte registers, then normalises each head inside its lane group. No
// shared memory, no CTA barrier: warps stream independently like a copy kernel.
// The body takes its CTA's index among `nctas` CTAs that share the slabs (a fused bundle kernel runs it
// on a subset of its grid).
template <typename TI, typename TO, int HD, int kU, bool SILU>
__device__ __forceinline__ void gdn_direct_body(const GdnArgs& a, int cta, int nctas) {
    constexpr int L = HD / 8;
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = (int64_t)nctas * (blockDim.x >> 5);
    const int64_t gwarp = (int64_t)cta * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int row_elems = a.heads * HD;
    const int slabs = (row_elems + 255) / 256;
    const int64_t items = a.T * slabs;
    const TI* __restrict__ o = static_cast<const TI*>(a.o);
    const TI* __restrict__ z = static_cast<const TI*>(a.z);
    TO* __restrict__ y = static_cast<TO*>(a.y);
    float2 g[4];
    Vec8<TI>::load_ro2(static_cast<const TI*>(a.gamma) + (lane % L) * 8, g);
#pragma unroll
    for (int i = 0; i < 4; ++i) g[i] = fadd2(splat2(a.w_offset), g[i]);

    StridePos pos(gwarp, nwarps, slabs);  // item it = (token q, slab r)
    for (int64_t base = gwarp; base < items; base += nwarps * kU) {
        typename Vec8<TI>::Raw ro[kU], rz[kU];
        int64_t off[kU];
#pragma unroll
        for (int k = 0; k < kU; ++k) {
            const int64_t it = base + k * nwarps;
            off[k] = -1;
            if (it < items) {
                const int e = pos.r * 256 + lane * 8;
                if (e < row_elems) {
                    off[k] = pos.q * row_elems + e;
                    ro[k] = Vec8<TI>::ldcs_raw(o + off[k]);
                    rz[k] = Vec8<TI>::ldcs_raw(z + off[k]);
                }
            }
            pos.advance();
        }
#pragma unroll
        for (int k = 0; k < kU; ++k) {
            if (base + k * nwarps >= items) break;  // warp-uniform
            float2 ov[4], zv[4], out[4];
            if (off[k] >= 0) {
                Vec8<TI>::cvt2(ro[k], ov);
                Vec8<TI>::cvt2(rz[k], zv);
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i) ov[i] = zv[i] = splat2(0.f);
            }
            gdn_vec<L, HD, SILU>(ov, zv, g, a.eps, out);
            if (off[k] >= 0) Vec8<TO>::store2(y + off[k], out);
        }
    }
}

template <typename TI, typename TO, int HD, int kU, bool SILU>
__global__ void __launch_bounds__(256, sizeof(TI) == 2 ? 3 : 2) gdn_direct_kernel(const GdnArgs a) {
    pdl_begin();
    gdn_direct_body<TI, TO, HD, kU, SILU>(a, blockIdx.x, gridDim.x);
}

// Async design: the direct design's warp-owned slabs, but the kP slabs in flight per warp sit in a
// lane-private shared-memory ring filled by cp.async instead of in registers. Each lane copies and
// later reads only its own 16-byte chunks, so the ring needs no barrier at all; the register file is
// no longer what bounds the bytes in flight.
template <typename TI, typename TO, int HD, int kP, bool SILU>
__global__ void __launch_bounds__(256) gdn_async_kernel(const GdnArgs a) {
    pdl_begin();
    constexpr int L = HD / 8;
    constexpr int C = Vec8<TI>::kChunks;   // 16-byte chunks per 8-element vector
    constexpr int SLOT = 2 * C * 32;       // uint4 per ring slot: o and z vectors of 32 lanes
    extern __shared__ __align__(16) uint4 sm_gdn[];
    const int lane = threadIdx.x & 31;
    uint4* ring = sm_gdn + (size_t)(threadIdx.x >> 5) * kP * SLOT;
    const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int64_t gwarp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int row_elems = a.heads * HD;
    const int slabs = (row_elems + 255) / 256;
    const int64_t items = a.T * slabs;
    const TI* __restrict__ o = static_cast<const TI*>(a.o);
    const TI* __restrict__ z = static_cast<const TI*>(a.z);
    TO* __restrict__ y = static_cast<TO*>(a.y);
    float2 g[4];
    Vec8<TI>::load_ro2(static_cast<const TI*>(a.gamma) + (lane % L) * 8, g);
#pragma unroll
    for (int i = 0; i < 4; ++i) g[i] = fadd2(splat2(a.w_offset), g[i]);

    // element offset of this lane's vector for the item at `p`, or -1
    auto offset = [&](int64_t it, const StridePos& p) -> int64_t {
        if (it >= items) return -1;
        const int e = p.r * 256 + lane * 8;
        return e < row_elems ? p.q * row_elems + e : -1;
    };
    StridePos ipos(gwarp, nwarps, slabs);  // next item to issue
    StridePos cpos(gwarp, nwarps, slabs);  // next item to consume
    auto issue = [&](int64_t it, int slot) {
        const int64_t off = offset(it, ipos);
        ipos.advance();
        if (off >= 0) {
            Vec8<TI>::stage_async(ring + slot * SLOT, lane, o + off);
            Vec8<TI>::stage_async(ring + slot * SLOT + C * 32, lane, z + off);
        }
        cp_async_commit();  // one group per item, empty or not, so wait_group counts items
    };
#pragma unroll
    for (int j = 0; j < kP; ++j) issue(gwarp + j * nwarps, j);

    for (int64_t j = 0;; ++j) {
        const int64_t it = gwarp + j * nwarps;
        if (it >= items) break;  // warp-uniform
        const int slot = (int)(j % kP);
        cp_async_wait<kP - 1>();
        const int64_t off = offset(it, cpos);
        cpos.advance();
        float2 ov[4], zv[4], out[4];
        if (off >= 0) {
            Vec8<TI>::unstage2(ring + slot * SLOT, lane, ov);
            Vec8<TI>::unstage2(ring + slot * SLOT + C * 32, lane, zv);
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) ov[i] = zv[i] = splat2(0.f);
        }
        // Refill the slot. Only this lane reads or writes its chunks of the slot, and its unstaging
        // loads precede the new copy in program order, which orders them before the copy's write.
        issue(it + kP * nwarps, slot);
        gdn_vec<L, HD, SILU>(ov, zv, g, a.eps, out);
        if (off >= 0) Vec8<TO>::store2(y + off, out);
    }
    cp_async_wait<0>();
}

// Launch one of the warp-owned designs (direct or cp.async) for head size hd.
template <typename TI, typename TO, bool SILU>
static int launch_gdn_warp(const GdnArgs& a, int hd, bool async_design, const DeviceInfo& di, cudaStream_t stream) {
    constexpr int kP = sizeof(TI) == 2 ? 8 : 4;
    const int64_t warp_items = a.T * (((int64_t)a.heads * hd + 255) / 256);
    if (async_design) {
        const void* kern = hd == 64    ? (const void*)gdn_async_kernel<TI, TO, 64, kP, SILU>
                           : hd == 128 ? (const void*)gdn_async_kernel<TI, TO, 128, kP, SILU>
                                       : (const void*)gdn_async_kernel<TI, TO, 256, kP, SILU>;
        const int smem = 8 * kP * 2 * Vec8<TI>::kChunks * 32 * 16;
        const int rc = ensure_smem(kern, smem);
        if (rc != WZYB_OK) return rc;
        const int grid = persistent_grid(di, resident_ctas(kern, 256, smem), (warp_items + 7) / 8);
        if (hd == 64) launch_k(gdn_async_kernel<TI, TO, 64, kP, SILU>, grid, 256, smem, stream, a);
        else if (hd == 128) launch_k(gdn_async_kernel<TI, TO, 128, kP, SILU>, grid, 256, smem, stream, a);
        else launch_k(gdn_async_kernel<TI, TO, 256, kP, SILU>, grid, 256, smem, stream, a);
        return launch_status();
    }
    const void* kern = hd == 64    ? (const void*)gdn_direct_kernel<TI, TO, 64, 4, SILU>
                       : hd == 128 ? (const void*)gdn_direct_kernel<TI, TO, 128, 4, SILU>
                                   : (const void*)gdn_direct_kernel<TI, TO, 256, 4, SILU>;
    const int grid = persistent_grid(di, resident_ctas(kern, 256, 0), (warp_items + 7) / 8);
    if (hd == 64) launch_k(gdn_direct_kernel<TI, TO, 64, 4, SILU>, grid, 256, 0, stream, a);
    else if (hd == 128) launch_k(gdn_direct_kernel<TI, TO, 128, 4, SILU>, grid, 256, 0, stream, a);
    else launch_k(gdn_direct_kernel<TI, TO, 256, 4, SILU>, grid, 256, 0, stream, a);
    return launch_status();
}

// Validates a GDN gated-norm call on the host and fills `a`. Returns WZYB_OK or the WZYB_ERR_* of the
// first bad argument; nothing is enqueued.
template <typename TI>
static int gdn_prepare(const void* o, const void* z, const void* gamma, void* y, int64_t T, int heads, int hd,
                       float eps, float w_offset, int gate_mode, GdnArgs& a) {
    if (o == nullptr || z == nullptr || gamma == nullptr || y == nullptr) return WZYB_ERR_NULL;
    if (gate_mode != WZYB_GATE_SIGMOID && gate_mode != WZYB_GATE_SILU) return WZYB_ERR_VALUE;
    if (hd != 64 && hd != 128 && hd != 256) return WZYB_ERR_SHAPE;
    if (T < 0 || T > (int64_t(1) << 40) || heads < 1 || heads > 512) return WZYB_ERR_SHAPE;
    if (!aligned16(o) || !aligned16(z) || !aligned16(gamma) || !aligned16(y)) return WZYB_ERR_ALIGN;
    a.o = o;
    a.z = z;
    a.gamma = gamma;
    a.y = y;
    a.T = T;
    a.heads = heads;
    a.eps = eps;
    a.w_offset = w_offset;
    a.gate_mode = gate_mode;
    return WZYB_OK;
}

template <typename TI, typename TO>
static int launch_gdn(const void* o, const void* z, const void* gamma, void* y, int64_t T, int heads, int hd, float eps,
                      float w_offset, int gate_mode, cudaStream_t stream) {
    GdnArgs a;
    int rc = gdn_prepare<TI>(o, z, gamma, y, T, heads, hd, eps, w_offset, gate_mode, a);
    if (rc != WZYB_OK || T == 0) return rc;
    DeviceInfo di;
    rc = device_info(&di);
    if (rc != WZYB_OK) return rc;

    // The direct design is the default (measured on B200 at 262,144 tokens: direct 84%, cp.async 83%,
    // and 43% for a TMA ring design of one barrier-synchronised unit per CTA, since removed).
    const bool async_design = variant(kFamGdn) == WZYB_VARIANT_ASYNC;
    return gate_mode == WZYB_GATE_SILU ? launch_gdn_warp<TI, TO, true>(a, hd, async_design, di, stream)
                                       : launch_gdn_warp<TI, TO, false>(a, hd, async_design, di, stream);
}

}  // namespace wzyb

extern "C" {

int wzyb_gdn_gated_norm_f16(const uint16_t* o, const uint16_t* z, const uint16_t* gamma, uint16_t* y, int64_t T,
                            int heads, int head_dim, float eps, float w_offset, int gate_mode, wzyb_stream_t stream) {
    return wzyb::launch_gdn<__half, __half>(o, z, gamma, y, T, heads, head_dim, eps, w_offset, gate_mode,
                                            (cudaStream_t)stream);
}

int wzyb_gdn_gated_norm_f32_f16(const float* o, const float* z, const float* gamma, uint16_t* y, int64_t T, int heads,
                                int head_dim, float eps, float w_offset, int gate_mode, wzyb_stream_t stream) {
    return wzyb::launch_gdn<float, __half>(o, z, gamma, y, T, heads, head_dim, eps, w_offset, gate_mode,
                                           (cudaStream_t)stream);
}

}  // extern "C"
