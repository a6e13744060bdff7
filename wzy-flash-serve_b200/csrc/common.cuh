// common.cuh -- device helpers shared by the wzyb200 layer kernels (sm_100a only).
//
// Everything on this path is HBM-bound streaming work (no dense contraction), so the helpers here are
// about moving bytes: 16-byte vector loads/stores of 8 elements, 1-D TMA bulk copies
// (cp.async.bulk) into shared memory completed on an mbarrier, and bounded mbarrier waits that give
// up after a time limit instead of spinning forever.
#pragma once
#include <cuda_fp16.h>
#include <cuda_fp4.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <cstring>

#include "../../include/wzyb200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "wzyb200 kernels are written for sm_100a (Blackwell) only"
#endif

namespace wzyb {

// ----------------------------------------------------------------------------------------------
// Fault word. Kernels never trap: when a bounded wait gives up or a device-side range check fails,
// they OR a WZYB_FAULT_* bit into this word and return. The host reads it with wzyb_read_faults().
// Defined here: the library is a single CUDA translation unit (wzyb200_all.cu).
// ----------------------------------------------------------------------------------------------
__device__ unsigned int g_fault_word = 0;

__device__ __forceinline__ void raise_fault(unsigned int bit) { atomicOr(&g_fault_word, bit); }

// A wait that has not completed after this many nanoseconds is treated as lost (1 s; a healthy
// wait here lasts a few microseconds at most).
constexpr unsigned long long kWaitLimitNs = 1000000000ull;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ----------------------------------------------------------------------------------------------
// mbarrier + 1-D bulk copy (TMA without a tensor map) primitives.
// ----------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Make mbarrier initialisation visible to the async (TMA) proxy before any bulk copy uses it.
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for phase `parity` of `bar` to complete. Returns false (and raises WZYB_FAULT_WAIT_TIMEOUT)
// if it has not completed within kWaitLimitNs; the caller must then stop using the pipeline.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 0u && globaltimer_ns() - t0 > kWaitLimitNs) {
            raise_fault(WZYB_FAULT_WAIT_TIMEOUT);
            return false;
        }
    }
}

// Like mbar_wait, but against an absolute %globaltimer deadline and without raising a fault:
// used to drain copies that are still in flight after a pipeline has been abandoned.
__device__ __forceinline__ bool mbar_wait_until(uint64_t* bar, uint32_t parity, unsigned long long deadline) {
    for (uint32_t it = 0;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 255u && globaltimer_ns() > deadline) return false;
    }
}

// L2 eviction policy for bytes that are read exactly once.
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// 1-D bulk copy global -> shared, completion counted on `bar` (bytes must be a multiple of 16 and
// both addresses 16-byte aligned; the launchers check this on the host).
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar,
                                          uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
            "r"(smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// ----------------------------------------------------------------------------------------------
// Per-thread asynchronous 16-byte copies global -> shared (cp.async.cg: L2 only). Each thread waits
// only for its own groups, so a lane that copies and later reads the same bytes needs no barrier.
// ----------------------------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// ----------------------------------------------------------------------------------------------
// 8-element vectors. fp16: one 16-byte access; fp32: two 16-byte accesses.
// ----------------------------------------------------------------------------------------------
template <typename T>
struct Vec8;

template <>
struct Vec8<__half> {
    static constexpr int kBytes = 16;
    // raw (unconverted) form, so several vectors can be in flight at 4 registers each
    struct Raw {
        uint4 u;
    };
    __device__ __forceinline__ static Raw ldcs_raw(const __half* p) {
        return Raw{__ldcs(reinterpret_cast<const uint4*>(p))};
    }
    __device__ __forceinline__ static void cvt(const Raw& r, float (&f)[8]) { to_f32(r.u, f); }
    // packed forms: 8 elements as float2[4]
    __device__ __forceinline__ static void cvt2(const uint4& u, float2 (&f)[4]) {
        const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) f[i] = __half22float2(h[i]);
    }
    __device__ __forceinline__ static void cvt2(const Raw& r, float2 (&f)[4]) { cvt2(r.u, f); }
    __device__ __forceinline__ static void load_ro2(const __half* p, float2 (&f)[4]) {
        cvt2(__ldg(reinterpret_cast<const uint4*>(p)), f);
    }
    // streaming (evict-first) store: the outputs of this path are not re-read by the same kernel
    __device__ __forceinline__ static void store2(__half* p, const float2 (&f)[4]) { __stcs(reinterpret_cast<uint4*>(p), pack2(f)); }
    // write-back store, for warps whose one store instruction covers only part of each 128-byte line
    // (an evict-first line can leave L2 before the other part arrives, costing a partial DRAM write)
    __device__ __forceinline__ static void store2_wb(__half* p, const float2 (&f)[4]) {
        *reinterpret_cast<uint4*>(p) = pack2(f);
    }
    __device__ __forceinline__ static uint4 pack2(const float2 (&f)[4]) {
        uint4 u;
        __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = __float22half2_rn(f[i]);
        return u;
    }
    // lane-private staging: a vector occupies kChunks 16-byte chunks, chunk c of lane l at slot[c*32 + l]
    static constexpr int kChunks = 1;
    __device__ __forceinline__ static void unstage2(const uint4* slot, int lane, float2 (&f)[4]) {
        cvt2(slot[lane], f);
    }
    __device__ __forceinline__ static void stage_async(uint4* slot, int lane, const __half* g) {
        cp_async16(slot + lane, g);
    }
    __device__ __forceinline__ static void unstage(const uint4* slot, int lane, float (&f)[8]) {
        to_f32(slot[lane], f);
    }
    __device__ __forceinline__ static void to_f32(const uint4& u, float (&f)[8]) {
        const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 p = __half22float2(h[i]);
            f[2 * i] = p.x;
            f[2 * i + 1] = p.y;
        }
    }
    __device__ __forceinline__ static uint4 from_f32(const float (&f)[8]) {
        uint4 u;
        __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
        return u;
    }
    // generic (smem or global) load
    __device__ __forceinline__ static void load(const __half* p, float (&f)[8]) {
        to_f32(*reinterpret_cast<const uint4*>(p), f);
    }
    // read-only global load through the non-coherent path
    __device__ __forceinline__ static void load_ro(const __half* p, float (&f)[8]) {
        to_f32(__ldg(reinterpret_cast<const uint4*>(p)), f);
    }
    // streaming global load (read once)
    __device__ __forceinline__ static void load_stream(const __half* p, float (&f)[8]) {
        to_f32(__ldcs(reinterpret_cast<const uint4*>(p)), f);
    }
    __device__ __forceinline__ static void store(__half* p, const float (&f)[8]) {
        *reinterpret_cast<uint4*>(p) = from_f32(f);
    }
    __device__ __forceinline__ static void store_stream(__half* p, const float (&f)[8]) {
        __stcs(reinterpret_cast<uint4*>(p), from_f32(f));
    }
};

template <>
struct Vec8<float> {
    static constexpr int kBytes = 32;
    struct Raw {
        float4 a, b;
    };
    __device__ __forceinline__ static Raw ldcs_raw(const float* p) {
        return Raw{__ldcs(reinterpret_cast<const float4*>(p)), __ldcs(reinterpret_cast<const float4*>(p) + 1)};
    }
    __device__ __forceinline__ static void cvt(const Raw& r, float (&f)[8]) {
        f[0] = r.a.x; f[1] = r.a.y; f[2] = r.a.z; f[3] = r.a.w;
        f[4] = r.b.x; f[5] = r.b.y; f[6] = r.b.z; f[7] = r.b.w;
    }
    __device__ __forceinline__ static void cvt2(const Raw& r, float2 (&f)[4]) {
        f[0] = make_float2(r.a.x, r.a.y);
        f[1] = make_float2(r.a.z, r.a.w);
        f[2] = make_float2(r.b.x, r.b.y);
        f[3] = make_float2(r.b.z, r.b.w);
    }
    __device__ __forceinline__ static void load_ro2(const float* p, float2 (&f)[4]) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(p));
        const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
        f[0] = make_float2(a.x, a.y);
        f[1] = make_float2(a.z, a.w);
        f[2] = make_float2(b.x, b.y);
        f[3] = make_float2(b.z, b.w);
    }
    // coherent load, for rows this kernel also writes
    __device__ __forceinline__ static void load2(const float* p, float2 (&f)[4]) {
        const float4 a = reinterpret_cast<const float4*>(p)[0];
        const float4 b = reinterpret_cast<const float4*>(p)[1];
        f[0] = make_float2(a.x, a.y);
        f[1] = make_float2(a.z, a.w);
        f[2] = make_float2(b.x, b.y);
        f[3] = make_float2(b.z, b.w);
    }
    __device__ __forceinline__ static void store2(float* p, const float2 (&f)[4]) {  // streaming
        __stcs(reinterpret_cast<float4*>(p), make_float4(f[0].x, f[0].y, f[1].x, f[1].y));
        __stcs(reinterpret_cast<float4*>(p) + 1, make_float4(f[2].x, f[2].y, f[3].x, f[3].y));
    }
    __device__ __forceinline__ static void store2_wb(float* p, const float2 (&f)[4]) {  // write-back
        reinterpret_cast<float4*>(p)[0] = make_float4(f[0].x, f[0].y, f[1].x, f[1].y);
        reinterpret_cast<float4*>(p)[1] = make_float4(f[2].x, f[2].y, f[3].x, f[3].y);
    }
    __device__ __forceinline__ static void unstage2(const uint4* slot, int lane, float2 (&f)[4]) {
        const float4 a = reinterpret_cast<const float4*>(slot)[lane];
        const float4 b = reinterpret_cast<const float4*>(slot)[32 + lane];
        f[0] = make_float2(a.x, a.y);
        f[1] = make_float2(a.z, a.w);
        f[2] = make_float2(b.x, b.y);
        f[3] = make_float2(b.z, b.w);
    }
    static constexpr int kChunks = 2;
    __device__ __forceinline__ static void stage_async(uint4* slot, int lane, const float* g) {
        cp_async16(slot + lane, g);
        cp_async16(slot + 32 + lane, g + 4);
    }
    __device__ __forceinline__ static void unstage(const uint4* slot, int lane, float (&f)[8]) {
        const float4 a = reinterpret_cast<const float4*>(slot)[lane];
        const float4 b = reinterpret_cast<const float4*>(slot)[32 + lane];
        f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
        f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
    }
    __device__ __forceinline__ static void load(const float* p, float (&f)[8]) {
        const float4 a = reinterpret_cast<const float4*>(p)[0];
        const float4 b = reinterpret_cast<const float4*>(p)[1];
        f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
        f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
    }
    __device__ __forceinline__ static void load_ro(const float* p, float (&f)[8]) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(p));
        const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
        f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
        f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
    }
    __device__ __forceinline__ static void load_stream(const float* p, float (&f)[8]) {
        const float4 a = __ldcs(reinterpret_cast<const float4*>(p));
        const float4 b = __ldcs(reinterpret_cast<const float4*>(p) + 1);
        f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
        f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
    }
    __device__ __forceinline__ static void store(float* p, const float (&f)[8]) {
        reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
        reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
    }
    __device__ __forceinline__ static void store_stream(float* p, const float (&f)[8]) {
        __stcs(reinterpret_cast<float4*>(p), make_float4(f[0], f[1], f[2], f[3]));
        __stcs(reinterpret_cast<float4*>(p) + 1, make_float4(f[4], f[5], f[6], f[7]));
    }
};

// Position q*d + r of a grid-stride walk, advanced by a fixed step without dividing: the quotient and
// remainder of the step are computed once, each advance is two adds and a carry. (A 64-bit division
// per work item costs dozens of instructions, which the byte-light kernels here cannot afford.)
// Programmatic dependent launch (PDL). Every kernel of the library starts with pdl_begin(): wait until
// the previous grid in the stream has completed and its writes are visible (a no-op when the launch
// carried no programmatic dependency), then allow the next grid in the stream to be launched. No
// kernel touches global memory before the wait, so PDL launches keep plain stream order semantics
// while the next launch's set-up and CTA placement overlap this grid's tail.
__device__ __forceinline__ void pdl_begin() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Hint that the 128-byte line holding p will be read soon: the line is fetched into L2 with no
// register held and nothing to wait for. Used to start the next work item's HBM reads while the
// current item is still being computed.
__device__ __forceinline__ void prefetch_l2(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

// x mod d for 64-bit x and d >= 1, with m = floor((2^64 - 1) / d) precomputed (Barrett reduction).
// q = mulhi(x, m) satisfies x/d - 2 < q <= x/d (m >= 2^64/d - 2 and m <= 2^64/d), so r = x - q*d lies
// in [0, 3d) and two conditional subtractions give the exact remainder -- a handful of instructions
// instead of the ~100 of a generic 64-bit division.
__host__ __device__ __forceinline__ uint64_t mod_u64(uint64_t x, uint64_t d, uint64_t m) {
#ifdef __CUDA_ARCH__
    const uint64_t q = __umul64hi(x, m);
#else
    const uint64_t q = (uint64_t)(((unsigned __int128)x * m) >> 64);
#endif
    uint64_t r = x - q * d;
    if (r >= d) r -= d;
    if (r >= d) r -= d;
    return r;
}

// Position (item / divisor, item % divisor) of a grid-stride loop over items start, start + step, ...,
// advanced without a division per item. start and step (a warp's or thread's index and the grid's
// count) fit 32 bits for every grid this library launches, where the two divisions are 32-bit ones
// (a few instructions instead of a 64-bit division routine each); larger values take the 64-bit path.
struct StridePos {
    int64_t q;
    int r;
    int64_t dq;
    int dr;
    int d;
    __device__ __forceinline__ StridePos(int64_t start, int64_t step, int divisor) : d(divisor) {
        if (((uint64_t)start | (uint64_t)step) <= 0xFFFFFFFFull) {
            const uint32_t s32 = (uint32_t)start, t32 = (uint32_t)step, d32 = (uint32_t)divisor;
            const uint32_t q32 = s32 / d32, dq32 = t32 / d32;
            q = q32;
            r = (int)(s32 - q32 * d32);
            dq = dq32;
            dr = (int)(t32 - dq32 * d32);
        } else {
            q = start / divisor;
            r = (int)(start - q * divisor);
            dq = step / divisor;
            dr = (int)(step - dq * divisor);
        }
    }
    __device__ __forceinline__ void advance() {
        q += dq;
        r += dr;
        if (r >= d) {
            r -= d;
            ++q;
        }
    }
};

// ----------------------------------------------------------------------------------------------
// Packed fp32 (sm_100 FFMA2 / FMUL2 / FADD2): two independent fp32 operations per instruction, each
// rounded exactly like its scalar counterpart. An 8-element vector is held as float2[4].
// ----------------------------------------------------------------------------------------------
__device__ __forceinline__ float2 splat2(float s) { return make_float2(s, s); }
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
// A packed product rounded on its own, for a following add that must see the rounded value. The
// compiler fuses a packed multiply with a following packed add into one FFMA2 even when both are
// written as PTX with .rn (measured on B200: at exact .5 ties of the product, the sum rounded the
// exact product instead). An fma with a +0 addend rounds the product exactly as a multiply does (only
// an exact -0 product comes out +0) and cannot be merged with the add.
__device__ __forceinline__ float2 fmul2_unfused(float2 a, float2 b) {
    uint64_t x, y, z, r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(a.x), "f"(a.y));
    asm("mov.b64 %0, {%1, %2};" : "=l"(y) : "f"(b.x), "f"(b.y));
    asm("mov.b64 %0, {%1, %2};" : "=l"(z) : "f"(0.0f), "f"(0.0f));
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(x), "l"(y), "l"(z));
    float2 o;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(o.x), "=f"(o.y) : "l"(r));
    return o;
}

// sum of squares of an 8-vector: two interleaved partial sums, then one add
__device__ __forceinline__ float sumsq8(const float2 (&v)[4]) {
    float2 acc = fmul2(v[0], v[0]);
#pragma unroll
    for (int i = 1; i < 4; ++i) acc = ffma2(v[i], v[i], acc);
    return acc.x + acc.y;
}

// 1/sqrt(x) with the hardware approximation (PTX rsqrt.approx, one instruction). The reference calls
// rsqrtf, also an approximate reciprocal square root; the .ftz form only differs for subnormal x,
// and here x = mean(v^2) + eps >= eps > 0 is never subnormal.
__device__ __forceinline__ float rsqrt_approx(float x) {
    float y;
    asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Logistic-function building blocks written from the identities e^x = 2^(x * log2 e) and
// a / b = a * (1 / b), on the PTX approximate base-2 exponential and reciprocal instructions
// (ex2.approx.ftz, rcp.approx.ftz; relative errors around 2^-22). For the gates here:
//   sigmoid(z) = 1 / (1 + 2^(-z * log2 e))
// which saturates correctly: z > 88 gives 2^(..) -> 0 (sigmoid 1), z < -88 gives inf (sigmoid 0).
constexpr float kLog2e = 1.4426950408889634f;
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
// sigmoid of a pair
__device__ __forceinline__ float2 sigmoid2(float2 z) {
    const float2 t = fmul2(z, splat2(-kLog2e));
    const float2 den = fadd2(splat2(1.0f), make_float2(ex2_approx(t.x), ex2_approx(t.y)));
    return make_float2(rcp_approx(den.x), rcp_approx(den.y));
}

// Q8_0-style int8 quantisation of one group of 8*kLanes elements held by kLanes consecutive lanes (8
// elements each): 32-element groups (kLanes 4) as the reference's xq8 path
// (src/wzy_kernels_v2.cuh:440-454), silu_mul_quant32_multi (:1247-1279) and quant_act_multi's q32;
// 16-element groups (kLanes 2) as quant_act_multi's q16 (:58-111). amax over the group,
// d = amax / 127, q = rint(v * (127 / amax)) clamped to [-127, 127] (q = 0 when amax = 0), d stored
// by the group's first lane. Every lane of the warp must call it (the group max is xor shuffles);
// `active` lanes store.
//
// Codes: t = fl(v * inv) (|t| <= 127 * (1 + 2^-23)^2 for finite v; rounded on its own, fmul2_unfused,
// so exact .5 ties of t stay ties), then rint(t) as the low byte of fl(t + 1.5 * 2^23), a float whose
// unit is 1 there, so the add itself is the round-to-nearest-even;
// packed FMA2 (+0 addend) and FADD2 on the FMA pipe instead of a conversion instruction per element
// (SwiGLU + Q8 80 -> 82 %, the quantiser 78 -> 81 % of HBM peak). A lane whose 8 values are not all
// finite (seen by a NaN-propagating max), or whose group max is so small (below ~3.7e-37) that
// 127 / amax overflows to infinity while amax / 127 does not underflow to 0, takes the reference's own
// conversion instead: __float2int_rn(v * inv) clamped to [-127, 127], which maps the NaN that t then is
// to 0 and t = +-inf to +-127; the group's amax drops NaNs (fmaxf) as the reference's does.
__device__ __forceinline__ float fmax_nan(float a, float b) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

// A lane's part of a Q8 group: the max |v| of its 8 values with NaNs dropped (fmaxf, as the reference)
// and whether all 8 are finite (a NaN-propagating max; false also for inf).
__device__ __forceinline__ float q8_lane_max(const float (&v)[8], bool active, bool& finite) {
    float am = 0.f;
    finite = true;
    if (active) {
#pragma unroll
        for (int i = 0; i < 8; ++i) am = fmax_nan(am, fabsf(v[i]));
        finite = am <= 3.402823466e38f;  // false for NaN and inf
        if (!finite) {
            am = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) am = fmaxf(am, fabsf(v[i]));
        }
    }
    return am;
}

// Codes and scale of a lane's 8 values given the group's max: d = am / 127 stored by the group's
// first lane (lane % kLanes == 0), 8 code bytes at q.
template <int kLanes>
__device__ __forceinline__ void q8_codes_store(const float (&v)[8], float am, bool finite, signed char* q, float* s,
                                               int lane) {
    const float d = am / 127.0f;
    const float inv = d > 0.f ? 127.0f / am : 0.f;
    uint32_t b[8];
    if (finite && inv <= 3.402823466e38f) {
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
            const float2 t = fadd2(fmul2_unfused(make_float2(v[i], v[i + 1]), splat2(inv)), splat2(12582912.0f));
            b[i] = __float_as_uint(t.x);
            b[i + 1] = __float_as_uint(t.y);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) b[i] = (uint32_t)max(-127, min(127, __float2int_rn(v[i] * inv)));
    }
    uint32_t w[2];
#pragma unroll
    for (int k = 0; k < 2; ++k)
        w[k] = __byte_perm(__byte_perm(b[4 * k], b[4 * k + 1], 0x0040), __byte_perm(b[4 * k + 2], b[4 * k + 3], 0x0040),
                           0x5410);
    *reinterpret_cast<uint2*>(q) = make_uint2(w[0], w[1]);
    if ((lane & (kLanes - 1)) == 0) *s = d;
}

template <int kLanes = 4>
__device__ __forceinline__ void q8_group_store(const float (&v)[8], bool active, signed char* q, float* s, int lane) {
    bool finite;
    float am = q8_lane_max(v, active, finite);
#pragma unroll
    for (int o = 1; o < kLanes; o <<= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    if (active) q8_codes_store<kLanes>(v, am, finite, q, s, lane);
}

// Both group sizes of quant_act_multi from one lane max: the 16-group max over 2 lanes, the 32-group
// max as the max of two 16-group maxima (max is exact in any order, so the scales are the same as
// two separate reductions).
__device__ __forceinline__ void q8_group_store_16_32(const float (&v)[8], bool active, signed char* q16, float* s16,
                                                     signed char* q32, float* s32, int lane) {
    bool finite;
    float am16 = q8_lane_max(v, active, finite);
    am16 = fmaxf(am16, __shfl_xor_sync(0xffffffffu, am16, 1));
    const float am32 = fmaxf(am16, __shfl_xor_sync(0xffffffffu, am16, 2));
    if (!active) return;
    q8_codes_store<2>(v, am16, finite, q16, s16, lane);
    q8_codes_store<4>(v, am32, finite, q32, s32, lane);
}

// Shared scale of an MXFP8 block as its E8M0 byte: X = 2^ceil(log2(amax / 448)), the smallest power
// of two that keeps every element of the block within E4M3's +-448 (OCP's floor(log2 amax) - 8 would
// clip the block maximum by up to 12.5 %). Integer work on the bits of t = amax / 448; t == 0 gives
// the smallest scale 2^-127 (byte 0), inf/NaN gives the E8M0 NaN byte 0xFF. Host-callable so the
// oracle-facing code paths agree bit for bit.
__host__ __device__ __forceinline__ uint32_t mxfp8_scale_byte(float amax) {
    const float t = amax / 448.0f;
    uint32_t tb;
    memcpy(&tb, &t, 4);
    const uint32_t et = tb >> 23;  // t >= 0
    if (et == 0xFFu) return 0xFFu;
    if (et == 0u) return tb <= 0x00400000u ? 0u : 1u;  // zero or subnormal t: 2^-127 or 2^-126
    return et + ((tb & 0x7FFFFFu) != 0u ? 1u : 0u);
}

// MXFP8 (E4M3 elements, E8M0 scale, block 32; the block-scaled MMA's MX format), one 32-element
// group over 4 consecutive lanes: scale byte e8 = mxfp8_scale_byte(amax), codes e4m3(x * 2^(127 - e8)),
// round-to-nearest-even, saturating at +-448. Every lane must call it; `active` lanes store 8 bytes.
__device__ __forceinline__ void mxfp8_group_store(const float (&v)[8], bool active, uint8_t* q, uint8_t* s,
                                                  int lane) {
    float am = 0.f;
    if (active) {
#pragma unroll
        for (int i = 0; i < 8; ++i) am = fmaxf(am, fabsf(v[i]));
    }
    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
    if (!active) return;
    const uint32_t e8 = mxfp8_scale_byte(am);
    const float inv = e8 == 0xFFu ? 0.f : __uint_as_float((254u - e8) << 23);  // 1 / X
    uint32_t w[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(v[4 * k] * inv, v[4 * k + 1] * inv), __NV_SATFINITE,
                                                     __NV_E4M3);
        const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(v[4 * k + 2] * inv, v[4 * k + 3] * inv),
                                                     __NV_SATFINITE, __NV_E4M3);
        w[k] = lo | (hi << 16);
    }
    *reinterpret_cast<uint2*>(q) = make_uint2(w[0], w[1]);
    if ((lane & 3) == 0) *s = (uint8_t)e8;
}

// NVFP4 (E2M1 elements, E4M3 block scale, block 16, plus a per-tensor scale gs), one 16-element group
// over 2 consecutive lanes. Scale byte sc = e4m3((amax * gs) / 6) (6 = the largest E2M1 value);
// codes e2m1(x * (gs / float(sc))), 0 when sc decodes to 0; round-to-nearest-even, saturating at +-6.
// A lane's 8 codes are 4 bytes, element 2i in the low nibble of byte i. Dequantisation:
// x ~= e2m1 * float(sc) / gs. Every lane must call it.
__device__ __forceinline__ void nvfp4_group_store(const float (&v)[8], bool active, float gs, uint8_t* q,
                                                  uint8_t* s, int lane) {
    float am = 0.f;
    if (active) {
#pragma unroll
        for (int i = 0; i < 8; ++i) am = fmaxf(am, fabsf(v[i]));
    }
    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
    if (!active) return;
    const __nv_fp8_storage_t sc = __nv_cvt_float_to_fp8((am * gs) / 6.0f, __NV_SATFINITE, __NV_E4M3);
    const __half_raw hr = __nv_cvt_fp8_to_halfraw(sc, __NV_E4M3);
    const float sf = __half2float(__half(hr));
    const float r = sf > 0.f ? gs / sf : 0.f;
    uint32_t w = 0u;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t b = __nv_cvt_float2_to_fp4x2(make_float2(v[2 * i] * r, v[2 * i + 1] * r), __NV_E2M1,
                                                    cudaRoundNearest);
        w |= (b & 0xFFu) << (8 * i);
    }
    *reinterpret_cast<uint32_t*>(q) = w;
    if ((lane & 1) == 0) *s = (uint8_t)sc;
}

// GEMM-input quantisation formats of the fused and standalone quantisers.
enum QuantFormat : int { kQfNone = 0, kQfQ8 = 1, kQfMxfp8 = 2, kQfNvfp4 = 3 };

// Store this lane's 8 values (flat 8-element vector index vi of the tensor) in format QF: codes at q,
// scales at s (Q8: int8 + fp32 per 32; MXFP8: e4m3 + E8M0 byte per 32; NVFP4: e2m1 pairs + E4M3 byte
// per 16, per-tensor scale gs). Every lane of the warp must call it.
template <int QF>
__device__ __forceinline__ void quant_group_store(const float (&v)[8], bool active, void* q, void* s, float gs,
                                                  int64_t vi, int lane) {
    if (QF == kQfQ8) {
        q8_group_store<4>(v, active, static_cast<signed char*>(q) + vi * 8, static_cast<float*>(s) + (vi >> 2), lane);
    } else if (QF == kQfMxfp8) {
        mxfp8_group_store(v, active, static_cast<uint8_t*>(q) + vi * 8, static_cast<uint8_t*>(s) + (vi >> 2), lane);
    } else if (QF == kQfNvfp4) {
        nvfp4_group_store(v, active, gs, static_cast<uint8_t*>(q) + vi * 4, static_cast<uint8_t*>(s) + (vi >> 1), lane);
    }
}

// Scale-factor layouts of the block formats. Row-major: scale (row, c) at row * scols + c, i.e. the flat
// element order. Tiled 128x4: the layout of sm_100's block-scaled MMA operands -- the [rows, scols]
// scale matrix cut into tiles of 128 rows x 4 scale columns, 512 bytes each, the tiles of one 128-row
// band consecutive along the scale columns (ncb = ceil(scols / 4) tiles per band), and inside a tile
// scale (r, c) at (r % 32) * 16 + (r / 32) * 4 + c.
enum ScaleLayout : int { kSfRowMajor = 0, kSfTiled128x4 = 1 };
__host__ __device__ __forceinline__ int64_t sf_tiled_offset(int64_t row, int scol, int ncb) {
    return ((row >> 7) * ncb + (scol >> 2)) * 512 + (row & 31) * 16 + ((row >> 5) & 3) * 4 + (scol & 3);
}

// The MXFP8 / NVFP4 store of quant_group_store with the group's scale byte at an explicit address
// (the group's first lane writes it), for the tiled layout.
template <int QF>
__device__ __forceinline__ void block_group_store_at(const float (&v)[8], bool active, void* q, uint8_t* s_at,
                                                     float gs, int64_t vi, int lane) {
    if (QF == kQfMxfp8) {
        mxfp8_group_store(v, active, static_cast<uint8_t*>(q) + vi * 8, s_at, lane);
    } else if (QF == kQfNvfp4) {
        nvfp4_group_store(v, active, gs, static_cast<uint8_t*>(q) + vi * 4, s_at, lane);
    }
}

// Sum over aligned groups of `kLanes` lanes (kLanes a power of two <= 32) with xor shuffles.
template <int kLanes>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
    for (int o = kLanes / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Named barrier among `nthreads` threads (a multiple of 32), id 1..15 (0 is __syncthreads).
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

}  // namespace wzyb
