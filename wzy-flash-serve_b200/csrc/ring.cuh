// ring.cuh -- the row-streaming pipeline shared by the norm kernels.
//
// Shape of every kernel built on it: a persistent grid (a few CTAs per SM); CTA b owns the units
// b, b+G, b+2G, ... (G = gridDim.x), so every SM gets the same number of units to within one.
// Thread 0 keeps up to S units in flight with 1-D TMA bulk copies (cp.async.bulk) into an S-deep
// ring of shared-memory stages, each completed on its own mbarrier. All threads consume: wait on
// the stage's mbarrier, read the unit from shared memory into registers, and meet at one
// __syncthreads per unit; after that barrier the stage is free and thread 0 refills it with unit
// i+S. Outputs go straight from registers to HBM with 16-byte stores, so every input byte crosses
// HBM once and every output byte once.
//
// Every wait is bounded. A thread whose wait gives up marks the CTA aborted before the barrier,
// all threads leave together after it, and thread 0 drains the copies still in flight (bounded).
#pragma once
#include "common.cuh"

namespace wzyb {

struct RingSmem {
    uint64_t* full;       // [S] mbarriers
    float* red;           // [2][32] per-warp partials (double-buffered by unit parity)
    int* abort_flag;      // CTA-wide abort
    unsigned char* data;  // [S][stage_bytes]
};

// Shared-memory layout: S mbarriers, 64 floats, one int, padding to 128 B, then the stages.
__host__ __device__ constexpr uint32_t ring_header_bytes(int stages) {
    return ((uint32_t)stages * 8u + 64u * 4u + 16u + 127u) & ~127u;
}

__device__ __forceinline__ RingSmem ring_carve(unsigned char* smem, int stages) {
    RingSmem r;
    r.full = reinterpret_cast<uint64_t*>(smem);
    r.red = reinterpret_cast<float*>(smem + stages * 8);
    r.abort_flag = reinterpret_cast<int*>(smem + stages * 8 + 64 * 4);
    r.data = smem + ring_header_bytes(stages);
    return r;
}

__device__ __forceinline__ void ring_init(const RingSmem& r, int stages) {
    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) mbar_init(&r.full[s], 1);
        *r.abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
}

// Drain: wait (bounded, shared deadline) for the copies of units [from, to) that were issued but
// not consumed, so the CTA never exits while a bulk copy is still writing its shared memory.
__device__ __forceinline__ void ring_drain(const RingSmem& r, int stages, int64_t from, int64_t to) {
    if (threadIdx.x != 0) return;
    const unsigned long long deadline = globaltimer_ns() + kWaitLimitNs;
    for (int64_t i = from; i < to; ++i) {
        if (!mbar_wait_until(&r.full[i % stages], (uint32_t)((i / stages) & 1), deadline)) break;
    }
}

}  // namespace wzyb
