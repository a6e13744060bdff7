// gather.cu -- token-embedding gather and 16-head 3-gram PLE gather (bit-exact row copies).
//
// The reference stages both on the host: stage_one_emb (src/wzy_engine_v2.cu:862-875) copies one
// bf16 row per token and converts it to fp32, and stage_ple_window / stage_emb_ple_pf
// (src/wzy_engine_v2.cu:943-978, :1210-1265) hash each token's 3-gram context into 16 rows and copy
// them, then H2D the result. Its only device gather, mtp_gather_bf16_emb (src/wzy_kernels_v2.cuh:27-36),
// reads 2-byte elements with a 256-thread block per token. Here both gathers run on the device:
// a warp (embedding) or a lane group (PLE) per row, 16-byte accesses, several row chunks in flight
// per lane before any store.
#include "launch.hpp"
#include "common.cuh"

namespace wzyb {

constexpr int kGatherThreads = 256;
constexpr int kRowUnroll = 8;  // 16-byte chunks in flight per lane

__device__ __forceinline__ int64_t resolve_id(int32_t id, int64_t vocab, int policy, uint32_t* oob, int lane) {
    if (id >= 0 && id < vocab) return id;
    if (oob != nullptr && lane == 0) atomicAdd(oob, 1u);
    if (policy == WZYB_OOB_ZERO_ID) return 0;
    return id < 0 ? 0 : vocab - 1;
}

struct EmbedArgs {
    const uint4* table;
    int64_t vocab;
    int64_t row_chunks;  // 16-byte chunks per row
    const int32_t* ids;
    int64_t T;
    uint4* out;
    int policy;
    uint32_t* oob;
};

// One warp per output row: out[t] = table[id(t)], row_chunks 16-byte chunks per row. The body takes
// its CTA's index among `nctas` CTAs that share the rows (a fused bundle kernel runs it on a subset of
// its grid).
__device__ __forceinline__ void gather_rows_body(const EmbedArgs& a, int cta, int nctas) {
    const uint4* __restrict__ table = a.table;
    const int32_t* __restrict__ ids = a.ids;
    uint4* __restrict__ out = a.out;
    const int64_t vocab = a.vocab, row_chunks = a.row_chunks, T = a.T;
    const int policy = a.policy;
    uint32_t* oob = a.oob;
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)nctas * (blockDim.x >> 5);
    for (int64_t t = (int64_t)cta * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T; t += warps) {
        const int64_t id = resolve_id(__ldg(ids + t), vocab, policy, oob, lane);
        const uint4* src = table + id * row_chunks;
        uint4* dst = out + t * row_chunks;
        for (int64_t c0 = lane; c0 < row_chunks; c0 += 32 * kRowUnroll) {
            uint4 buf[kRowUnroll];
#pragma unroll
            for (int k = 0; k < kRowUnroll; ++k)
                if (c0 + 32 * k < row_chunks) buf[k] = __ldg(src + c0 + 32 * k);
#pragma unroll
            for (int k = 0; k < kRowUnroll; ++k)
                if (c0 + 32 * k < row_chunks) __stcs(dst + c0 + 32 * k, buf[k]);
        }
    }
}

__global__ void __launch_bounds__(kGatherThreads) gather_rows_kernel(const EmbedArgs a) {
    pdl_begin();
    gather_rows_body(a, blockIdx.x, gridDim.x);
}

// Validates an embedding-gather call on the host and fills `a`. Returns WZYB_OK or the WZYB_ERR_* of the
// first bad argument; nothing is enqueued.
static int embed_prepare(const void* table, int64_t vocab, int64_t row_bytes, const int32_t* ids, int64_t T,
                         void* out, int oob_policy, uint32_t* d_oob_count, EmbedArgs& a) {
    if (!table || !ids || !out) return WZYB_ERR_NULL;
    if (oob_policy != WZYB_OOB_CLAMP && oob_policy != WZYB_OOB_ZERO_ID) return WZYB_ERR_VALUE;
    if (vocab < 1 || T < 0 || row_bytes < 16 || (row_bytes % 16) != 0) return WZYB_ERR_SHAPE;
    if (!aligned16(table) || !aligned16(out)) return WZYB_ERR_ALIGN;
    a.table = (const uint4*)table;
    a.vocab = vocab;
    a.row_chunks = row_bytes / 16;
    a.ids = ids;
    a.T = T;
    a.out = (uint4*)out;
    a.policy = oob_policy;
    a.oob = d_oob_count;
    return WZYB_OK;
}

// bf16 table -> fp32 rows: each lane converts 8 bf16 (16 B in) to 8 fp32 (32 B out) by shifting the
// bit pattern into the high half, which is exactly the reference's db2f (src/wzy_kernels_v2.cuh:23).
__global__ void __launch_bounds__(kGatherThreads) gather_bf16_f32_kernel(const uint4* __restrict__ table,
                                                                          int64_t vocab, int64_t row_chunks,
                                                                          const int32_t* __restrict__ ids, int64_t T,
                                                                          uint4* __restrict__ out, int policy,
                                                                          uint32_t* oob) {
    pdl_begin();
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T; t += warps) {
        const int64_t id = resolve_id(__ldg(ids + t), vocab, policy, oob, lane);
        const uint4* src = table + id * row_chunks;
        uint4* dst = out + t * row_chunks * 2;
        for (int64_t c0 = lane; c0 < row_chunks; c0 += 32 * kRowUnroll) {
            uint4 buf[kRowUnroll];
#pragma unroll
            for (int k = 0; k < kRowUnroll; ++k)
                if (c0 + 32 * k < row_chunks) buf[k] = __ldg(src + c0 + 32 * k);
#pragma unroll
            for (int k = 0; k < kRowUnroll; ++k) {
                const int64_t c = c0 + 32 * k;
                if (c < row_chunks) {
                    const uint4 b = buf[k];
                    const uint4 lo = make_uint4(b.x << 16, b.x & 0xFFFF0000u, b.y << 16, b.y & 0xFFFF0000u);
                    const uint4 hi = make_uint4(b.z << 16, b.z & 0xFFFF0000u, b.w << 16, b.w & 0xFFFF0000u);
                    __stcs(dst + 2 * c, lo);
                    __stcs(dst + 2 * c + 1, hi);
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------
// PLE
// ---------------------------------------------------------------------------------------------
__host__ __device__ __forceinline__ uint32_t ple_row(int32_t t0, int32_t h1, int32_t h2, int head, uint64_t rows,
                                                     int32_t eos, int variant) {
    // EOS cut over the history, as the reference builds ctx[1..2] (src/wzy_engine_v2.cu:946-953):
    // once an id is negative or EOS, it and every older id become EOS.
    bool cut = h1 < 0 || h1 == eos;
    const int32_t c1 = cut ? eos : h1;
    cut = cut || h2 < 0 || h2 == eos;
    const int32_t c2 = cut ? eos : h2;
    const uint32_t a = (uint32_t)t0 * 0x9E3779B1u;
    const uint32_t b = (uint32_t)c1 * 0x85EBCA77u;
    const uint32_t c = (uint32_t)c2 * 0xC2B2AE3Du;
    const uint32_t h = variant == WZYB_PLE_HASH_XOR_THEN_ADD ? ((a ^ b ^ c) + (uint32_t)head)
                                                             : (a ^ b ^ (c + (uint32_t)head));
    return (uint32_t)((uint64_t)h % rows);
}

// Same index with the modulo specialised: rows_mask = rows - 1 when rows is a power of two.
__device__ __forceinline__ uint32_t ple_row_fast(int32_t t0, int32_t h1, int32_t h2, int head, uint64_t rows,
                                                 uint32_t rows_mask, int32_t eos, int variant) {
    bool cut = h1 < 0 || h1 == eos;
    const int32_t c1 = cut ? eos : h1;
    cut = cut || h2 < 0 || h2 == eos;
    const int32_t c2 = cut ? eos : h2;
    const uint32_t a = (uint32_t)t0 * 0x9E3779B1u;
    const uint32_t b = (uint32_t)c1 * 0x85EBCA77u;
    const uint32_t c = (uint32_t)c2 * 0xC2B2AE3Du;
    const uint32_t h = variant == WZYB_PLE_HASH_XOR_THEN_ADD ? ((a ^ b ^ c) + (uint32_t)head)
                                                             : (a ^ b ^ (c + (uint32_t)head));
    if (rows_mask != 0u || rows == 1) return h & rows_mask;
    if (rows > 0xFFFFFFFFull) return h;  // every 32-bit hash value is a valid row
    return h % (uint32_t)rows;
}

struct PleArgs {
    const uint4* tables[32];
    int heads;
    uint64_t rows;
    uint32_t rows_mask;  // rows - 1 when rows is a power of two, else 0
    int chunks;  // 16-byte chunks per head row
    const int32_t* ids;
    int64_t T;
    int32_t prev2;  // id[-2]
    int32_t prev1;  // id[-1]
    int32_t eos;
    int variant;
    uint4* out;  // [T, heads * chunks]
};

// Flattened over (token, head, chunk); each thread keeps kRowUnroll chunks in flight.
__global__ void __launch_bounds__(kGatherThreads) ple_gather_kernel(const PleArgs a) {
    pdl_begin();
    const int64_t per_tok = (int64_t)a.heads * a.chunks;
    const int64_t total = a.T * per_tok;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t base = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; base < total; base += stride * kRowUnroll) {
        uint4 buf[kRowUnroll];
        int64_t dsti[kRowUnroll];
#pragma unroll
        for (int k = 0; k < kRowUnroll; ++k) {
            const int64_t idx = base + k * stride;
            dsti[k] = idx;
            if (idx < total) {
                const int64_t t = idx / per_tok;
                const int rem = (int)(idx - t * per_tok);
                const int h = rem / a.chunks;
                const int c = rem - h * a.chunks;
                const int32_t t0 = __ldg(a.ids + t);
                const int32_t h1 = t >= 1 ? __ldg(a.ids + t - 1) : a.prev1;
                const int32_t h2 = t >= 2 ? __ldg(a.ids + t - 2) : (t == 1 ? a.prev1 : a.prev2);
                const uint32_t row = ple_row(t0, h1, h2, h, a.rows, a.eos, a.variant);
                buf[k] = __ldg(a.tables[h] + (int64_t)row * a.chunks + c);
            }
        }
#pragma unroll
        for (int k = 0; k < kRowUnroll; ++k)
            if (dsti[k] < total) __stcs(a.out + dsti[k], buf[k]);
    }
}

// Fast path when a head row is CH = 8, 16 or 32 chunks of 16 bytes: a group of CH lanes copies one
// (token, head) row, 32/CH groups per warp, U rows in flight per group. The (token, head) position
// is stepped without division and the row index uses a mask for power-of-two tables.
// The body takes its CTA's index among `nctas` CTAs that share the rows (a fused bundle kernel runs it
// on a subset of its grid).
template <int CH, int U>
__device__ __forceinline__ void ple_gather_groups_body(const PleArgs& a, int cta, int nctas) {
    constexpr int GPW = 32 / CH;
    const int lane = threadIdx.x & 31;
    const int c = lane % CH;
    const int64_t ngroups = (int64_t)nctas * (blockDim.x >> 5) * GPW;
    const int64_t ggrp = ((int64_t)cta * (blockDim.x >> 5) + (threadIdx.x >> 5)) * GPW + lane / CH;
    const int64_t items = a.T * a.heads;
    StridePos pos(ggrp, ngroups, a.heads);  // item it = (token q, head r)
    for (int64_t base = ggrp; base < items; base += ngroups * U) {
        uint4 buf[U];
        int64_t dst[U];
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const int64_t it = base + k * ngroups;
            dst[k] = -1;
            if (it < items) {
                const int64_t t = pos.q;
                const int h = pos.r;
                const int32_t t0 = __ldg(a.ids + t);
                const int32_t h1 = t >= 1 ? __ldg(a.ids + t - 1) : a.prev1;
                const int32_t h2 = t >= 2 ? __ldg(a.ids + t - 2) : (t == 1 ? a.prev1 : a.prev2);
                const uint32_t row = ple_row_fast(t0, h1, h2, h, a.rows, a.rows_mask, a.eos, a.variant);
                buf[k] = __ldg(a.tables[h] + (int64_t)row * CH + c);
                dst[k] = it * CH + c;
            }
            pos.advance();
        }
#pragma unroll
        for (int k = 0; k < U; ++k)
            if (dst[k] >= 0) __stcs(a.out + dst[k], buf[k]);
    }
}

template <int CH, int U>
__global__ void __launch_bounds__(kGatherThreads) ple_gather_groups_kernel(const PleArgs a) {
    pdl_begin();
    ple_gather_groups_body<CH, U>(a, blockIdx.x, gridDim.x);
}

// Validates a PLE-gather call on the host and fills `a` (the table pointers are read from the host
// array `tables`). Returns WZYB_OK or the WZYB_ERR_* of the first bad argument; nothing is enqueued.
static int ple_prepare(const uint16_t* const* tables, int heads, int64_t rows_per_table, int head_dim,
                       const int32_t* ids, int64_t T, const int32_t* prev_ids, int32_t eos_id, int hash_variant,
                       uint16_t* out, PleArgs& a) {
    if (!tables || !ids || !out) return WZYB_ERR_NULL;
    if (hash_variant != WZYB_PLE_HASH_C_PRECEDENCE && hash_variant != WZYB_PLE_HASH_XOR_THEN_ADD)
        return WZYB_ERR_VALUE;
    if (heads < 1 || heads > 32 || rows_per_table < 1 || rows_per_table > (int64_t(1) << 32) || head_dim < 8 ||
        (head_dim % 8) != 0 || T < 0)
        return WZYB_ERR_SHAPE;
    for (int h = 0; h < 32; ++h) a.tables[h] = nullptr;
    for (int h = 0; h < heads; ++h) {
        if (!tables[h]) return WZYB_ERR_NULL;
        if (!aligned16(tables[h])) return WZYB_ERR_ALIGN;
        a.tables[h] = (const uint4*)tables[h];
    }
    if (!aligned16(out)) return WZYB_ERR_ALIGN;
    a.heads = heads;
    a.rows = (uint64_t)rows_per_table;
    a.chunks = head_dim / 8;
    a.ids = ids;
    a.T = T;
    a.prev2 = prev_ids ? prev_ids[0] : -1;
    a.prev1 = prev_ids ? prev_ids[1] : -1;
    a.eos = eos_id;
    a.variant = hash_variant;
    a.out = (uint4*)out;
    a.rows_mask = (rows_per_table & (rows_per_table - 1)) == 0 ? (uint32_t)(rows_per_table - 1) : 0u;
    return WZYB_OK;
}

// ---------------------------------------------------------------------------------------------
// Bulk design (TMA): both gathers as 1-D bulk copies through shared memory, no data in registers.
//
// A warp owns a ring of S shared-memory slots with one mbarrier each. For each of its units -- a
// token's embedding row, or a token's `heads` PLE rows, which land side by side in the slot exactly
// as they sit in the output row -- it issues bulk loads (cp.async.bulk global -> shared, completion
// counted on the slot's mbarrier: one load per row, the PLE rows' loads from `heads` lanes at once),
// then, once the slot is full, one bulk store of the whole output row (cp.async.bulk shared -> global,
// a bulk async-group). A slot is refilled with the unit S ahead after the store that read it has
// finished reading (wait_group.read), one unit behind the newest store. The ids of the warp's next
// 32 units are loaded up front, one unit per lane, and broadcast by shuffle, so issuing a unit waits
// on no global load. With S slots per warp, S units per warp are in flight: at 4096 tokens nearly
// every row of the call is requested at once, which the register designs cannot hold.
// Every wait is bounded; a warp whose wait gives up raises WZYB_FAULT_WAIT_TIMEOUT, drains the loads
// it issued (bounded) and its stores, and stops.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void bulk_store(void* gdst, const void* ssrc, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(smem_u32(ssrc)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// all but the newest N bulk groups of this thread have finished reading their shared memory
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// order this thread's generic-proxy view of shared memory before its later async-proxy operations
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

constexpr int kBulkWarps = 4;                 // warps per CTA, each with its own ring
constexpr uint32_t kBulkMaxSlot = 16 * 1024;  // largest unit (output row) the bulk design stages

struct BulkGatherArgs {
    EmbedArgs e;      // token rows (e.T == 0: none)
    PleArgs p;        // PLE rows of the same ids (p.T == 0: none)
    int64_t units;    // e.T + p.T
    uint32_t slot_bytes;
    int stages;       // slots per warp
};

__global__ void __launch_bounds__(kBulkWarps * 32) gather_bulk_kernel(const BulkGatherArgs a) {
    pdl_begin();
    extern __shared__ __align__(128) unsigned char smem_bg[];
    const int S = a.stages;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem_bg) + warp * S;
    unsigned char* ring = smem_bg + ((kBulkWarps * S * 8 + 127) & ~127) + (size_t)warp * S * a.slot_bytes;
    const int64_t GW = (int64_t)gridDim.x * kBulkWarps;
    const int64_t gw = (int64_t)blockIdx.x * kBulkWarps + warp;
    if (gw >= a.units) return;  // warp-uniform; this warp has no unit
    const int64_t nmine = (a.units - 1 - gw) / GW + 1;
    const int64_t Te = a.e.T;
    const uint32_t erow = (uint32_t)(a.e.row_chunks * 16), hbytes = (uint32_t)(a.p.chunks * 16);
    const uint32_t prow = hbytes * (uint32_t)a.p.heads;

    if (lane == 0) {
        for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    __syncwarp();
    const uint64_t pol = policy_evict_first();

    // ids of units [32c, 32c + 32) of this warp, one unit per lane: (t0, h1, h2) of its token
    int32_t my_t0 = 0, my_h1 = 0, my_h2 = 0;
    int64_t chunk = -1;
    auto load_ids = [&](int64_t c) {
        const int64_t k = c * 32 + lane;
        if (k < nmine) {
            const int64_t u = gw + k * GW;
            const int64_t t = u < Te ? u : u - Te;
            my_t0 = __ldg(a.e.ids + t);
            if (u >= Te) {
                my_h1 = t >= 1 ? __ldg(a.e.ids + t - 1) : a.p.prev1;
                my_h2 = t >= 2 ? __ldg(a.e.ids + t - 2) : (t == 1 ? a.p.prev1 : a.p.prev2);
            }
        }
        chunk = c;
    };
    // issue the loads of unit k into slot k % S (warp-collective)
    auto issue = [&](int64_t k) {
        if (k / 32 != chunk) load_ids(k / 32);
        const int src = (int)(k & 31);
        const int32_t t0 = __shfl_sync(0xffffffffu, my_t0, src);
        const int32_t h1 = __shfl_sync(0xffffffffu, my_h1, src);
        const int32_t h2 = __shfl_sync(0xffffffffu, my_h2, src);
        const int64_t u = gw + k * GW;
        const int s = (int)(k % S);
        unsigned char* slot = ring + (size_t)s * a.slot_bytes;
        if (u < Te) {
            if (lane == 0) {
                const int64_t id = resolve_id(t0, a.e.vocab, a.e.policy, a.e.oob, 0);
                mbar_arrive_expect_tx(&bars[s], erow);
                bulk_load(slot, reinterpret_cast<const unsigned char*>(a.e.table) + id * erow, erow, &bars[s], pol);
            }
        } else {
            if (lane == 0) mbar_arrive_expect_tx(&bars[s], prow);
            __syncwarp();
            for (int h = lane; h < a.p.heads; h += 32) {
                const uint32_t row = ple_row_fast(t0, h1, h2, h, a.p.rows, a.p.rows_mask, a.p.eos, a.p.variant);
                bulk_load(slot + (size_t)h * hbytes,
                          reinterpret_cast<const unsigned char*>(a.p.tables[h]) + (size_t)row * hbytes, hbytes,
                          &bars[s], pol);
            }
        }
    };

    const int64_t pre = nmine < S ? nmine : (int64_t)S;
    for (int64_t k = 0; k < pre; ++k) issue(k);
    int64_t issued = pre;
    bool ok = true;
    int64_t k = 0;
    for (; k < nmine; ++k) {
        const int s = (int)(k % S);
        if (lane == 0) ok = mbar_wait(&bars[s], (uint32_t)((k / S) & 1));
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
        const int64_t u = gw + k * GW;
        if (lane == 0) {
            fence_proxy_async_smem();
            if (u < Te) bulk_store(reinterpret_cast<unsigned char*>(a.e.out) + u * erow, ring + (size_t)s * a.slot_bytes, erow);
            else bulk_store(reinterpret_cast<unsigned char*>(a.p.out) + (u - Te) * prow, ring + (size_t)s * a.slot_bytes, prow);
            bulk_commit();
            bulk_wait_read<1>();  // the store of unit k - 1 has read its slot
        }
        __syncwarp();
        // refill the slot of unit k - 1 with unit k - 1 + S (the first slot is refilled one unit late)
        if (k >= 1 && issued < nmine) {
            issue(issued);
            ++issued;
        }
    }
    if (!ok) {
        // drain the loads that were issued but not consumed, then stop
        if (lane == 0) {
            const unsigned long long deadline = globaltimer_ns() + kWaitLimitNs;
            for (int64_t i = k; i < issued; ++i)
                if (!mbar_wait_until(&bars[i % S], (uint32_t)((i / S) & 1), deadline)) break;
        }
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
}

// Launch of the bulk design over an embedding gather (e.T > 0) and/or a PLE gather (p.T > 0) of the
// same ids. Returns WZYB_OK, a launch status, or WZYB_ERR_SHAPE when a unit does not fit a slot.
static int gather_bulk_launch(const EmbedArgs& e, const PleArgs& p, cudaStream_t stream) {
    BulkGatherArgs a;
    a.e = e;
    a.p = p;
    a.units = e.T + p.T;
    if (a.units == 0) return WZYB_OK;
    const uint32_t erow = e.T > 0 ? (uint32_t)(e.row_chunks * 16) : 0u;
    const uint32_t prow = p.T > 0 ? (uint32_t)(p.chunks * 16 * p.heads) : 0u;
    const uint32_t unit = erow > prow ? erow : prow;
    if (unit == 0 || unit > kBulkMaxSlot) return WZYB_ERR_SHAPE;
    a.slot_bytes = (unit + 127u) & ~127u;
    DeviceInfo di;
    int rc = device_info(&di);
    if (rc != WZYB_OK) return rc;
    const Tuning tu = tuning(kFamGather);
    int ctas_per_sm = tu.ctas_per_sm >= 1 && tu.ctas_per_sm <= 4 ? tu.ctas_per_sm : 1;
    while (ctas_per_sm > 1 && kSmemPerSm / ctas_per_sm / kBulkWarps / (int)a.slot_bytes < 2) --ctas_per_sm;
    int stages = (int)(kSmemPerSm / ctas_per_sm / kBulkWarps / a.slot_bytes);
    if (tu.stages > 0 && tu.stages < stages) stages = tu.stages;
    if (stages < 2) return WZYB_ERR_SHAPE;
    // no more slots than units per warp at one CTA per SM
    const int64_t per_warp = (a.units + (int64_t)di.sms * kBulkWarps - 1) / ((int64_t)di.sms * kBulkWarps);
    if (per_warp < stages) stages = per_warp < 2 ? 2 : (int)per_warp;
    a.stages = stages;
    const int smem = ((kBulkWarps * stages * 8 + 127) & ~127) + kBulkWarps * stages * (int)a.slot_bytes;
    rc = ensure_smem((const void*)gather_bulk_kernel, smem);
    if (rc != WZYB_OK) return rc;
    const int grid = persistent_grid(di, ctas_per_sm, (a.units + kBulkWarps - 1) / kBulkWarps);
    launch_k(gather_bulk_kernel, grid, kBulkWarps * 32, (size_t)smem, stream, a);
    return launch_status();
}

static int grid_for(int64_t work_threads, int ctas_per_sm, const DeviceInfo& di) {
    return persistent_grid(di, ctas_per_sm, (work_threads + kGatherThreads - 1) / kGatherThreads);
}

}  // namespace wzyb

extern "C" {

int wzyb_embed_gather_rows(const void* table, int64_t vocab, int64_t row_bytes, const int32_t* ids, int64_t T,
                           void* out, int oob_policy, uint32_t* d_oob_count, wzyb_stream_t stream) {
    wzyb::EmbedArgs a;
    int rc = wzyb::embed_prepare(table, vocab, row_bytes, ids, T, out, oob_policy, d_oob_count, a);
    if (rc != WZYB_OK || T == 0) return rc;
    if (wzyb::variant(wzyb::kFamGather) == WZYB_VARIANT_RING && row_bytes <= wzyb::kBulkMaxSlot) {
        wzyb::PleArgs none = {};
        return wzyb::gather_bulk_launch(a, none, (cudaStream_t)stream);
    }
    wzyb::DeviceInfo di;
    rc = wzyb::device_info(&di);
    if (rc != WZYB_OK) return rc;
    const int grid = wzyb::grid_for(T * 32, 8, di);
    wzyb::launch_k(wzyb::gather_rows_kernel, grid, wzyb::kGatherThreads, 0, (cudaStream_t)stream, a);
    return wzyb::launch_status();
}

int wzyb_embed_gather_f16(const uint16_t* table, int64_t vocab, int hidden, const int32_t* ids, int64_t T,
                          uint16_t* out, int oob_policy, uint32_t* d_oob_count, wzyb_stream_t stream) {
    if (hidden < 8 || (hidden % 8) != 0) return WZYB_ERR_SHAPE;
    return wzyb_embed_gather_rows(table, vocab, (int64_t)hidden * 2, ids, T, out, oob_policy, d_oob_count, stream);
}

int wzyb_embed_gather_bf16_f32(const uint16_t* table, int64_t vocab, int hidden, const int32_t* ids, int64_t T,
                               float* out, int oob_policy, uint32_t* d_oob_count, wzyb_stream_t stream) {
    if (!table || !ids || !out) return WZYB_ERR_NULL;
    if (oob_policy != WZYB_OOB_CLAMP && oob_policy != WZYB_OOB_ZERO_ID) return WZYB_ERR_VALUE;
    if (vocab < 1 || T < 0 || hidden < 8 || (hidden % 8) != 0) return WZYB_ERR_SHAPE;
    if (!wzyb::aligned16(table) || !wzyb::aligned16(out)) return WZYB_ERR_ALIGN;
    if (T == 0) return WZYB_OK;
    wzyb::DeviceInfo di;
    const int rc = wzyb::device_info(&di);
    if (rc != WZYB_OK) return rc;
    const int grid = wzyb::grid_for(T * 32, 8, di);
    wzyb::launch_k(wzyb::gather_bf16_f32_kernel, grid, wzyb::kGatherThreads, 0, (cudaStream_t)stream, 
        (const uint4*)table, vocab, hidden / 8, ids, T, (uint4*)out, oob_policy, d_oob_count);
    return wzyb::launch_status();
}

uint32_t wzyb_ple_row_index(int32_t t0, int32_t t1, int32_t t2, int head, int64_t rows_per_table, int32_t eos_id,
                            int hash_variant) {
    if (rows_per_table < 1) return 0;
    return wzyb::ple_row(t0, t1, t2, head, (uint64_t)rows_per_table, eos_id, hash_variant);
}

int wzyb_ple_gather_f16(const uint16_t* const* tables, int heads, int64_t rows_per_table, int head_dim,
                        const int32_t* ids, int64_t T, const int32_t* prev_ids, int32_t eos_id, int hash_variant,
                        uint16_t* out, wzyb_stream_t stream) {
    wzyb::PleArgs a;
    int rc = wzyb::ple_prepare(tables, heads, rows_per_table, head_dim, ids, T, prev_ids, eos_id, hash_variant, out, a);
    if (rc != WZYB_OK || T == 0) return rc;
    if (wzyb::variant(wzyb::kFamGather) == WZYB_VARIANT_RING && (int64_t)head_dim * 2 * heads <= wzyb::kBulkMaxSlot) {
        // the bulk design reads the ids through EmbedArgs; no token rows
        wzyb::EmbedArgs none = {};
        none.ids = ids;
        return wzyb::gather_bulk_launch(none, a, (cudaStream_t)stream);
    }
    wzyb::DeviceInfo di;
    rc = wzyb::device_info(&di);
    if (rc != WZYB_OK) return rc;
    if (a.chunks == 8 || a.chunks == 16 || a.chunks == 32) {
        // 2 rows in flight per lane group and correspondingly more groups (vs 8): 4.96 -> 6.12 TB/s at
        // 262,144 tokens x 16 heads, 4.60 -> 5.72 TB/s at 65,536, 14.1 -> 12.3 us at 4096 tokens
        constexpr int kU = 2;
        cudaStream_t s = (cudaStream_t)stream;
        const int grid = wzyb::grid_for(T * heads * (int64_t)a.chunks / kU, 8, di);
        if (a.chunks == 8) wzyb::launch_k(wzyb::ple_gather_groups_kernel<8, kU>, grid, wzyb::kGatherThreads, 0, s, a);
        else if (a.chunks == 16) wzyb::launch_k(wzyb::ple_gather_groups_kernel<16, kU>, grid, wzyb::kGatherThreads, 0, s, a);
        else wzyb::launch_k(wzyb::ple_gather_groups_kernel<32, kU>, grid, wzyb::kGatherThreads, 0, s, a);
        return wzyb::launch_status();
    }
    const int64_t total = T * heads * (int64_t)a.chunks;
    const int grid = wzyb::grid_for((total + wzyb::kRowUnroll - 1) / wzyb::kRowUnroll, 8, di);
    wzyb::launch_k(wzyb::ple_gather_kernel, grid, wzyb::kGatherThreads, 0, (cudaStream_t)stream, a);
    return wzyb::launch_status();
}

}  // extern "C"
