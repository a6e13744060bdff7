// ple_block.cu -- the reference model's per-layer-embedding (PLE) path in its own format.
//
//   fp8 gather  16 rows of fp8 e4m3 per token, picked by the reference's 2-gram / 3-gram u64 hash,
//               decoded times a global scale into fp32 [T, 16 * row_bytes].
//               Hash and cut rule: stage_ple_window (src/wzy_engine_v2.cu:943-978, constants :909-916);
//               row decode: PleSrc (src/wzy_stage_v2.cuh:215-324, fp8 table :278-285).
//   gate        gv[t,c,:] = value[t,:] * sigmoid(sign(d) * sqrt(max(|d|, 1e-6))),
//               d = dot(key[t,c,:], query[t,c,:]) / sqrt(n)       ple_gate_gv_multi (src/wzy_kernels_v2.cuh:1321-1346)
//   conv        4-tap causal conv of dilation 3 over time per channel, history of 9 inputs carried
//               between calls, SiLU, added into R with gv            ple_conv_multi (src/wzy_kernels_v2.cuh:1348-1373)
// (the block's RMSNorms, ple_group_multi, are the norm family's no-add form.)
//
// The reference stages the PLE rows on the host (a hash + an 84 MB direct-mapped row cache + an
// H2D copy per window). Here the 51 GB fp8 table sits in HBM and a warp per 4 heads of a token
// hashes them (one lane each) and streams their 4 rows. ple_conv_multi walks T sequentially per channel
// (10,240 threads); its output does not feed back, so here a thread takes 4 channels of 4 tokens
// spaced by the dilation (or of one token, when the per-token history snapshots are written).
#include <cuda_fp8.h>

#include "launch.hpp"
#include "common.cuh"

namespace wzyb {

// ---- fp8 PLE gather -----------------------------------------------------------------------------
constexpr int kPleHeads = 16;  // 8 heads per n-gram order, orders 2 and 3
constexpr int kPleHpn = 8;
constexpr int kPleQuads = 20;  // 4-byte loads per lane in flight

struct PleFp8Args {
    const uint8_t* table;
    int row_bytes;
    float scale;
    uint64_t mult[3];
    uint64_t vocab[kPleHeads];
    uint64_t off[kPleHeads];
    uint64_t recip[kPleHeads];  // floor((2^64 - 1) / vocab[h]), for mod_u64 (set on the host)
    const int32_t* ids;
    int64_t T;
    int32_t prev2, prev1;  // id[-2], id[-1] (negative: none)
    int32_t eos;
    float* out;
};

// Row of head h for token t (the reference's context and cut rule, then the u64 mix of order n).
__device__ __forceinline__ uint32_t ple_fp8_row(const PleFp8Args& a, int64_t t, int h) {
    const int32_t cur = a.ids[t];
    const int32_t p1 = t >= 1 ? a.ids[t - 1] : a.prev1;
    const int32_t p0 = t >= 2 ? a.ids[t - 2] : (t == 1 ? a.prev1 : a.prev2);
    int64_t c1, c2;
    bool cut = p1 < 0 || p1 == a.eos;
    c1 = cut ? a.eos : p1;
    cut = cut || p0 < 0 || p0 == a.eos;
    c2 = cut ? a.eos : p0;
    uint64_t mixed = (uint64_t)(int64_t)cur * a.mult[0] ^ (uint64_t)c1 * a.mult[1];
    if (h >= kPleHpn) mixed ^= (uint64_t)c2 * a.mult[2];
    return (uint32_t)(mod_u64(mixed, a.vocab[h], a.recip[h]) + a.off[h]);
}

// 4 fp8 e4m3 bytes (little-endian in a u32) -> 4 fp32 values times the scale. e4m3 -> fp16 is exact
// (hardware convert); the NaN codes (0x7F, 0xFF) read as signed zero, as in the reference's table.
// The NaN bytes are found four at a time: (b & 0x7F) + 1 carries into bit 7 exactly when the low seven
// bits are all ones (no carry crosses a byte), and clearing their low seven bits leaves the sign: 0x7F ->
// 0x00 (+0), 0xFF -> 0x80 (-0). Each zero then times the scale is the same signed zero as before.
__device__ __forceinline__ float4 fp8x4_decode(uint32_t w, float scale) {
    const uint32_t nan = ((w & 0x7F7F7F7Fu) + 0x01010101u) & 0x80808080u;
    w &= ~(nan - (nan >> 7));
    float2 f[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const __nv_fp8x2_storage_t pair = (__nv_fp8x2_storage_t)((w >> (16 * j)) & 0xFFFFu);
        const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(pair, __NV_E4M3);
        __half2 h2;
        *reinterpret_cast<__half2_raw*>(&h2) = hr;
        f[j] = fmul2(__half22float2(h2), splat2(scale));
    }
    return make_float4(f[0].x, f[0].y, f[1].x, f[1].y);
}

// One warp per item of HPI heads of a token (HPI = 16: the whole token): lanes 0..HPI-1 hash one head
// each; the item's rows are then read in 4-byte quads spread over the lanes (each quad fetches its row
// index from the hashing lane).
// RB > 0: rows of RB bytes known at compile time (the reference's 160), so the quad -> head division
// is a multiply; RB == 0: a.row_bytes.
template <int HPI, int RB>
__global__ void __launch_bounds__(256) ple_fp8_gather_kernel(const PleFp8Args a) {
    pdl_begin();
    constexpr int kParts = kPleHeads / HPI;             // items per token
    constexpr int kQ = (kPleQuads * HPI + 15) / 16;     // quads per lane in flight (20 for a whole token)
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int rb = RB > 0 ? RB : a.row_bytes;
    const int qpr = rb / 4;  // 4-byte quads per row
    const int quads = HPI * qpr;
    const int width = kPleHeads * rb;  // output floats per token
    const int64_t items = a.T * kParts;
    for (int64_t it = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); it < items; it += nwarps) {
        const int64_t t = it / kParts;
        const int h0 = (int)(it - t * kParts) * HPI;
        const uint32_t my_row = lane < HPI ? ple_fp8_row(a, t, h0 + lane) : 0u;
        float4* dst = reinterpret_cast<float4*>(a.out + t * width + (int64_t)h0 * rb);
        if constexpr (RB > 0 && (RB / 4) % (32 / HPI) == 0) {
            // Rows of known size: 32/HPI lanes per head, each with RB/4/(32/HPI) quads of that head's
            // row (one row index per lane, no division); each warp-wide load reads HPI 32-byte spans
            // and each store writes HPI whole 128-byte lines.
            constexpr int kLph = 32 / HPI, kQpl = RB / 4 / kLph;
            const int hl = lane / kLph, ql = lane % kLph;
            const uint32_t row = __shfl_sync(0xffffffffu, my_row, hl);
            const uint32_t* src = reinterpret_cast<const uint32_t*>(a.table + (uint64_t)row * RB) + ql;
            float4* d = dst + hl * (RB / 4) + ql;
            uint32_t raw[kQpl];
#pragma unroll
            for (int j = 0; j < kQpl; ++j) raw[j] = __ldg(src + j * kLph);
#pragma unroll
            for (int j = 0; j < kQpl; ++j) __stcs(d + j * kLph, fp8x4_decode(raw[j], a.scale));
            continue;
        }
        // Lane l produces output float4s q = k*32 + l: 4 fp8 bytes each, so every warp-wide load
        // reads 128 contiguous bytes (within at most two rows) and every store writes 512 contiguous
        // bytes. kQ loads per lane are in flight before any is decoded.
        for (int q0 = 0; q0 < quads; q0 += 32 * kQ) {
            uint32_t raw[kQ];
#pragma unroll
            for (int k = 0; k < kQ; ++k) {
                const int q = q0 + k * 32 + lane;
                const int h = q < quads ? q / qpr : 0;
                const uint32_t row = __shfl_sync(0xffffffffu, my_row, h);
                if (q < quads)
                    raw[k] = __ldg(reinterpret_cast<const uint32_t*>(a.table + (uint64_t)row * rb) + (q - h * qpr));
            }
#pragma unroll
            for (int k = 0; k < kQ; ++k) {
                const int q = q0 + k * 32 + lane;
                if (q < quads) __stcs(dst + q, fp8x4_decode(raw[k], a.scale));
            }
        }
    }
}

// ---- gate ---------------------------------------------------------------------------------------
// CTA-owned (token, stream) rows, as the wide norm design: thread i holds the 8-element vectors
// k*blockDim + i of key, query and value, the dot product meets in shared memory behind one barrier
// (partials double-buffered by row parity), then gv = value * gate.
template <int VPL>
__global__ void __launch_bounds__(512) ple_gate_kernel(const float* __restrict__ key, const float* __restrict__ query,
                                                       const float* __restrict__ value, float* __restrict__ gv,
                                                       int64_t units, int n, int hc) {
    pdl_begin();
    __shared__ float part[2][16];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int span = blockDim.x * 8;
    const float sqrt_n = sqrtf((float)n);
    int par = 0;
    for (int64_t u = blockIdx.x; u < units; u += gridDim.x, par ^= 1) {
        const int64_t t = u / hc;
        float2 kv[VPL][4], qv[VPL][4], vv[VPL][4];
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            const int e = k * span + threadIdx.x * 8;
            if (e < n) {
                Vec8<float>::cvt2(Vec8<float>::ldcs_raw(key + u * n + e), kv[k]);
                Vec8<float>::cvt2(Vec8<float>::ldcs_raw(query + u * n + e), qv[k]);
                Vec8<float>::load_ro2(value + t * n + e, vv[k]);
            }
        }
        float d = 0.f;
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            if (k * span + threadIdx.x * 8 < n) {
                float2 acc = splat2(0.f);
#pragma unroll
                for (int i = 0; i < 4; ++i) acc = ffma2(kv[k][i], qv[k][i], acc);
                d += acc.x + acc.y;
            }
        }
        d = group_sum<32>(d);
        if (lane == 0) part[par][warp] = d;
        __syncthreads();
        float tot = 0.f;
        for (int i = 0; i < nw; ++i) tot += part[par][i];
        tot /= sqrt_n;
        const float sg = tot < 0.f ? -1.f : 1.f;
        const float2 g = splat2(1.f / (1.f + __expf(-sg * sqrtf(fmaxf(fabsf(tot), 1e-6f)))));
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            const int e = k * span + threadIdx.x * 8;
            if (e < n) {
                float2 o[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) o[i] = fmul2(vv[k][i], g);
                Vec8<float>::store2(gv + u * n + e, o);
            }
        }
    }
}

// ---- conv ---------------------------------------------------------------------------------------
// x(s) = norm[s, c] for s >= 0, hist[c, 9 + s] for -9 <= s < 0 (the previous call's last 9 inputs).
//   acc(t) = w0*x(t-9) + w1*x(t-6) + w2*x(t-3) + w3*x(t)          (cw [c, 4])
//   R[t,c] += gv[t,c] + acc / (1 + exp(-acc))
// then hist[c, i] = x(T - 9 + i). With hist_snaps, the window after token t, x(t-8..t), is written
// to hist_snaps[t, c, 0..8]. The output never feeds back, so the work splits freely over (token,
// 4 channels): with snapshots one thread per pair (6 independent 16-byte loads; x(t-3..t-9) are rows
// other threads load too, L2 hits), without them one thread per 4 tokens spaced by the dilation
// (ple_conv_strided_kernel). The new history is written by a second, tiny launch once every thread
// of the first has read the old one.
constexpr int kConvHist = 9;

// x(s) for 4 channels starting at c
__device__ __forceinline__ float4 conv_x(const float* __restrict__ norm, const float* __restrict__ hist, int64_t s,
                                         int hcd, int c) {
    if (s >= 0) return __ldg(reinterpret_cast<const float4*>(norm + s * hcd + c));
    const int64_t i = kConvHist + s;
    return make_float4(hist[(int64_t)c * kConvHist + i], hist[(int64_t)(c + 1) * kConvHist + i],
                       hist[(int64_t)(c + 2) * kConvHist + i], hist[(int64_t)(c + 3) * kConvHist + i]);
}

__device__ __forceinline__ float conv_lane(const float4& v, int j) {
    return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w;
}

template <bool SNAPS>
__global__ void __launch_bounds__(256) ple_conv_kernel(const float* __restrict__ norm, const float* __restrict__ cw,
                                                       const float* __restrict__ hist, const float* __restrict__ gv,
                                                       float* __restrict__ R, int64_t T, int hcd,
                                                       float* __restrict__ snaps) {
    pdl_begin();
    const int c4n = hcd / 4;
    const int64_t items = T * c4n;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    StridePos ps(i0, stride, c4n);  // item = (token q, channel group r)
    for (int64_t it = i0; it < items; it += stride, ps.advance()) {
        const int64_t t = ps.q;
        const int c = ps.r * 4;
        const float4 x0 = __ldg(reinterpret_cast<const float4*>(norm + t * hcd + c));
        const float4 gq = __ldcs(reinterpret_cast<const float4*>(gv + t * hcd + c));
        float4* rp = reinterpret_cast<float4*>(R + t * hcd + c);
        const float4 rq = *rp;
        const float4 x3 = conv_x(norm, hist, t - 3, hcd, c);
        const float4 x6 = conv_x(norm, hist, t - 6, hcd, c);
        const float4 x9 = conv_x(norm, hist, t - 9, hcd, c);
        float rr[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float4 w = __ldg(reinterpret_cast<const float4*>(cw) + c + j);  // taps of channel c + j
            const float acc = w.x * conv_lane(x9, j) + w.y * conv_lane(x6, j) + w.z * conv_lane(x3, j) +
                              w.w * conv_lane(x0, j);
            float r = conv_lane(rq, j);
            r += conv_lane(gq, j) + acc / (1.0f + __expf(-acc));
            rr[j] = r;
        }
        __stcs(rp, make_float4(rr[0], rr[1], rr[2], rr[3]));
        if (SNAPS) {
            // x(t-8..t) of channel c + j at snaps[t, c + j, 0..8]: 36 consecutive floats
            float win[kConvHist][4];
#pragma unroll
            for (int i = 0; i < kConvHist; ++i) {
                const float4 v = conv_x(norm, hist, t - 8 + i, hcd, c);
                win[i][0] = v.x; win[i][1] = v.y; win[i][2] = v.z; win[i][3] = v.w;
            }
            float4* sp = reinterpret_cast<float4*>(snaps + (t * hcd + c) * kConvHist);
#pragma unroll
            for (int k = 0; k < kConvHist; ++k) {
                float q[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int f = 4 * k + e;  // flat index j * 9 + i
                    q[e] = win[f % kConvHist][f / kConvHist];
                }
                sp[k] = make_float4(q[0], q[1], q[2], q[3]);
            }
        }
    }
}

// Same outputs without snapshots, K tokens per thread: the tokens t0, t0 + 3, ..., t0 + 3(K-1) of one
// 4-channel group share their dilated inputs, so the thread loads the K + 3 rows x(t0 - 9 + 3i) once
// (instead of 4 per token) and keeps K tokens' gv and R loads in flight together. Tokens are taken in
// blocks of 3K; item q = 3 * block + residue covers tokens 3K * block + residue + 3j.
template <int K>
__global__ void __launch_bounds__(256) ple_conv_strided_kernel(const float* __restrict__ norm,
                                                               const float* __restrict__ cw,
                                                               const float* __restrict__ hist,
                                                               const float* __restrict__ gv, float* __restrict__ R,
                                                               int64_t T, int hcd) {
    pdl_begin();
    const int c4n = hcd / 4;
    const int64_t groups = ((T + 3 * K - 1) / (3 * K)) * 3;
    const int64_t items = groups * c4n;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    StridePos ps(i0, stride, c4n);  // item = (token group q, channel group r)
    for (int64_t it = i0; it < items; it += stride, ps.advance()) {
        const int res = (int)(ps.q % 3);
        const int64_t t0 = (ps.q - res) * K + res;
        if (t0 >= T) continue;
        const int c = ps.r * 4;
        float4 x[K + 3], gq[K], rq[K];
#pragma unroll
        for (int j = 0; j < K; ++j) {
            const int64_t t = t0 + 3 * j;
            if (t < T) {
                x[j + 3] = __ldg(reinterpret_cast<const float4*>(norm + t * hcd + c));
                gq[j] = __ldcs(reinterpret_cast<const float4*>(gv + t * hcd + c));
                rq[j] = *reinterpret_cast<const float4*>(R + t * hcd + c);
            }
        }
#pragma unroll
        for (int i = 0; i < 3; ++i) x[i] = conv_x(norm, hist, t0 - 9 + 3 * i, hcd, c);
        float4 w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) w[j] = __ldg(reinterpret_cast<const float4*>(cw) + c + j);  // taps of c + j
#pragma unroll
        for (int j = 0; j < K; ++j) {
            const int64_t t = t0 + 3 * j;
            if (t >= T) break;
            float rr[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float acc = w[e].x * conv_lane(x[j], e) + w[e].y * conv_lane(x[j + 1], e) +
                                  w[e].z * conv_lane(x[j + 2], e) + w[e].w * conv_lane(x[j + 3], e);
                rr[e] = conv_lane(rq[j], e) + (conv_lane(gq[j], e) + acc / (1.0f + __expf(-acc)));
            }
            __stcs(reinterpret_cast<float4*>(R + t * hcd + c), make_float4(rr[0], rr[1], rr[2], rr[3]));
        }
    }
}

// hist[c, i] = x(T - 9 + i): one thread per channel; runs after ple_conv_kernel (stream order), so no
// reader of the old history is left. Values with T - 9 + i < 0 shift down within the old history
// (read in full before any write by the same thread).
__global__ void __launch_bounds__(256) ple_conv_hist_kernel(const float* __restrict__ norm, float* __restrict__ hist,
                                                            int64_t T, int hcd) {
    pdl_begin();
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= hcd) return;
    float nh[kConvHist];
#pragma unroll
    for (int i = 0; i < kConvHist; ++i) {
        const int64_t s = T - kConvHist + i;
        nh[i] = s >= 0 ? norm[s * hcd + c] : hist[(int64_t)c * kConvHist + kConvHist + s];
    }
#pragma unroll
    for (int i = 0; i < kConvHist; ++i) hist[(int64_t)c * kConvHist + i] = nh[i];
}

}  // namespace wzyb

extern "C" {

int wzyb_ple_fp8_reference_hash(wzyb_ple_fp8_hash* out) {
    if (!out) return WZYB_ERR_NULL;
    // stage_ple_window's multipliers and per-head table sizes / offsets (src/wzy_engine_v2.cu:909-916):
    // 16 consecutive sub-tables of prime row counts just above 2e7, packed end to end.
    static const uint64_t mult[3] = {23703573157769ull, 20109073645365ull, 8052911324071ull};
    static const uint64_t vocab[16] = {20000003, 20000023, 20000033, 20000047, 20000059, 20000063,
                                       20000069, 20000077, 20000081, 20000093, 20000107, 20000147,
                                       20000153, 20000159, 20000161, 20000171};
    for (int i = 0; i < 3; ++i) out->mult[i] = mult[i];
    uint64_t off = 0;
    for (int h = 0; h < 16; ++h) {
        out->vocab[h] = vocab[h];
        out->off[h] = off;
        off += vocab[h];
    }
    return WZYB_OK;
}

int wzyb_ple_gather_fp8_f32(const uint8_t* table, int64_t table_rows, int row_bytes, float scale,
                            const wzyb_ple_fp8_hash* hash, const int32_t* ids, int64_t T, const int32_t* prev_ids,
                            int32_t eos_id, float* out, wzyb_stream_t stream) {
    if (!table || !hash || !ids || !out) return WZYB_ERR_NULL;
    if (T < 0 || row_bytes < 16 || row_bytes > 1024 || (row_bytes % 16) != 0 || table_rows < 1 ||
        table_rows > (int64_t(1) << 32))
        return WZYB_ERR_SHAPE;
    // every hashed row must lie in the table: off[h] + vocab[h] <= table_rows for each head
    for (int h = 0; h < 16; ++h) {
        if (hash->vocab[h] < 1 || hash->off[h] > (uint64_t)table_rows ||
            hash->vocab[h] > (uint64_t)table_rows - hash->off[h])
            return WZYB_ERR_SHAPE;
    }
    if (!wzyb::aligned16(table) || !wzyb::aligned16(out)) return WZYB_ERR_ALIGN;
    if (T == 0) return WZYB_OK;
    wzyb::DeviceInfo di;
    const int rc = wzyb::device_info(&di);
    if (rc != WZYB_OK) return rc;
    wzyb::PleFp8Args a;
    a.table = table;
    a.row_bytes = row_bytes;
    a.scale = scale;
    for (int i = 0; i < 3; ++i) a.mult[i] = hash->mult[i];
    for (int h = 0; h < 16; ++h) {
        a.vocab[h] = hash->vocab[h];
        a.off[h] = hash->off[h];
    }
    a.ids = ids;
    a.T = T;
    a.prev2 = prev_ids ? prev_ids[0] : -1;
    a.prev1 = prev_ids ? prev_ids[1] : -1;
    a.eos = eos_id;
    a.out = out;
    // 4 heads per warp item (4 items per token, 5 quads per lane in flight): 4.18 -> 4.83 TB/s at 262,144
    // tokens and 22.5 -> 20.1 us at 4096 against a warp per token; 8 heads: 3.81 TB/s, 2: 3.49, 1: 2.15
    constexpr int kHpi = 4;
    for (int h = 0; h < 16; ++h) a.recip[h] = ~0ull / a.vocab[h];
    const int grid = wzyb::persistent_grid(di, 8, (T * (16 / kHpi) + 7) / 8);
    if (row_bytes == 160) wzyb::launch_k(wzyb::ple_fp8_gather_kernel<kHpi, 160>, grid, 256, 0, (cudaStream_t)stream, a);
    else wzyb::launch_k(wzyb::ple_fp8_gather_kernel<kHpi, 0>, grid, 256, 0, (cudaStream_t)stream, a);
    return wzyb::launch_status();
}

int wzyb_ple_gate_f32(const float* key, const float* query, const float* value, float* gv, int64_t T, int n_embd,
                      int hc, wzyb_stream_t stream) {
    if (!key || !query || !value || !gv) return WZYB_ERR_NULL;
    if (T < 0 || T > (int64_t(1) << 40) || n_embd < 8 || n_embd > 16384 || (n_embd % 8) != 0 || hc < 1 || hc > 64)
        return WZYB_ERR_SHAPE;
    if (!wzyb::aligned16(key) || !wzyb::aligned16(query) || !wzyb::aligned16(value) || !wzyb::aligned16(gv))
        return WZYB_ERR_ALIGN;
    if (T == 0) return WZYB_OK;
    wzyb::DeviceInfo di;
    const int rc = wzyb::device_info(&di);
    if (rc != WZYB_OK) return rc;
    // fewest warps (4, 8, 16) keeping <= 3 vectors of each operand per thread
    const int vecs = n_embd / 8;
    int nw = 4;
    while (nw < 16 && (vecs + nw * 32 - 1) / (nw * 32) > 3) nw *= 2;
    const int need = (vecs + nw * 32 - 1) / (nw * 32);
    if (need > 4) return WZYB_ERR_SHAPE;
    const int threads = nw * 32;
    const int64_t units = T * hc;
    cudaStream_t s = (cudaStream_t)stream;
    const void* kern = need <= 1 ? (const void*)wzyb::ple_gate_kernel<1>
                     : need <= 2 ? (const void*)wzyb::ple_gate_kernel<2>
                     : need <= 3 ? (const void*)wzyb::ple_gate_kernel<3>
                                 : (const void*)wzyb::ple_gate_kernel<4>;
    const int grid = wzyb::persistent_grid(di, wzyb::resident_ctas(kern, threads, 0), units);
    switch (need) {
        case 1: wzyb::launch_k(wzyb::ple_gate_kernel<1>, grid, threads, 0, s, key, query, value, gv, units, n_embd, hc); break;
        case 2: wzyb::launch_k(wzyb::ple_gate_kernel<2>, grid, threads, 0, s, key, query, value, gv, units, n_embd, hc); break;
        case 3: wzyb::launch_k(wzyb::ple_gate_kernel<3>, grid, threads, 0, s, key, query, value, gv, units, n_embd, hc); break;
        default: wzyb::launch_k(wzyb::ple_gate_kernel<4>, grid, threads, 0, s, key, query, value, gv, units, n_embd, hc); break;
    }
    return wzyb::launch_status();
}

int wzyb_ple_conv_f32(const float* norm, const float* cw, float* hist, const float* gv, float* R, int64_t T, int hcd,
                      float* hist_snaps, wzyb_stream_t stream) {
    if (!norm || !cw || !hist || !gv || !R) return WZYB_ERR_NULL;
    if (T < 0 || T > (int64_t(1) << 40) || hcd < 4 || (hcd % 4) != 0) return WZYB_ERR_SHAPE;
    if (!wzyb::aligned16(norm) || !wzyb::aligned16(cw) || !wzyb::aligned16(gv) || !wzyb::aligned16(R) ||
        ((uintptr_t)hist & 3) || (hist_snaps && !wzyb::aligned16(hist_snaps)))
        return WZYB_ERR_ALIGN;
    if (T == 0) return WZYB_OK;
    wzyb::DeviceInfo di;
    const int rc = wzyb::device_info(&di);
    if (rc != WZYB_OK) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    if (hist_snaps) {
        const int64_t items = T * (hcd / 4);
        const int grid = wzyb::persistent_grid(di, 8, (items + 255) / 256);
        wzyb::launch_k(wzyb::ple_conv_kernel<true>, grid, 256, 0, st, norm, cw, hist, gv, R, T, hcd, hist_snaps);
    } else {
        // 4 tokens per thread: 150 -> 108 us at 4096 tokens x 10240 channels (68 -> 95 % of HBM peak;
        // 2 tokens: 109 us, 3: 115 us)
        constexpr int kK = 4;
        const int64_t items = ((T + 3 * kK - 1) / (3 * kK)) * 3 * (hcd / 4);
        const void* kern = (const void*)wzyb::ple_conv_strided_kernel<kK>;
        const int grid = wzyb::persistent_grid(di, wzyb::resident_ctas(kern, 256, 0), (items + 255) / 256);
        wzyb::launch_k(wzyb::ple_conv_strided_kernel<kK>, grid, 256, 0, st, norm, cw, hist, gv, R, T, hcd);
    }
    wzyb::launch_k(wzyb::ple_conv_hist_kernel, (hcd + 255) / 256, 256, 0, st, norm, hist, T, hcd);
    return wzyb::launch_status();
}

}  // extern "C"
