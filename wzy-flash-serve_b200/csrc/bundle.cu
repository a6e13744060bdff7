// bundle.cu -- one kernel launch per layer bundle.
//
// The reference launches the ops of a bundle one after another inside its prefill layer loop
// (PrefillStageCtx::run_stage_prefill: the residual norm at src/wzy_prefill_tc.cuh:697 and the q/k
// norm + RoPE at :862-867; the SwiGLU at :942 and the GDN gated norm at :845) and stages the
// token-embedding and PLE rows of a chunk in one host routine (stage_emb_ple_pf,
// src/wzy_engine_v2.cu:1210-1265). The two ops of each bundle share no tensor, so here a bundle is ONE
// persistent grid in which every CTA runs both ops' bodies in turn (by default; the schedules below
// also split the grid between the ops). The bodies are the per-op kernels' own device code
// (norm_rows.cu, head_rope.cu, swiglu.cu, gdn_norm.cu, gather.cu), so every output is bit-identical
// to the separate launches.
//
// Why: at layer-sized calls (4096 tokens, 67-140 MB per op) a launch is dominated by its fixed costs --
// the launch itself, the DRAM ramp while the first loads are in flight, and the tail where the last
// warps finish alone. One grid pays them once per bundle, and DRAM streams both ops' traffic at once.
// Past a size measured per bundle (1.25 GiB for attn_prep, 1 GiB for act, 96 MiB for embed_ple) those
// costs are small, and the ops' own launches (each with its own tuned occupancy) are as fast or
// faster, so larger bundles are issued that way.
#include "launch.hpp"

namespace wzyb {

constexpr int kBundleThreads = 256;
constexpr int kBundleWarps = kBundleThreads / 32;

// One op of a bundle as per-warp work items: `items` items of `bytes` algorithmic bytes each.
struct RoleWork {
    int64_t items;
    double bytes;
};

// CTAs of op 0 when a grid of G >= 2 CTAs is split between two ops that both have work: the split
// whose most loaded warp (a whole number of items) moves the fewest bytes, ties broken towards equal
// mean bytes per warp.
static int split_grid(int G, const RoleWork& r0, const RoleWork& r1) {
    int best = 1;
    double best_cost = 0.0, best_gap = 0.0;
    for (int g0 = 1; g0 < G; ++g0) {
        const int64_t w0 = (int64_t)g0 * kBundleWarps, w1 = (int64_t)(G - g0) * kBundleWarps;
        const double c0 = (double)((r0.items + w0 - 1) / w0) * r0.bytes;
        const double c1 = (double)((r1.items + w1 - 1) / w1) * r1.bytes;
        const double cost = c0 > c1 ? c0 : c1;
        const double m0 = (double)r0.items * r0.bytes / (double)w0, m1 = (double)r1.items * r1.bytes / (double)w1;
        const double gap = m0 > m1 ? m0 - m1 : m1 - m0;
        if (g0 == 1 || cost < best_cost || (cost == best_cost && gap < best_gap)) {
            best = g0;
            best_cost = cost;
            best_gap = gap;
        }
    }
    return best;
}

// Schedules of a bundle's grid (wzyb_set_launch_tuning(WZYB_FAM_BUNDLE, ., schedule) for A/B):
enum BundleSchedule : int {
    kSchedAuto = 0,
    kSchedSplit = 1,    // persistent grid split between the ops (CTAs [0, g0) op 0, the rest op 1)
    kSchedPerItem = 2,  // one item per warp: the grid is sized to the work and the hardware's CTA
                        // scheduler balances it (op 0's CTAs first)
    kSchedShared = 3,   // persistent grid, every CTA runs both ops
    kSchedLaunches = 4, // each op as its own launch
};
// Bundles of up to `max_bytes` algorithmic bytes run as one launch with both ops on every CTA (the
// larger items first); larger ones as the ops' own launches, each with its own tuned occupancy, once
// a launch's fixed costs no longer matter. Measured on B200 with L2 flushed before each call (us, one
// launch / the ops' launches), by token count of the benchmark's layer:
//   attn_prep (34,816 B/token)  4096: 30.8 / 33.8   8192: 53.3 / 58.4   16384: 103.3 / 109.6
//                               32768: 197.5 / 202.4   65536: 387.6 / 383.7
//   act (58,368 B/token)        4096: 38.9 / 42.0   8192: 75.7 / 80.3   16384: 154.8 / 155.3
//                               32768: 317.6 / 310.0
//   embed_ple (16,384 B/token)  4096: 16.4 / 17.4   8192: 26.6 / 25.9   16384: 49.7 / 46.2
constexpr double kFuseMaxAttn = 1.25 * (1 << 30);
constexpr double kFuseMaxAct = 1.0 * (1 << 30);
constexpr double kFuseMaxGather = 96.0 * (1 << 20);

static int bundle_schedule(double bundle_bytes, double max_bytes) {
    const int s = tuning(kFamBundle).stages;
    if (s >= kSchedSplit && s <= kSchedLaunches) return s;
    return bundle_bytes <= max_bytes ? kSchedShared : kSchedLaunches;
}

// Grid and split for a bundle: every SM filled with `resident` CTAs, or, when the two ops together
// have no more items than that many warps (or the schedule asks for it), one item per warp. g0 < 0
// asks every CTA to run both ops.
static void bundle_grid(const DeviceInfo& di, int resident, const RoleWork& r0, const RoleWork& r1, int sched,
                        int& grid, int& g0) {
    const int64_t need0 = (r0.items + kBundleWarps - 1) / kBundleWarps;
    const int64_t need1 = (r1.items + kBundleWarps - 1) / kBundleWarps;
    const int64_t full = (int64_t)di.sms * resident;
    if (sched == kSchedShared) {
        const int64_t need = need0 > need1 ? need0 : need1;
        grid = (int)(need < full ? need : full);
        g0 = -1;
    } else if (need0 + need1 <= full || sched == kSchedPerItem) {
        g0 = (int)need0;
        grid = (int)(need0 + need1);
    } else if (need0 == 0 || need1 == 0) {
        g0 = need0 == 0 ? 0 : (int)full;
        grid = (int)full;
    } else {
        grid = (int)full;
        g0 = split_grid(grid, r0, r1);
    }
    if (grid < 1) grid = 1;
}

// Byte ranges of the tensors an op reads and writes, to tell whether two ops may run concurrently.
struct Span {
    uintptr_t lo, hi;  // [lo, hi)
};
static Span span(const void* p, int64_t bytes) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    return Span{a, p && bytes > 0 ? a + (uintptr_t)bytes : a};
}
static bool overlap(const Span& a, const Span& b) { return a.lo < b.hi && b.lo < a.hi; }
// True when a write of one op may touch a byte the other op reads or writes.
template <int NW0, int NR0, int NW1, int NR1>
static bool ops_conflict(const Span (&w0)[NW0], const Span (&r0)[NR0], const Span (&w1)[NW1], const Span (&r1)[NR1]) {
    for (const Span& a : w0) {
        for (const Span& b : w1)
            if (overlap(a, b)) return true;
        for (const Span& b : r1)
            if (overlap(a, b)) return true;
    }
    for (const Span& a : w1)
        for (const Span& b : r0)
            if (overlap(a, b)) return true;
    return false;
}
// Bytes spanned by a strided head tensor of T tokens.
static int64_t head_span_bytes(const HeadSection& s, int64_t T, int hd, int esize) {
    if (s.heads <= 0 || T <= 0) return 0;
    return ((T - 1) * s.row_stride + (int64_t)(s.heads - 1) * s.head_stride + hd) * esize;
}

// ---------------------------------------------------------------------------------------------
// configs[1] bundle: residual add + RMSNorm rows (direct design) and q/k norm + RoPE (pair design).
// ---------------------------------------------------------------------------------------------
// g_norm < 0: every CTA runs both ops over the whole grid: the norm rows first (the head body's
// gamma table is filled before them), then the head items with the CTA order reversed, so the warps
// that took one more row than others take fewer head items.
template <int VPL, int HD>
__global__ void __launch_bounds__(kBundleThreads, 2) attn_prep_kernel(const NormRowsArgs na, const HeadRopeArgs ha,
                                                                      int g_norm) {
    pdl_begin();
    if (g_norm < 0) {
        // the norm rows (the larger items) first, the head items after them fill the tail
        head_rope_pair_body<__half, HD, 3>(ha, blockIdx.x, gridDim.x, 1);
        norm_rows_direct_body<__half, __half, VPL>(na, blockIdx.x, gridDim.x);
        head_rope_pair_body<__half, HD, 3>(ha, (int)gridDim.x - 1 - (int)blockIdx.x, gridDim.x, 2);
    } else if ((int)blockIdx.x < g_norm) {
        norm_rows_direct_body<__half, __half, VPL>(na, blockIdx.x, g_norm);
    } else {
        head_rope_pair_body<__half, HD, 3>(ha, (int)blockIdx.x - g_norm, (int)gridDim.x - g_norm);
    }
}

template <int VPL>
static const void* attn_prep_kernel_ptr(int hd) {
    return hd == 64 ? (const void*)attn_prep_kernel<VPL, 64>
                    : hd == 128 ? (const void*)attn_prep_kernel<VPL, 128> : (const void*)attn_prep_kernel<VPL, 256>;
}

template <int VPL>
static void attn_prep_launch(int hd, int grid, cudaStream_t s, const NormRowsArgs& na, const HeadRopeArgs& ha, int g0) {
    if (hd == 64) launch_k(attn_prep_kernel<VPL, 64>, grid, kBundleThreads, 0, s, na, ha, g0);
    else if (hd == 128) launch_k(attn_prep_kernel<VPL, 128>, grid, kBundleThreads, 0, s, na, ha, g0);
    else launch_k(attn_prep_kernel<VPL, 256>, grid, kBundleThreads, 0, s, na, ha, g0);
}

static int attn_prep_run(const wzyb_attn_prep_args* p, int64_t T, cudaStream_t stream) {
    NormRowsArgs na;
    int rc = norm_rows_prepare<__half>(p->x, p->residual, p->norm_weight, nullptr, p->normed, T, p->hidden, 1,
                                       p->eps, p->w_offset, na);
    if (rc != WZYB_OK) return rc;
    const HeadSection q{p->q.data, p->q.gamma, p->q.heads, p->q.head_stride, p->q.row_stride};
    const HeadSection k{p->k.data, p->k.gamma, p->k.heads > 0 ? p->k.heads : 0, p->k.head_stride, p->k.row_stride};
    HeadRopeArgs ha;
    rc = head_rope_prepare<__half>(q, k, p->cos_tab, p->sin_tab, p->table_rows, p->d_base_pos, p->pos_offset, T,
                                   p->head_dim, p->rot_dims, p->eps, p->w_offset, ha);
    if (rc != WZYB_OK || T == 0) return rc;

    const int hd = p->head_dim, n = p->hidden;
    const int vpl_need = (n + 255) / 256;
    const int vpl = vpl_need <= 2 ? 2 : vpl_need <= 4 ? 4 : vpl_need <= 8 ? 8 : vpl_need <= 10 ? 10 : 0;
    const int vn = variant(kFamNorm), vh = variant(kFamHeadRope);
    const double bytes = (double)T * (8.0 * n + 4.0 * (q.heads + k.heads) * hd);
    const int sched = bundle_schedule(bytes, kFuseMaxAttn);
    bool fused = variant(kFamBundle) != WZYB_VARIANT_SPLIT && sched != kSchedLaunches && vpl != 0 &&
                 (vn == WZYB_VARIANT_AUTO || vn == WZYB_VARIANT_DIRECT) &&
                 (vh == WZYB_VARIANT_AUTO || vh == WZYB_VARIANT_PAIR) && tuning(kFamHeadRope).ctas_per_sm != 2;
    if (fused) {
        const int64_t row = (int64_t)n * 2;
        const Span w0[2] = {span(p->x ? p->residual : nullptr, T * row), span(p->normed, T * row)};
        const Span r0[3] = {span(p->x, T * row), span(p->residual, T * row), span(p->norm_weight, row)};
        const Span w1[2] = {span(q.data, head_span_bytes(q, T, hd, 2)), span(k.data, head_span_bytes(k, T, hd, 2))};
        const Span r1[4] = {span(q.gamma, hd * 2), span(k.heads > 0 ? k.gamma : nullptr, hd * 2),
                            span(p->cos_tab, p->table_rows * (p->rot_dims / 2) * 4),
                            span(p->sin_tab, p->table_rows * (p->rot_dims / 2) * 4)};
        fused = !ops_conflict(w0, r0, w1, r1);
    }
    if (!fused) {
        rc = wzyb_add_rmsnorm_f16(p->x, p->residual, p->norm_weight, p->normed, T, n, p->eps, p->w_offset, stream);
        if (rc != WZYB_OK) return rc;
        return wzyb_qk_norm_rope_f16(&p->q, p->k.heads > 0 ? &p->k : nullptr, p->cos_tab, p->sin_tab,
                                     p->table_rows, p->d_base_pos, p->pos_offset, T, hd, p->rot_dims, p->eps,
                                     p->w_offset, stream);
    }

    DeviceInfo di;
    rc = device_info(&di);
    if (rc != WZYB_OK) return rc;
    const void* kern = vpl == 2 ? attn_prep_kernel_ptr<2>(hd)
                       : vpl == 4 ? attn_prep_kernel_ptr<4>(hd)
                                  : vpl == 8 ? attn_prep_kernel_ptr<8>(hd) : attn_prep_kernel_ptr<10>(hd);
    const int htot = q.heads + k.heads;
    const int ch = 3 * (512 / hd);  // heads per pair-design item (3 rounds of 512/hd heads)
    const int64_t chunks = (htot + ch - 1) / ch;
    const RoleWork r_norm{T, (double)(4 * (int64_t)n * 2)};
    const RoleWork r_head{T * chunks, 2.0 * htot * hd * 2 / (double)chunks};
    int grid = 0, g0 = 0;
    bundle_grid(di, resident_ctas(kern, kBundleThreads, 0), r_norm, r_head, sched, grid, g0);
    if (vpl == 2) attn_prep_launch<2>(hd, grid, stream, na, ha, g0);
    else if (vpl == 4) attn_prep_launch<4>(hd, grid, stream, na, ha, g0);
    else if (vpl == 8) attn_prep_launch<8>(hd, grid, stream, na, ha, g0);
    else attn_prep_launch<10>(hd, grid, stream, na, ha, g0);
    return launch_status();
}

// ---------------------------------------------------------------------------------------------
// configs[2] bundle: SwiGLU over the expert rows (flat stream) and the GDN gated norm (direct design).
// ---------------------------------------------------------------------------------------------
template <int HD, bool SILU, bool PACKED>
__global__ void __launch_bounds__(kBundleThreads, 3) act_kernel(const __half* __restrict__ gate,
                                                                const __half* __restrict__ up, __half* __restrict__ out,
                                                                int64_t nvec, const GdnArgs ga, int g_swiglu) {
    pdl_begin();
    if (g_swiglu < 0) {  // both ops on every CTA: the larger SwiGLU items first (as attn_prep_kernel)
        swiglu_body<__half, __half, false, PACKED>(gate, up, out, nvec, 0, 0, blockIdx.x, gridDim.x);
        gdn_direct_body<__half, __half, HD, 4, SILU>(ga, (int)gridDim.x - 1 - (int)blockIdx.x, gridDim.x);
    } else if ((int)blockIdx.x < g_swiglu) {
        swiglu_body<__half, __half, false, PACKED>(gate, up, out, nvec, 0, 0, blockIdx.x, g_swiglu);
    } else {
        gdn_direct_body<__half, __half, HD, 4, SILU>(ga, (int)blockIdx.x - g_swiglu, (int)gridDim.x - g_swiglu);
    }
}

template <bool SILU, bool PACKED>
static const void* act_kernel_ptr(int hd) {
    return hd == 64 ? (const void*)act_kernel<64, SILU, PACKED>
                    : hd == 128 ? (const void*)act_kernel<128, SILU, PACKED> : (const void*)act_kernel<256, SILU, PACKED>;
}

template <bool SILU, bool PACKED>
static void act_launch(int hd, int grid, cudaStream_t s, const __half* g, const __half* u, __half* o, int64_t nvec,
                       const GdnArgs& ga, int g0) {
    if (hd == 64) launch_k(act_kernel<64, SILU, PACKED>, grid, kBundleThreads, 0, s, g, u, o, nvec, ga, g0);
    else if (hd == 128) launch_k(act_kernel<128, SILU, PACKED>, grid, kBundleThreads, 0, s, g, u, o, nvec, ga, g0);
    else launch_k(act_kernel<256, SILU, PACKED>, grid, kBundleThreads, 0, s, g, u, o, nvec, ga, g0);
}

static int act_run(const wzyb_act_args* p, int64_t T, cudaStream_t stream) {
    if (p->act_rows < 0 || p->ffn < 0) return WZYB_ERR_SHAPE;
    const int64_t n = p->act_rows * (int64_t)p->ffn;
    if (!p->gate || !p->up || !p->act) return WZYB_ERR_NULL;
    if ((n % 8) != 0) return WZYB_ERR_SHAPE;
    if (!aligned16(p->gate) || !aligned16(p->up) || !aligned16(p->act)) return WZYB_ERR_ALIGN;
    GdnArgs ga;
    int rc = gdn_prepare<__half>(p->o, p->z, p->gdn_gamma, p->gdn_out, T, p->gdn_heads, p->gdn_head_dim, p->eps,
                                 p->gdn_w_offset, p->gate_mode, ga);
    if (rc != WZYB_OK) return rc;
    if (n == 0 && T == 0) return WZYB_OK;

    const int hd = p->gdn_head_dim;
    const int vg = variant(kFamGdn);
    const double bytes = 6.0 * (double)n + 6.0 * (double)T * p->gdn_heads * hd;
    const int sched = bundle_schedule(bytes, kFuseMaxAct);
    bool fused = variant(kFamBundle) != WZYB_VARIANT_SPLIT && sched != kSchedLaunches &&
                 (vg == WZYB_VARIANT_AUTO || vg == WZYB_VARIANT_DIRECT) &&
                 n > 0 && T > 0;
    if (fused) {
        const int64_t gb = T * p->gdn_heads * (int64_t)hd * 2;
        const Span w0[1] = {span(p->act, n * 2)};
        const Span r0[2] = {span(p->gate, n * 2), span(p->up, n * 2)};
        const Span w1[1] = {span(p->gdn_out, gb)};
        const Span r1[3] = {span(p->o, gb), span(p->z, gb), span(p->gdn_gamma, hd * 2)};
        fused = !ops_conflict(w0, r0, w1, r1);
    }
    if (!fused) {
        rc = wzyb_swiglu_f16(p->gate, p->up, p->act, n, stream);
        if (rc != WZYB_OK) return rc;
        return wzyb_gdn_gated_norm_f16(p->o, p->z, p->gdn_gamma, p->gdn_out, T, p->gdn_heads, hd, p->eps,
                                       p->gdn_w_offset, p->gate_mode, stream);
    }

    DeviceInfo di;
    rc = device_info(&di);
    if (rc != WZYB_OK) return rc;
    const int64_t nvec = n / 8;
    const bool silu = p->gate_mode == WZYB_GATE_SILU;
    const bool packed = !swiglu_scalar_math(nvec);
    const void* kern = silu ? (packed ? act_kernel_ptr<true, true>(hd) : act_kernel_ptr<true, false>(hd))
                            : (packed ? act_kernel_ptr<false, true>(hd) : act_kernel_ptr<false, false>(hd));
    // SwiGLU warp item: 32 lanes x 4 vectors (gate, up, out: 48 bytes each); GDN warp item: one
    // 256-element slab of o, z and y.
    const int64_t slabs = ((int64_t)p->gdn_heads * hd + 255) / 256;
    const RoleWork r_swiglu{(nvec + 127) / 128, 128.0 * 48.0};
    const RoleWork r_gdn{T * slabs, 3.0 * p->gdn_heads * hd * 2 / (double)slabs};
    int grid = 0, g0 = 0;
    bundle_grid(di, resident_ctas(kern, kBundleThreads, 0), r_swiglu, r_gdn, sched, grid, g0);
    const __half* g = (const __half*)p->gate;
    const __half* u = (const __half*)p->up;
    __half* o = (__half*)p->act;
    if (silu) {
        if (packed) act_launch<true, true>(hd, grid, stream, g, u, o, nvec, ga, g0);
        else act_launch<true, false>(hd, grid, stream, g, u, o, nvec, ga, g0);
    } else {
        if (packed) act_launch<false, true>(hd, grid, stream, g, u, o, nvec, ga, g0);
        else act_launch<false, false>(hd, grid, stream, g, u, o, nvec, ga, g0);
    }
    return launch_status();
}

// ---------------------------------------------------------------------------------------------
// configs[3] bundle: token-embedding rows (a warp per row) and 3-gram PLE rows (lane groups).
// ---------------------------------------------------------------------------------------------
template <int CH, int U>
__global__ void __launch_bounds__(kBundleThreads) embed_ple_kernel(const EmbedArgs ea, const PleArgs pa, int g_embed) {
    pdl_begin();
    if (g_embed < 0) {  // both ops on every CTA: the larger token rows first (as attn_prep_kernel)
        gather_rows_body(ea, blockIdx.x, gridDim.x);
        ple_gather_groups_body<CH, U>(pa, (int)gridDim.x - 1 - (int)blockIdx.x, gridDim.x);
    } else if ((int)blockIdx.x < g_embed) {
        gather_rows_body(ea, blockIdx.x, g_embed);
    } else {
        ple_gather_groups_body<CH, U>(pa, (int)blockIdx.x - g_embed, (int)gridDim.x - g_embed);
    }
}

template <int CH>
static void embed_ple_launch(int grid, cudaStream_t s, const EmbedArgs& ea, const PleArgs& pa, int g0) {
    launch_k(embed_ple_kernel<CH, 2>, grid, kBundleThreads, 0, s, ea, pa, g0);
}

static int embed_ple_run(const wzyb_embed_ple_args* p, int64_t T, cudaStream_t stream) {
    if (p->hidden < 8 || (p->hidden % 8) != 0) return WZYB_ERR_SHAPE;
    EmbedArgs ea;
    int rc = embed_prepare(p->table, p->vocab, (int64_t)p->hidden * 2, p->ids, T, p->emb_out, p->oob_policy,
                           p->d_oob_count, ea);
    if (rc != WZYB_OK) return rc;
    PleArgs pa;
    rc = ple_prepare(p->ple_tables, p->ple_heads, p->ple_rows, p->ple_head_dim, p->ids, T, p->prev_ids, p->eos_id,
                     p->hash_variant, p->ple_out, pa);
    if (rc != WZYB_OK || T == 0) return rc;

    const int ch = pa.chunks;
    const double bytes = (double)T * (4.0 * p->hidden + 4.0 * p->ple_heads * p->ple_head_dim);
    const int sched = bundle_schedule(bytes, kFuseMaxGather);
    bool fused = variant(kFamBundle) != WZYB_VARIANT_SPLIT && sched != kSchedLaunches && (ch == 8 || ch == 16 || ch == 32);
    if (fused) {
        const int64_t erow = (int64_t)p->hidden * 2, prow = (int64_t)p->ple_head_dim * 2;
        const Span w0[2] = {span(p->emb_out, T * erow), span(p->d_oob_count, 4)};
        const Span r0[2] = {span(p->table, p->vocab * erow), span(p->ids, T * 4)};
        const Span w1[1] = {span(p->ple_out, T * p->ple_heads * prow)};
        Span r1[33];
        r1[0] = span(p->ids, T * 4);
        for (int h = 0; h < 32; ++h) r1[1 + h] = span(h < p->ple_heads ? p->ple_tables[h] : nullptr, p->ple_rows * prow);
        fused = !ops_conflict(w0, r0, w1, r1);
    }
    if (fused && variant(kFamGather) == WZYB_VARIANT_RING) {
        rc = gather_bulk_launch(ea, pa, stream);  // both gathers as bulk copies in one launch
        if (rc != WZYB_ERR_SHAPE) return rc;
    }
    if (!fused) {
        rc = wzyb_embed_gather_f16(p->table, p->vocab, p->hidden, p->ids, T, p->emb_out, p->oob_policy,
                                   p->d_oob_count, stream);
        if (rc != WZYB_OK) return rc;
        return wzyb_ple_gather_f16(p->ple_tables, p->ple_heads, p->ple_rows, p->ple_head_dim, p->ids, T, p->prev_ids,
                                   p->eos_id, p->hash_variant, p->ple_out, stream);
    }

    DeviceInfo di;
    rc = device_info(&di);
    if (rc != WZYB_OK) return rc;
    const void* kern = ch == 8 ? (const void*)embed_ple_kernel<8, 2>
                       : ch == 16 ? (const void*)embed_ple_kernel<16, 2> : (const void*)embed_ple_kernel<32, 2>;
    const int gpw = 32 / ch;  // PLE rows side by side in one warp
    const RoleWork r_embed{T, 2.0 * (double)ea.row_chunks * 16.0};
    const RoleWork r_ple{(T * p->ple_heads + gpw - 1) / gpw, gpw * 2.0 * ch * 16.0};
    int grid = 0, g0 = 0;
    bundle_grid(di, resident_ctas(kern, kBundleThreads, 0), r_embed, r_ple, sched, grid, g0);
    if (ch == 8) embed_ple_launch<8>(grid, stream, ea, pa, g0);
    else if (ch == 16) embed_ple_launch<16>(grid, stream, ea, pa, g0);
    else embed_ple_launch<32>(grid, stream, ea, pa, g0);
    return launch_status();
}

}  // namespace wzyb

extern "C" {

int wzyb_attn_prep_f16(const wzyb_attn_prep_args* a, int64_t T, wzyb_stream_t stream) {
    if (a == nullptr) return WZYB_ERR_NULL;
    return wzyb::attn_prep_run(a, T, (cudaStream_t)stream);
}

int wzyb_act_f16(const wzyb_act_args* a, int64_t T, wzyb_stream_t stream) {
    if (a == nullptr) return WZYB_ERR_NULL;
    return wzyb::act_run(a, T, (cudaStream_t)stream);
}

int wzyb_embed_ple_f16(const wzyb_embed_ple_args* a, int64_t T, wzyb_stream_t stream) {
    if (a == nullptr) return WZYB_ERR_NULL;
    return wzyb::embed_ple_run(a, T, (cudaStream_t)stream);
}

}  // extern "C"
