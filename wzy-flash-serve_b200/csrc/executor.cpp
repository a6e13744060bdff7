// executor.cpp -- host-side planning for token-sharded runs (plain C++, no CUDA here).
//
// The path shards by token rows with no exchange step: each GPU takes a contiguous row range of the
// sequence, its RoPE positions start at the range's first row, and its 3-gram PLE rows need the two ids
// that precede the range (the history the reference's stage_emb_ple_pf keeps in ple_prev across
// chunks, src/wzy_engine_v2.cu:1210-1265). The layer bundles themselves are in bundle.cu.
#include <cstdint>

#include "../../include/wzyb200.h"

extern "C" {

int wzyb_shard_rows(int64_t total, int world, int rank, int64_t* row0, int64_t* rows) {
    if (row0 == nullptr || rows == nullptr) return WZYB_ERR_NULL;
    if (total < 0 || world < 1 || rank < 0 || rank >= world) return WZYB_ERR_SHAPE;
    const int64_t per = (total + world - 1) / world;
    int64_t a = per * rank;
    if (a > total) a = total;
    int64_t b = a + per;
    if (b > total) b = total;
    *row0 = a;
    *rows = b - a;
    return WZYB_OK;
}

int wzyb_ple_halo(const int32_t* ids, int64_t row0, const int32_t* seq_prev, int32_t out_prev[2]) {
    if (out_prev == nullptr) return WZYB_ERR_NULL;
    if (row0 < 0 || (row0 > 0 && ids == nullptr)) return WZYB_ERR_SHAPE;
    // the ids at positions row0-2 and row0-1 of the sequence that seq_prev = {id[-2], id[-1]} precedes
    const int32_t before[2] = {seq_prev ? seq_prev[0] : -1, seq_prev ? seq_prev[1] : -1};
    for (int j = 0; j < 2; ++j) {
        const int64_t p = row0 - 2 + j;
        out_prev[j] = p >= 0 ? ids[p] : before[p + 2];
    }
    return WZYB_OK;
}

}  // extern "C"
