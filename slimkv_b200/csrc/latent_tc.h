// Launch interface of the tcgen05 decode attention (latent_tc.cu): one launch
// streams the latent cache (one shared latent head, all query heads per CTA)
// and the raw sink + tail (per KV head) with the same tensor-core pipeline.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace slimkv {

// Per-branch job as the kernel sees it.
struct TcJob {
    int kchunks, vchunks;     // 64-column chunks of a K / V row
    int kv_heads;             // KV heads per sequence in the grid (1 for the latent branch)
    int group;                // query heads per KV head (rows of a Q box in row mode)
    int causal;               // two queries: the first excludes the last key (the new Beacon)
    int q_rows;               // Q read per query from [B*L][H][dim] rows (exact bf16: no lo part)
    const int32_t* seqlens;   // keys per sequence
    const int32_t* qlens;     // queries per sequence (1 or 2), nullable
    int length;
    float scale_log2;
    int splits, rows_alloc, out_width;
    float* part_o;            // [B][kv_heads][splits][rows_alloc][out_width]
    float* part_lse;          // [B][kv_heads][splits][rows_alloc]
    unsigned int* status;
    // Paged K/V (nullptr table = dense maps): row n of sequence b is row
    // n % slots of page table[b * table_stride + n / slots]; the K/V maps are
    // then one page map [pages][slots][W] and V starts at column v_col.
    const int32_t* table;
    int64_t table_stride;
    int slots, v_col, box_rows;   // box_rows: rows per page-map box (divides slots and 128)
    // Work list (nullable): work[i] = sequence << 11 | its split count << 5 |
    // split for CTA i of the branch, -1 for an unused CTA; a sequence has
    // latent_splits_of(seqlens[b], tps, splits) splits.  Without it CTA i is
    // (i / splits, i % splits).
    const int32_t* work;
    int tps;
};

// One branch as the host describes it.
struct TcSide {
    const void* k;
    const void* v;
    int dim_k, dim_v;          // latent ranks, or the head dim
    int kv_heads, capacity;
    int64_t stride_batch, stride_row, stride_head;   // elements
    // Latent: q_hilo [B][128][width] bf16 with row hl*32*nq + l*32 + head
    // (hl 0 = hi, 1 = lo).  Raw: q_rot [B][L][H][dim] bf16.
    const void* q;
    int q_rows, heads, group, causal;
    const int32_t* seqlens;
    int splits, rows_alloc, width;
    float* part_o;
    float* part_lse;
    // Paged K/V: pages [num_pages] of page_stride elements holding
    // [sink][slots x (dim_k + dim_v)] (k / v unused).
    const void* pages;
    int64_t page_stride;
    int slots, sink_elements, num_pages;
    const int32_t* table;
    int64_t table_stride;
    const int32_t* work;       // see TcJob::work
    int tiles_per_split;
};

struct TcLaunch {
    int batch, length;
    float scale;
    const int32_t* query_len;
    unsigned int* status;
    TcSide lat, raw;
    int with_raw;
};

constexpr int kTcTileKeys = 128;

// Latent splits of a sequence with `len` latent rows when every split holds
// at most `tps` 128-key tiles (at least one split, at most `smax`).  The
// prologue's work list, the attention kernel and the merge agree on it.
__host__ __device__ inline int latent_splits_of(int len, int tps, int smax) {
    const int tiles = len > 0 ? (len + kTcTileKeys - 1) / kTcTileKeys : 0;
    const int n = (tiles + tps - 1) / tps;
    return n < 1 ? 1 : (n > smax ? smax : n);
}

int launch_decode_tc(const TcLaunch& launch, cudaStream_t stream);

}  // namespace slimkv
