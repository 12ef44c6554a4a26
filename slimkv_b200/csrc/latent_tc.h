// Launch interface of the tcgen05 decode attention (latent_tc.cu).
//
// One persistent launch streams both branches of a decode step: the latent
// cache (one shared latent head, all query heads per CTA) and the raw sink +
// tail (per KV head).  The work is planned on the device (plan_tc_work() in
// latent_tc_plan.cuh, run by the prologue's first block) as three classes of
// CTAs, each class with a fixed shared-memory layout:
//   class 0: latent segments of sequences with one query this step,
//   class 1: latent segments of sequences that insert a Beacon (two queries),
//   class 2: raw segments, one per (sequence, KV head).
// A segment's 128-key tiles are laid end to end with the other segments of
// its class; each CTA of the class takes one contiguous, equal range of that
// tile sequence, so a CTA may finish one segment and start the next (its
// pipeline keeps streaming across the boundary) and a long segment spreads
// over several CTAs.  Every (segment, CTA) intersection is a "piece" with its
// own partial output and LSE; the pieces of a segment are numbered
// consecutively, so the merge combines a contiguous range.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace slimkv {

constexpr int kTcTileKeys = 128;
constexpr int kTcClasses = 3;
constexpr int kTcMaxCtas = 160;          // CTAs of one launch (at most)

// Device-written plan (int32 words in the workspace), header then arrays.
// In the split-query plan (the 40-head layout, whose Q buffer holds one
// query) a latent segment is one (sequence, query): class 0 carries them all,
// id 2b + l, the two of a sequence adjacent; class 1 stays empty.
//   hdr[4k + 0..3] = CTAs, first CTA, segments, tiles of class k
//   seg_start[k] : [segments + 1] tile prefix of the class's segments
//   seg_piece[k] : [segments + 1] first piece of each segment (prefix)
//   seg_id[k]    : [segments] sequence b (latent) or b * Hkv + g (raw)
//   lat_seg[b]   : (class << 24) | segment of sequence b's latent segment
//   lat_range[b] : {(class << 24) | first piece in its class, pieces} of
//                  sequence b's latent segment (the merge's one lookup)
//   cta_start[k] : [CTAs + 1] first tile of each CTA of class k (then the
//                  class's tile count)
struct TcPlanLayout {
    int max_lat_segs;      // batch
    int max_raw_segs;      // batch * kv_heads
    // Word offsets inside the plan array.
    int hdr, seg_start[kTcClasses], seg_piece[kTcClasses], seg_id[kTcClasses], lat_seg, lat_range;
    int cta_start[kTcClasses];
    int words;
};

__host__ __device__ inline TcPlanLayout tc_plan_layout(int batch, int kv_heads, int split = 0) {
    TcPlanLayout L{};
    L.max_lat_segs = split ? 2 * batch : batch;
    L.max_raw_segs = batch * kv_heads;
    int at = 16;
    L.hdr = 0;
    for (int k = 0; k < kTcClasses; ++k) {
        const int n = k < 2 ? L.max_lat_segs : L.max_raw_segs;
        L.seg_start[k] = at; at += n + 1;
        L.seg_piece[k] = at; at += n + 1;
        L.seg_id[k] = at; at += n;
    }
    L.lat_seg = at; at += batch;
    at = (at + 1) & ~1;                      // int2 entries
    L.lat_range = at; at += 2 * batch;
    for (int k = 0; k < kTcClasses; ++k) {
        L.cta_start[k] = at;
        at += kTcMaxCtas + 1;
    }
    L.words = at;
    return L;
}

// Pieces a class can produce: one per segment plus one per CTA boundary
// that falls inside a segment.
__host__ __device__ inline int tc_max_pieces(int segments, int ctas) { return segments + ctas; }

// Inputs of the device planner.
struct TcPlanArgs {
    int batch, kv_heads, length;
    const int32_t* latent_len;
    const int32_t* raw_len;
    const int32_t* query_len;        // nullable: `length` for every sequence
    int lat_chunks;                  // 64-column chunks per latent key row (K + V)
    int ctas;                        // CTAs of the launch
    int raw_ctas;                    // > 0: CTAs of the raw class (else by volume)
    int with_raw;
    int split_queries;               // one latent segment per (sequence, query)
    int32_t* plan;
};

// Per-class job as the kernel sees it.
struct TcJob {
    int kchunks, vchunks;     // 64-column chunks of a K / V row
    int kv_heads;             // KV heads per sequence in the grid (1 for the latent branch)
    int group;                // query heads per KV head (rows of a Q box in row mode)
    int causal;               // two queries: the first excludes the last key (the new Beacon)
    int q_rows;               // Q read per query from [B*L][H][dim] rows (exact bf16: no lo part)
    int split;                // latent segments per (sequence, query): segment id 2b + l
    const int32_t* seqlens;   // keys per sequence
    const int32_t* qlens;     // queries per sequence (1 or 2), nullable
    int length;
    float scale_log2;
    int rows_alloc, out_width;
    float* part_o;            // [pieces][rows_alloc][out_width], row l * rows_per_query + head
    float* part_lse;          // [pieces][rows_alloc]
    int piece_base;           // first piece of this class in part_o / part_lse
    unsigned int* status;
    // Paged K/V (nullptr table = dense maps): row n of sequence b is row
    // n % slots of page table[b * table_stride + n / slots]; the K/V maps are
    // then one page map [pages][slots][W] and V starts at column v_col.
    const int32_t* table;
    int64_t table_stride;
    int slots, v_col, box_rows;   // box_rows: rows per page-map box (divides slots and 128)
    uint64_t wait_ns;             // bound of every pipeline wait
};

// One branch as the host describes it.
struct TcSide {
    const void* k;
    const void* v;
    int dim_k, dim_v;          // latent ranks, or the head dim
    int kv_heads, capacity;
    int64_t stride_batch, stride_row, stride_head;   // elements
    // Latent: q_hilo [B][128][width] bf16 with row hl*32*nq + l*32 + head
    // (hl 0 = hi, 1 = lo); 40 heads: [B][160][width] with row l*80 + hl*40 +
    // head.  Raw: q_rot [B][L][H][dim] bf16.
    const void* q;
    int q_rows, heads, group, causal;
    const int32_t* seqlens;
    int rows_alloc, width;
    float* part_o;
    float* part_lse;
    // Paged K/V: pages [num_pages] of page_stride elements holding
    // [sink][slots x (dim_k + dim_v)] (k / v unused).
    const void* pages;
    int64_t page_stride;
    int slots, sink_elements, num_pages;
    const int32_t* table;
    int64_t table_stride;
};

struct TcLaunch {
    int batch, length;
    float scale;
    const int32_t* query_len;
    unsigned int* status;
    TcSide lat, raw;
    int with_raw;
    int kv_heads;              // the plan's KV heads (raw segments per sequence)
    int wide;                  // 40 query heads, latent ranks <= 512 (split-query plan)
    int ctas;                  // grid size (persistent CTAs)
    const int32_t* plan;       // device plan written by plan_tc_work
    int lat_pieces;            // pieces reserved per latent class (class 1 starts after class 0's)
    uint64_t wait_ns;
    // The plan was written before the prologue: the launch may start while
    // the prologue finishes (programmatic dependent launch); the kernel waits
    // for it only before reading what the prologue writes (Q rows, the new
    // raw and Beacon rows).
    int early;
};

// Query heads of the latent branch the kernel is built for: 32 (ranks <=
// 320, both query counts in one CTA) or 40 (ranks <= 512 with an even
// number of 64-column V chunks, one query per CTA).
constexpr int kTcHeads = 32;
constexpr int kTcWideHeads = 40;
constexpr int kTcWideRows = 4 * kTcWideHeads;     // q_hilo rows per sequence (2 queries x hi, lo)

// Shared memory of the launch (same for every class).
size_t tc_smem_bytes();

int launch_decode_tc(const TcLaunch& launch, cudaStream_t stream);

}  // namespace slimkv
