// Device planner of the persistent tcgen05 decode attention (latent_tc.h).
//
// Run by one thread block (the prologue's first block, so it needs no launch
// of its own) from this step's device lengths:
//   1. segments: the latent rows of every sequence (class 0 for one query,
//      class 1 for two; with split queries, one class-0 segment per
//      (sequence, query)) and the raw rows of every (sequence, KV head)
//      (class 2), in sequence order, with the tile prefix of each class;
//   2. CTAs per class in proportion to the bytes the class streams, weighted
//      by how fast its layout streams them;
//   3. pieces: one per segment plus one per CTA boundary falling inside a
//      segment; seg_piece is their prefix, so segment s owns pieces
//      [seg_piece[s], seg_piece[s + 1]).
// The attention CTAs recompute their ranges from the header (class tile
// count x i / CTAs) and find their segments by binary search.
#pragma once

#include "latent_tc.h"

namespace slimkv {

// Exclusive prefix of v over the block; *total receives the block sum.
// blockDim.x a multiple of 32 (<= 1024); every thread must call it.
__device__ inline int block_exclusive_scan(int v, int* total, int* s_warp) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) s_warp[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = lane < nw ? s_warp[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        if (lane < nw) s_warp[lane] = w;
    }
    __syncthreads();
    const int before = warp ? s_warp[warp - 1] : 0;
    *total = s_warp[nw - 1];
    __syncthreads();
    return before + x - v;
}

__device__ inline int tc_tiles_of(int len) { return len > 0 ? (len + kTcTileKeys - 1) / kTcTileKeys : 0; }

// Largest s in [0, n) with start[s] <= r (start[0] = 0 <= r).
__device__ inline int tc_segment_of(const int32_t* start, int n, long long r) {
    int lo = 0, hi = n - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (start[mid] <= r) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

// First tile of CTA i of a class with `tiles` tiles over `ctas` CTAs.
__device__ __host__ inline long long tc_cta_start(int tiles, int ctas, int i) {
    return (long long)tiles * i / ctas;
}

// Relative cost of a tile by class, in 16 KB latent chunks streamed: a
// class-0 tile counts its chunks; the two-query layout (class 1, a K ring of
// two chunks) streams them more slowly; a raw tile (64 KB, with a Q load and
// an epilogue every few tiles) costs TcPlanArgs::raw_weight, which the host
// sets from measured launch times (raw_tile_weight()).  With the piece-aware
// shares, two-query weights of 1.3 / 1.5 / 1.6 against 1.4 gave 76 / 75 / 72.6
// against 75.5 us at config 2 and 835 / 820 / 788 against 786 us at config 3
// (kernel-only); 1.6 then measured 74.0 against 72.5 us per launch in the full
// 32-layer bench, so 1.4 stays.
#ifndef SLIMKV_TC_W_TWO_QUERY
#define SLIMKV_TC_W_TWO_QUERY 1.4f
#endif
// CTA boundaries move to a segment edge within (tiles per CTA) / this.
#ifndef SLIMKV_TC_SNAP_DIV
#define SLIMKV_TC_SNAP_DIV 4
#endif
#ifndef SLIMKV_TC_W_RAW_FRACTION
#define SLIMKV_TC_W_RAW_FRACTION 0.65f
#endif
#ifndef SLIMKV_TC_W_RAW_WIDE
#define SLIMKV_TC_W_RAW_WIDE 7.5f
#endif
// The raw tile's weight: 0.65 of a class-0 tile in the 32-head layout (the
// best of the fractions tried at config 2, 10 chunks per latent tile, and at
// config 3, 6 chunks in pages, with the piece-aware boundaries below: 0.75
// gave 77 / 807 us, 0.65 75.4 / 797 us, 0.55 74.2 / 874 us); 7.5 chunks in the
// 40-head layout (config 5, 16 chunks per latent tile: 706 us against 731 us
// at 0.75 x 16).
// Piece overhead, in tiles of its class, for placing CTA boundaries: every
// piece (a segment, or the part of one, inside a CTA) pays a Q load, the
// pipeline drain before its epilogue and the epilogue.  Globaltimer stamps of
// a config-2 launch put it at ~4 us per raw piece against ~1.25 us per raw
// tile, and at ~6 us per latent piece against ~4 us per latent tile; over
// the round values tried, 3.2 / 1.5 made the launch 3 % faster at config 2
// (79.3 -> 77.0 us) and 5 % faster at config 3 (851 -> 806 us).  The 40-head
// layout keeps equal tile shares (every value tried there was slower).
#ifndef SLIMKV_TC_BOUND_RAW
#define SLIMKV_TC_BOUND_RAW 3.2f
#endif
#ifndef SLIMKV_TC_BOUND_LAT
#define SLIMKV_TC_BOUND_LAT 1.5f
#endif
__host__ __device__ inline float raw_tile_weight(int lat_chunks, bool wide) {
    return wide ? SLIMKV_TC_W_RAW_WIDE : SLIMKV_TC_W_RAW_FRACTION * float(lat_chunks);
}

// `scratch` (shared memory, `scratch_words` ints): when the whole plan fits,
// it is built there — every prefix, binary search and atomic stays on chip —
// and copied to `a.plan` at the end; otherwise it is built in place.
__device__ inline void plan_tc_work(const TcPlanArgs& a, int32_t* scratch, int scratch_words) {
    __shared__ int s_warp[32];
    const TcPlanLayout L = tc_plan_layout(a.batch, a.kv_heads, a.split_queries);
    const bool on_chip = L.words <= scratch_words;
    int32_t* P = on_chip ? scratch : a.plan;
    const int tid = threadIdx.x;
    if (on_chip) {
        for (int i = tid; i < L.words; i += blockDim.x) P[i] = 0;
        __syncthreads();
    }
    // 1. Latent segments of both classes, raw tile prefix.
    int carry[5] = {0, 0, 0, 0, 0};      // segments / tiles of class 0, 1; raw tiles
    for (int b0 = 0; b0 < a.batch; b0 += blockDim.x) {
        const int b = b0 + tid;
        const bool ok = b < a.batch;
        const int nq = ok ? (a.query_len ? a.query_len[b] : a.length) : 1;
        const int cls = nq == 2 && !a.split_queries ? 1 : 0;
        const int ns = a.split_queries ? nq : 1;        // latent segments of sequence b
        const int tl = ok ? tc_tiles_of(a.latent_len[b]) : 0;
        const int tr = ok && a.with_raw ? tc_tiles_of(a.raw_len[b]) : 0;
        int tot[5];
        const int seg0 = block_exclusive_scan(ok && cls == 0 ? ns : 0, &tot[0], s_warp);
        const int til0 = block_exclusive_scan(ok && cls == 0 ? ns * tl : 0, &tot[1], s_warp);
        const int seg1 = block_exclusive_scan(ok && cls == 1, &tot[2], s_warp);
        const int til1 = block_exclusive_scan(ok && cls == 1 ? tl : 0, &tot[3], s_warp);
        const int rawp = block_exclusive_scan(tr, &tot[4], s_warp);
        if (ok) {
            const int seg = cls ? carry[2] + seg1 : carry[0] + seg0;
            const int til = cls ? carry[3] + til1 : carry[1] + til0;
            for (int q = 0; q < ns; ++q) {
                P[L.seg_start[cls] + seg + q] = til + q * tl;
                P[L.seg_id[cls] + seg + q] = a.split_queries ? 2 * b + q : b;
            }
            P[L.lat_seg + b] = (cls << 24) | seg;
            // Raw segments (b, g): tile prefix Hkv * (raw tiles before b) + g * tr.
            const int rbase = a.kv_heads * (carry[4] + rawp);
            for (int g = 0; g < a.kv_heads; ++g) {
                P[L.seg_start[2] + b * a.kv_heads + g] = rbase + g * tr;
                P[L.seg_id[2] + b * a.kv_heads + g] = b * a.kv_heads + g;
            }
        }
        for (int k = 0; k < 5; ++k) carry[k] += tot[k];
    }
    const int nseg[3] = {carry[0], carry[2], a.with_raw ? a.batch * a.kv_heads : 0};
    const int tiles[3] = {carry[1], carry[3], a.with_raw ? a.kv_heads * carry[4] : 0};
    if (tid < 3) P[L.seg_start[tid] + nseg[tid]] = tiles[tid];
    // 2. CTAs per class (thread 0).
    if (tid == 0) {
        const float w[3] = {float(tiles[0]) * a.lat_chunks, SLIMKV_TC_W_TWO_QUERY * tiles[1] * a.lat_chunks,
                            raw_tile_weight(a.lat_chunks, a.split_queries != 0) * tiles[2]};
        // A raw CTA count given by the caller is kept; the other classes share
        // the rest by weight, at least one CTA each and at most one per tile.
        const bool fixed2 = a.raw_ctas > 0 && tiles[2] > 0;
        int n[3] = {0, 0, fixed2 ? min(a.raw_ctas, tiles[2]) : 0};
        const int avail = a.ctas - n[2];
        const float wl = w[0] + w[1] + (fixed2 ? 0.f : w[2]);
        for (int k = 0; k < 3; ++k)
            if (!(fixed2 && k == 2) && tiles[k] > 0) n[k] = min(tiles[k], max(1, int(avail * w[k] / wl + 0.5f)));
        for (;;) {                       // too many: take from the class with the most CTAs
            if (n[0] + n[1] + n[2] <= a.ctas) break;
            int kmax = -1;
            for (int k = 0; k < 3; ++k)
                if (!(fixed2 && k == 2) && n[k] > 1 && (kmax < 0 || n[k] > n[kmax])) kmax = k;
            if (kmax < 0) break;
            --n[kmax];
        }
        for (;;) {                       // too few: give to the class with the most work per CTA
            if (n[0] + n[1] + n[2] >= a.ctas) break;
            int kbest = -1;
            float best = 0.f;
            for (int k = 0; k < 3; ++k)
                if (!(fixed2 && k == 2) && n[k] > 0 && n[k] < tiles[k] && w[k] / n[k] > best) {
                    best = w[k] / n[k];
                    kbest = k;
                }
            if (kbest < 0) break;
            ++n[kbest];
        }
        int base = 0;
        for (int k = 0; k < 3; ++k) {
            P[L.hdr + 4 * k + 0] = n[k];
            P[L.hdr + 4 * k + 1] = base;
            P[L.hdr + 4 * k + 2] = nseg[k];
            P[L.hdr + 4 * k + 3] = tiles[k];
            base += n[k];
        }
    }
    __syncthreads();
    // 3. CTA ranges: equal shares of the class's tiles, each boundary moved to
    // a segment boundary within a quarter share of it (a piece costs a query
    // load and an epilogue; a boundary on a segment edge adds none).  Then
    // the pieces of every segment: zero for an empty one, else one plus the
    // CTA boundaries strictly inside it.
    if (tid < 3) {
        const int k = tid, n = P[L.hdr + 4 * k], ns = nseg[k];
        const int32_t* start = P + L.seg_start[k];
        int32_t* cs = P + L.cta_start[k];
        const long long snap = n > 0 && SLIMKV_TC_SNAP_DIV > 0 ? (long long)tiles[k] / n / SLIMKV_TC_SNAP_DIV : 0;
        // Equal shares of the class's cost: segment s starts at tile start[s]
        // and at cost start[s] + c s, its piece overhead c (in tiles) paid
        // before its first tile; a share boundary inside an overhead lands on
        // the segment's first tile.
        const float c = a.split_queries ? 0.f : (k == 2 ? SLIMKV_TC_BOUND_RAW : SLIMKV_TC_BOUND_LAT);
        const double cost = double(tiles[k]) + double(c) * ns;
        long long prev = 0;
        cs[0] = 0;
        for (int i = 1; i < n; ++i) {
            long long r = tc_cta_start(tiles[k], n, i);
            if (c > 0.f) {
                const double rc = cost * i / n;
                int lo = 0, hi = ns - 1;                 // last segment whose cost start is <= rc
                while (lo < hi) {
                    const int mid = (lo + hi + 1) >> 1;
                    if (double(start[mid]) + double(c) * mid <= rc) lo = mid;
                    else hi = mid - 1;
                }
                const double off = rc - double(start[lo]) - double(c) * (lo + 1);
                const long long len = start[lo + 1] - start[lo];
                r = start[lo] + (off <= 0.0 ? 0 : min(len, (long long)(off + 0.5)));
            }
            const int s = tc_segment_of(start, ns, r);
            if (r - start[s] <= snap) r = start[s];
            else if (start[s + 1] - r <= snap) r = start[s + 1];
            r = max(r, prev);
            cs[i] = int(r);
            prev = r;
        }
        if (n > 0) cs[n] = tiles[k];
    }
    __syncthreads();
    for (int k = 0; k < 3; ++k) {
        const int n = P[L.hdr + 4 * k], ns = nseg[k];
        int32_t* start = P + L.seg_start[k];
        int32_t* piece = P + L.seg_piece[k];
        const int32_t* cs = P + L.cta_start[k];
        for (int s = tid; s < ns; s += blockDim.x) piece[s] = start[s + 1] > start[s] ? 1 : 0;
        __syncthreads();
        for (int i = 1 + tid; i < n; i += blockDim.x) {
            const long long r = cs[i];
            if (r == cs[i - 1] || r >= tiles[k]) continue;     // an empty CTA adds no boundary
            const int s = tc_segment_of(start, ns, r);
            if (r > start[s]) atomicAdd(piece + s, 1);
        }
        __syncthreads();
        int carry_p = 0;
        for (int s0 = 0; s0 < ns; s0 += blockDim.x) {
            const int s = s0 + tid;
            const int v = s < ns ? piece[s] : 0;
            int total;
            const int ex = block_exclusive_scan(v, &total, s_warp);
            if (s < ns) piece[s] = carry_p + ex;
            carry_p += total;
        }
        if (tid == 0) piece[ns] = carry_p;
        __syncthreads();
    }
    // 4. Each sequence's latent piece range (both query segments of a split
    // sequence: they are adjacent).
    for (int b = tid; b < a.batch; b += blockDim.x) {
        const int ls = P[L.lat_seg + b], cls = ls >> 24, s = ls & 0xffffff;
        const int ns = a.split_queries ? (a.query_len ? a.query_len[b] : a.length) : 1;
        const int32_t* pc = P + L.seg_piece[cls];
        P[L.lat_range + 2 * b] = (cls << 24) | pc[s];
        P[L.lat_range + 2 * b + 1] = pc[s + ns] - pc[s];
    }
    __syncthreads();
    if (on_chip)
        for (int i = tid; i < L.words; i += blockDim.x) a.plan[i] = P[i];
}

}  // namespace slimkv
