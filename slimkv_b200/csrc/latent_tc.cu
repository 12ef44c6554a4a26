// Split-KV decode attention of both branches on the 5th-generation tensor
// cores: one persistent launch of at most one CTA per SM.
//
// Work.  The device plan (latent_tc_plan.cuh) puts every segment of a class
// — a sequence's latent rows (classes 0 and 1 by query count) or one (sequence,
// KV head) of raw rows (class 2) — end to end as 128-key tiles and gives each
// CTA of the class one contiguous, equal range of them.  A CTA walks its range
// piece by piece (a piece = the part of one segment inside the range); its
// loads, MMAs and softmax run across piece boundaries without draining, and
// every piece ends with a normalised partial output and LSE per query row.
//
// Per tile, swap-AB so the keys fill M:
//
//   S^T [128 keys x 64]        = K_tile . Q^T          (M=128, K-major A/B)
//   O^T [128 dims x 64] (x2,3) += V_pair^T . P^T       (M=128 over two 64-dim
//                                                       V chunks; M=64 for an
//                                                       odd last chunk)
//
// Q and P are split into bf16 hi + lo (x = hi + lo to ~16 mantissa bits), so
// the bf16 K/V tiles are used as stored and the result keeps fp32-level
// accuracy.  How the split uses the 64 MMA columns depends on the queries:
//   nq = 1: hi and lo are separate columns (cols 0-31 hi, 32-63 lo, one MMA
//           per k-step); the softmax and the epilogue add the two halves.
//   nq = 2: columns are (query, head); hi and lo accumulate into the same
//           columns (two MMAs per k-step).
// Raw pieces read exact bf16 query rows (no lo part): query l of head h of
// the group is row / score column 8 l + h, so the softmax handles 16 columns,
// and P^T holds hi in columns 0-15 and lo in 16-31 (one MMA per k-step).
//
// Streams.  K and V chunks (16 KB, [128 keys x 64 columns], 128-byte
// swizzle, no multicast) flow through two rings so that V chunks waiting for
// a tile's probabilities never hold up the K prefetch; Q has one buffer per
// latent CTA and two per raw CTA (raw pieces are short), and is reloaded per
// piece.  S and O are double-buffered in TMEM (O by piece, so the epilogue of
// one piece overlaps the next piece's first tiles).
//
// Softmax: one key per thread reading its TMEM lane, column maxima and sums
// via warp transpose-reduce, and a lazy rescale (the running max moves only
// when a column max exceeds it by 2^8).  The epilogue reads O from TMEM and
// stores the normalised rows directly (a warp writes 32 consecutive floats of
// a row).
//
// Warp roles (8 warps): 0 = TMA producer of Q and K, 1 = P.V issuer, 2 = TMEM
// allocator and S issuer, 3-6 = softmax / epilogue (TMEM lane quarters 3, 0,
// 1, 2), 7 = TMA producer of V.  No cluster multicast.  Every wait is bounded: on expiry the CTA reports
// SLIMKV_DEVICE_TIMEOUT, drains its copies and MMAs (bounded), frees TMEM and
// returns.
#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "host_utils.h"
#include "latent_tc.h"
#include "latent_tc_plan.cuh"

namespace slimkv {

namespace {

constexpr int kKeys = 128;
constexpr int kThreads8 = 256;
constexpr int kProducerV = 7;                        // warp of the V producer
constexpr int kMaxChunks = 5;                        // ranks <= 320
constexpr int kKRingMax = 6;
constexpr int kRawCols = 8;                          // raw score columns per query (group <= 8)
constexpr int kRawS = 2 * kRawCols;                  // raw score columns (two queries)
constexpr uint32_t kChunkBytes = 128 * 128;          // [128 keys x 64 bf16], 128-byte swizzle
constexpr uint32_t kQChunkBytes = 64 * 128;          // [64 rows x 64 bf16]
constexpr float kLazyLog2 = 8.f;
constexpr uint32_t kTmemCols = 512;
constexpr int kN = 64;                               // MMA N
constexpr uint32_t kOBufCols = 3 * kN;               // one O accumulator (<= 3 blocks)
constexpr uint32_t kSCol = 2 * kOBufCols;            // S buffers after the two O buffers
constexpr uint32_t kTileBytes = 224 * 1024;          // tile area of the largest layout

struct Misc {
    uint64_t kfull[kKRingMax], kempty[kKRingMax], vfull[kMaxChunks], vempty[kMaxChunks];
    uint64_t qfull[2], qempty[2], sfull[2], sempty[2], pfull[2], odone[2], oempty[2], final_mma;
    uint32_t tmem_base;
    int abort;
    float m_run[64], l_run[64], alpha[64];
    float red[4][64];
};
// The tiles start at the first 1024-byte boundary of dynamic shared memory
// (the base itself on this GPU; a base more than kMaxPad bytes short of a
// boundary is reported as SLIMKV_DEVICE_MISALIGNED), Misc right after them.
constexpr uint32_t kMaxPad = 960;
constexpr uint32_t kSmemBytes = kMaxPad + kTileBytes + uint32_t(sizeof(Misc));
static_assert(kSmemBytes <= 232448, "shared memory budget");

// Tile-area layout of a class: V ring | K ring | Q buffers | P buffers,
// and its TMEM map: `obufs` O accumulators of `o_cols` columns from column
// 0, two S buffers of `n` columns (the MMA N) from `s_col`.
// The raw class double-buffers P (pdbl: P(j) in buffer j & 1).
//
// 40-head latent layout (wide): N = 80 (hi | lo of one query), Q [80 rows x
// 64] per chunk (10 KB, 8 chunks), P^T [128 keys x 80] as two 64-column
// swizzle atoms (32 KB), a V ring of 4 slots that a tile's 8 chunks cycle
// through and a K ring of 3: 224 KB.  TMEM: one O of 4 x 80 columns (its
// epilogue finishes before the next piece's first P.V), S at 320 and 400.
struct Layout {
    int kring, vslots, qbufs, pbufs, obufs, n;
    bool pdbl;
    uint32_t off_k, off_q, qbytes, qchunk, off_p, o_cols, s_col;
};
template <bool WIDE>
__host__ __device__ __forceinline__ Layout class_layout(int cls, int kc) {
    Layout L;
    if (WIDE && cls < 2) {
        L.vslots = 4;
        L.kring = 3;
        L.pdbl = false;
        L.qbufs = 1;
        L.pbufs = 2;                                   // the two N atoms of one P
        L.n = 2 * kTcWideHeads;
        L.qchunk = uint32_t(L.n) * 128;
        L.qbytes = 8 * L.qchunk;
        L.obufs = 1;
        L.o_cols = 4 * uint32_t(L.n);
        L.s_col = L.o_cols;
    } else {
        L.vslots = cls == 2 ? 4 : kMaxChunks;
        L.kring = cls == 1 ? 2 : cls == 0 ? kMaxChunks : kKRingMax;
        L.pdbl = cls == 2;
        L.qbufs = cls == 2 ? 2 : 1;
        L.pbufs = cls == 0 ? 1 : 2;
        L.n = kN;
        L.qchunk = kQChunkBytes;
        L.qbytes = uint32_t(cls == 1 ? 2 : 1) * uint32_t(cls == 2 ? kc : kMaxChunks) * kQChunkBytes;
        L.obufs = 2;
        L.o_cols = kOBufCols;
        L.s_col = kSCol;
    }
    L.off_k = uint32_t(L.vslots) * kChunkBytes;
    L.off_q = L.off_k + uint32_t(L.kring) * kChunkBytes;
    L.off_p = L.off_q + uint32_t(L.qbufs) * L.qbytes;
    return L;
}

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, Misc* ms, unsigned* status,
                                              uint64_t limit) {
    if (ms->abort) return false;
    if (mbar_wait(bar, parity, limit)) return true;
    ms->abort = 1;
    report(status, SLIMKV_DEVICE_TIMEOUT);
    return false;
}

// OR of `pred` over the `count` threads of named barrier `id`.
__device__ __forceinline__ bool named_bar_or(int id, int count, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}\n"
        : "=r"(r)
        : "r"(uint32_t(pred)), "r"(id), "r"(count)
        : "memory");
    return r != 0;
}

// 16 columns: after this, lanes l and l + 16 hold the reduction of column
// v[l & 15] over the warp's 32 lanes (15 shuffles, then one across halves).
template <bool MAX>
__device__ __forceinline__ float warp_transpose_reduce16(float (&v)[16], int lane) {
#pragma unroll
    for (int half = 8; half >= 1; half >>= 1) {
        const bool upper = lane & half;
#pragma unroll
        for (int i = 0; i < half; ++i) {
            const float send = upper ? v[i] : v[i + half];
            const float keep = upper ? v[i + half] : v[i];
            const float recv = __shfl_xor_sync(0xffffffffu, send, half);
            v[i] = MAX ? fmaxf(keep, recv) : keep + recv;
        }
    }
    const float other = __shfl_xor_sync(0xffffffffu, v[0], 16);
    return MAX ? fmaxf(v[0], other) : v[0] + other;
}

// After this, lane `l` holds the reduction of column v[l] over the warp's 32
// lanes (a transpose-reduce: 31 shuffles for 32 columns).
template <bool MAX>
__device__ __forceinline__ float warp_transpose_reduce(float (&v)[32], int lane) {
#pragma unroll
    for (int half = 16; half >= 1; half >>= 1) {
        const bool upper = lane & half;
#pragma unroll
        for (int i = 0; i < half; ++i) {
            const float send = upper ? v[i] : v[i + half];
            const float keep = upper ? v[i + half] : v[i];
            const float recv = __shfl_xor_sync(0xffffffffu, send, half);
            v[i] = MAX ? fmaxf(keep, recv) : keep + recv;
        }
    }
    return v[0];
}

// Column reductions of x[0 .. NS) over the warp's 32 lanes into dst[0 ..
// NS): 32-column transpose-reduces, then one of 16 for a remainder of at
// most 16 columns (padded with the identity).
template <bool MAX, int NS>
__device__ __forceinline__ void transpose_reduce_to(const float* x, int lane, float* dst) {
#pragma unroll
    for (int g = 0; g < NS / 32; ++g) {
        float t[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) t[i] = x[32 * g + i];
        dst[32 * g + lane] = warp_transpose_reduce<MAX>(t, lane);
    }
    if constexpr (NS % 32 != 0) {
        static_assert(NS % 32 <= 16, "remainder of at most 16 columns");
        constexpr int R = NS % 32, G = NS - R;
        float t[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) t[i] = i < R ? x[G + i] : (MAX ? -INFINITY : 0.f);
        const float r = warp_transpose_reduce16<MAX>(t, lane);
        if (lane < R) dst[G + lane] = r;
    }
}

// Eight packed bf16 pairs of (hi, lo) for p[8u .. 8u+8).
template <int N>
__device__ __forceinline__ void split_hilo(const float (&p)[N], int u, uint4& hi, uint4& lo) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const float a0 = p[8 * u + 2 * e], a1 = p[8 * u + 2 * e + 1];
        const float h0 = bf16_round(a0), h1 = bf16_round(a1);
        h[e] = pack_bf16x2(h0, h1);
        l[e] = pack_bf16x2(a0 - h0, a1 - h1);
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// A CTA's place in its class: tile range [r0, r1) and the piece walk.
struct Range {
    const int32_t* start;   // class segment tile prefix
    const int32_t* pieces;  // class segment piece prefix
    const int32_t* ids;     // class segment -> b or b * Hkv + g
    int nseg;
    long long r0, r1;
    int s0, first_piece;
};

// One piece: segment s, its local tiles [t0, t1), and where its output goes
// (sequence b, KV head g of a raw segment, query l of a split latent one).
struct Piece {
    int s, t0, t1, piece, b, g, l;
};

// Piece k of the walk (k = 0, 1, ... while pos < r1); `s` and `pos` carry
// the walk's position.
__device__ __forceinline__ void next_piece(const Range& R, int k, int& s, long long& pos, int kv_heads, int split,
                                           Piece& p) {
    while (R.start[s + 1] <= pos) ++s;                 // skip segments without tiles
    const long long seg0 = R.start[s], seg1 = R.start[s + 1];
    p.s = s;
    p.t0 = int(pos - seg0);
    p.t1 = int(min(R.r1, seg1) - seg0);
    p.piece = k == 0 ? R.first_piece : R.pieces[s];
    const int id = R.ids[s];
    if (split) {
        p.b = id >> 1;
        p.l = id & 1;
        p.g = 0;
    } else {
        p.b = id / kv_heads;
        p.g = id - p.b * kv_heads;
        p.l = 0;
    }
    pos = seg0 + p.t1;
    ++s;
}

}  // namespace

// Kernel parameters: the K / V / Q maps of both branches (latent, raw), both
// jobs, the plan and its layout.  WIDE: the 40-head latent layout.
template <bool WIDE>
__global__ void __launch_bounds__(kThreads8, 1)
decode_tc_kernel(const __grid_constant__ CUtensorMap lkmap, const __grid_constant__ CUtensorMap lvmap,
                 const __grid_constant__ CUtensorMap lqmap, const __grid_constant__ CUtensorMap rkmap,
                 const __grid_constant__ CUtensorMap rvmap, const __grid_constant__ CUtensorMap rqmap,
                 const __grid_constant__ TcJob jl, const __grid_constant__ TcJob jr, const int32_t* __restrict__ plan,
                 const TcPlanLayout PL, int lat_pieces, int early) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    if (smem - smem_raw > int(kMaxPad)) {                     // uniform over the CTA, before any barrier
        if (threadIdx.x == 0) report(jl.status, SLIMKV_DEVICE_MISALIGNED);
        return;
    }
    Misc* ms = reinterpret_cast<Misc*>(smem + kTileBytes);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    // ---- class and range of this CTA ----
    int cls = -1, idx = 0;
    for (int k = 0; k < kTcClasses; ++k) {
        const int n = plan[PL.hdr + 4 * k], base = plan[PL.hdr + 4 * k + 1];
        if (int(blockIdx.x) >= base && int(blockIdx.x) < base + n) {
            cls = k;
            idx = int(blockIdx.x) - base;
        }
    }
    if (cls < 0) return;                                      // an idle CTA (before any barrier or TMEM)
    const bool is_lat = cls < 2;
    const TcJob& J = is_lat ? jl : jr;
    const CUtensorMap* kmap = is_lat ? &lkmap : &rkmap;
    const CUtensorMap* vmap = is_lat ? &lvmap : &rvmap;
    const CUtensorMap* qmap = is_lat ? &lqmap : &rqmap;
    Range R;
    R.start = plan + PL.seg_start[cls];
    R.pieces = plan + PL.seg_piece[cls];
    R.ids = plan + PL.seg_id[cls];
    R.nseg = plan[PL.hdr + 4 * cls + 2];
    const int32_t* cta_start = plan + PL.cta_start[cls];
    R.r0 = cta_start[idx];
    R.r1 = cta_start[idx + 1];
    if (R.r0 >= R.r1) return;
    R.s0 = tc_segment_of(R.start, R.nseg, R.r0);
    {
        int cnt = 0;                                          // CTAs <= idx starting strictly inside s0
        for (int j = idx; j >= 1; --j) {
            if (cta_start[j] > R.start[R.s0]) ++cnt;
            else break;
        }
        R.first_piece = R.pieces[R.s0] + cnt;
    }
    const int piece_base = J.piece_base + (cls == 1 ? lat_pieces : 0);
    const int kc = J.kchunks, vc = J.vchunks;
    const Layout LY = class_layout<WIDE>(cls, kc);
    const int kring = LY.kring;
    const uint64_t wait_ns = J.wait_ns;
    // V chunk c of CTA tile T: in V slot c; with <= 2 chunks per tile (raw)
    // tiles alternate between slot pairs (0,1) and (2,3), so two tiles of V
    // are in flight; with more chunks than slots (the wide layout, an even
    // chunk count) chunk n = T * vc + c cycles through the ring, so a chunk
    // pair always takes two adjacent slots.
    // The TMEM map, MMA N and Q chunk: compile-time constants outside the
    // wide layout.
    const int n_mma = WIDE ? LY.n : kN;
    const int obufs = WIDE ? LY.obufs : 2;
    const uint32_t o_cols = WIDE ? LY.o_cols : kOBufCols;
    const uint32_t s_col = WIDE ? LY.s_col : kSCol;
    const uint32_t qchunk = WIDE ? LY.qchunk : kQChunkBytes;
    const bool dbl = vc <= 2;
    const bool vring = WIDE && vc > LY.vslots;
    auto v_slot = [&](int T, int c) -> int {
        return vring ? (T * vc + c) % LY.vslots : dbl ? 2 * (T & 1) + c : c;
    };
    auto v_use = [&](int T, int c) -> int {                             // earlier uses of the slot
        return vring ? (T * vc + c) / LY.vslots : dbl ? T >> 1 : T;
    };

    if (J.q_rows) {
        // Row-mode Q fills only the query rows of each chunk; the rest must
        // read as zero in every piece.
        for (int i = tid; i < LY.qbufs * int(LY.qbytes / 16); i += kThreads8)
            reinterpret_cast<uint4*>(smem + LY.off_q)[i] = make_uint4(0, 0, 0, 0);
        fence_async_shared();
    }
    if (tid == 0) {
        for (int s = 0; s < kKRingMax; ++s) { mbar_init(&ms->kfull[s], 1); mbar_init(&ms->kempty[s], 1); }
        for (int s = 0; s < kMaxChunks; ++s) { mbar_init(&ms->vfull[s], 1); mbar_init(&ms->vempty[s], 1); }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&ms->qfull[s], 1);
            mbar_init(&ms->qempty[s], 1);
            mbar_init(&ms->sfull[s], 1);
            mbar_init(&ms->sempty[s], 4);
            mbar_init(&ms->oempty[s], 4);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&ms->pfull[s], 4);
            mbar_init(&ms->odone[s], 1);
        }
        mbar_init(&ms->final_mma, 2);
        ms->abort = 0;
        fence_barrier_init();
    }
    if (warp == 2) {
        tmem_alloc(&ms->tmem_base, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = ms->tmem_base;
    const uint32_t sbase = smem_u32(smem);
    const int vblocks = (vc + 1) / 2;

    if ((warp == 0 || warp == kProducerV) && lane == 0) {
        // ---- TMA producers: warp 0 streams each piece's Q then its K chunks,
        // warp 7 its V chunks.  Each waits (blocking, bounded) for the slot
        // its next copy needs, so the V stream never queues behind K
        // prefetches and neither thread polls.
        const bool kq = warp == 0;
        // Paged K/V: the page of each box of one tile, cached.
        struct PageCache { int b = -1, tile = -1; int page[kKeys / 16]; };
        PageCache pc;
        const int boxes = J.table ? kKeys / J.box_rows : 1;
        auto load_chunk = [&](uint8_t* dst, const CUtensorMap* map, uint64_t* bar, int col, const Piece& p, int tile) {
            if (!J.table) {
                tma_load_4d(dst, map, bar, col, p.g, tile * kKeys, p.b);
                return;
            }
            const int last = max(J.seqlens[p.b] - 1, 0);
            if (pc.b != p.b || pc.tile != tile) {
                pc.b = p.b;
                pc.tile = tile;
#pragma unroll
                for (int i = 0; i < kKeys / 16; ++i) {
                    if (i >= boxes) break;
                    const int key = min(tile * kKeys + J.box_rows * i, last);
                    pc.page[i] = __ldg(J.table + p.b * J.table_stride + key / J.slots);
                }
            }
#pragma unroll
            for (int i = 0; i < kKeys / 16; ++i) {
                if (i >= boxes) break;
                const int key = min(tile * kKeys + J.box_rows * i, last);
                tma_load_4d(dst + i * J.box_rows * 128, map, bar, col, 0, (key % J.slots) & ~(J.box_rows - 1),
                            pc.page[i]);
            }
        };
        int s = R.s0;
        long long pos = R.r0;
        bool ok = true;
        int j = 0;                                           // CTA tile
        // An early launch waits for the prologue before its first copy of
        // something the prologue writes: Q, and a segment's last tile (this
        // step's raw token or Beacon row).  Copies before that overlap it.
        bool waited = !early;
        auto await_prologue = [&]() {
            if (!waited) {
                grid_dependency_wait();
                waited = true;
            }
        };
        for (int k = 0; pos < R.r1 && ok; ++k) {
            Piece p;
            next_piece(R, k, s, pos, J.kv_heads, J.split, p);
            const int last_tile = (max(J.seqlens[p.b], 1) - 1) / kKeys;
            // Q of the piece, issued once the first K chunks of the piece that
            // fit the ring are on their way (S of the piece needs Q before it
            // frees a K slot).
            auto load_q = [&]() {
                await_prologue();
                const int qb = k % LY.qbufs;
                if (k >= LY.qbufs &&
                    !(ok = wait_or_abort(&ms->qempty[qb], ((k / LY.qbufs) - 1) & 1, ms, J.status, wait_ns)))
                    return;
                uint8_t* qdst = smem + LY.off_q + qb * LY.qbytes;
                const int nq = J.qlens ? J.qlens[p.b] : J.length;
                if (J.q_rows) {
                    // The group's query heads of query l -> rows kRawCols l + j
                    // (the other rows of the chunk stay zero from the start).
                    mbar_expect_tx(&ms->qfull[qb], uint32_t(kc * nq * J.group) * 128u);
                    for (int c = 0; c < kc; ++c)
                        for (int l = 0; l < nq; ++l)
                            tma_load_4d(qdst + c * kQChunkBytes + l * kRawCols * 128, qmap, &ms->qfull[qb], c * 64,
                                        0, p.g * J.group, p.b * J.length + l);
                } else if (J.split) {
                    // [hi | lo] x 40 rows of query l: one 80-row box per chunk.
                    mbar_expect_tx(&ms->qfull[qb], uint32_t(kc) * qchunk);
                    for (int c = 0; c < kc; ++c)
                        tma_load_4d(qdst + c * qchunk, qmap, &ms->qfull[qb], c * 64, 0, p.l * n_mma, p.b);
                } else {
                    // [hi | lo] x 32 * nq rows: one 64-row box per chunk for
                    // nq = 1, hi and lo boxes for nq = 2.
                    mbar_expect_tx(&ms->qfull[qb], uint32_t(nq * kc) * kQChunkBytes);
                    for (int c = 0; c < kc; ++c)
                        for (int hl = 0; hl < nq; ++hl)
                            tma_load_4d(qdst + (hl * kMaxChunks + c) * kQChunkBytes, qmap, &ms->qfull[qb], c * 64, 0,
                                        hl * 64, p.b);
                }
            };
            for (int t = p.t0; t < p.t1 && ok; ++t, ++j) {
                if (t == last_tile) await_prologue();
                if (kq) {
                    for (int c = 0; c < kc; ++c) {
                        const int n = j * kc + c, slot = n % kring;
                        if (n >= kring &&
                            !(ok = wait_or_abort(&ms->kempty[slot], ((n / kring) - 1) & 1, ms, J.status, wait_ns)))
                            break;
                        mbar_expect_tx(&ms->kfull[slot], kChunkBytes);
                        load_chunk(smem + LY.off_k + slot * kChunkBytes, kmap, &ms->kfull[slot], c * 64, p, t);
                        if (t == p.t0 && c == min(kc, kring) - 1) {
                            load_q();
                            if (!ok) break;
                        }
                    }
                } else {
                    for (int c = 0; c < vc; ++c) {
                        const int slot = v_slot(j, c), use = v_use(j, c);
                        if (use > 0 && !(ok = wait_or_abort(&ms->vempty[slot], (use - 1) & 1, ms, J.status, wait_ns)))
                            break;
                        mbar_expect_tx(&ms->vfull[slot], kChunkBytes);
                        load_chunk(smem + slot * kChunkBytes, vmap, &ms->vfull[slot], J.v_col + c * 64, p, t);
                    }
                }
            }
        }
    } else if (warp == 2 && lane == 0) {
        // ---- S issuer: S(j) = K(j) . Q^T as K chunks land ----
        const uint32_t idesc_s = umma_idesc_bf16(128, n_mma, 0, 0);
        int s = R.s0;
        long long pos = R.r0;
        bool ok = true;
        int j = 0;
        for (int k = 0; pos < R.r1 && ok; ++k) {
            Piece p;
            next_piece(R, k, s, pos, J.kv_heads, J.split, p);
            const int qb = k % LY.qbufs;
            const uint32_t q0 = sbase + LY.off_q + qb * LY.qbytes, q1 = q0 + kMaxChunks * kQChunkBytes;
            const int nq = J.qlens ? J.qlens[p.b] : J.length;
            const bool two = nq == 2 && !J.q_rows && !J.split;   // hi and lo into the same columns
            if (!(ok = wait_or_abort(&ms->qfull[qb], (k / LY.qbufs) & 1, ms, J.status, wait_ns))) break;
            for (int t = p.t0; t < p.t1; ++t, ++j) {
                const int sb = j & 1;
                const uint32_t s_tmem = tbase + s_col + uint32_t(sb * n_mma);
                if (j >= 2 && !(ok = wait_or_abort(&ms->sempty[sb], ((j - 2) >> 1) & 1, ms, J.status, wait_ns)))
                    break;
                tc_fence_after();
                for (int c = 0; c < kc; ++c) {
                    const int n = j * kc + c, slot = n % kring;
                    if (!(ok = wait_or_abort(&ms->kfull[slot], (n / kring) & 1, ms, J.status, wait_ns))) break;
                    tc_fence_after();
                    const uint32_t ka = sbase + LY.off_k + slot * kChunkBytes;
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint64_t ad = umma_desc_sw128(ka + kk * 32, 16, 1024);
                        umma_bf16(s_tmem, ad, umma_desc_sw128(q0 + c * qchunk + kk * 32, 16, 1024), idesc_s,
                                  (c | kk) != 0);
                        if (two)
                            umma_bf16(s_tmem, ad, umma_desc_sw128(q1 + c * kQChunkBytes + kk * 32, 16, 1024), idesc_s,
                                      1u);
                    }
                    umma_commit(&ms->kempty[slot]);
                }
                if (!ok) break;
                umma_commit(&ms->sfull[sb]);
            }
            if (ok) umma_commit(&ms->qempty[qb]);            // the piece's last MMA read Q
        }
        umma_commit(&ms->final_mma);
    } else if (warp == 1 && (WIDE || lane == 0)) {
        // ---- P.V issuer: O^T += V(j)^T . P(j)^T once P(j) is written ----
        // Lane 0 issues.  In the wide layout a tile's V chunks only land as
        // the ring turns, after P(j) is released, so the whole warp follows
        // lane 0 and clears the V rows past a sequence's length in its partial
        // last tile before their MMA (the cache may hold non-finite values
        // there, and 0 * inf would poison O).
        const unsigned wm = WIDE ? 0xffffffffu : 1u;       // the lanes taking part
        const bool leader = lane == 0;
        const bool clear_v = WIDE && is_lat;
        const uint32_t idesc_pair = umma_idesc_bf16(128, n_mma, 1, 1);
        const uint32_t idesc_one = umma_idesc_bf16(64, n_mma, 1, 1);
        const uint32_t p0 = sbase + LY.off_p, p1 = p0 + kChunkBytes;
        int s = R.s0;
        long long pos = R.r0;
        bool ok = true;
        int j = 0;
        for (int k = 0; pos < R.r1 && ok; ++k) {
            Piece p;
            next_piece(R, k, s, pos, J.kv_heads, J.split, p);
            const int ob = k % obufs;
            const uint32_t o_tmem = tbase + uint32_t(ob) * o_cols;
            const int nq = J.qlens ? J.qlens[p.b] : J.length;
            const bool cols = nq == 1 || J.q_rows || J.split;   // hi and lo in separate columns of one P
            const int n_keys = J.seqlens[p.b];
            const int valid_last = n_keys & (kKeys - 1);        // keys of a partial last tile (0: none)
            const int last_tile = (max(n_keys, 1) - 1) / kKeys;
            for (int t = p.t0; t < p.t1; ++t, ++j) {
                ok = __all_sync(wm, wait_or_abort(&ms->pfull[j & 1], (j >> 1) & 1, ms, J.status, wait_ns));
                if (!ok) break;
                const uint32_t pb = LY.pdbl ? p0 + uint32_t(j & 1) * kChunkBytes : p0;
                // The first tile of a piece overwrites the O buffer the
                // epilogue of piece k - obufs read.
                if (t == p.t0 && k >= obufs) {
                    ok = __all_sync(wm, wait_or_abort(&ms->oempty[ob], ((k / obufs) - 1) & 1, ms,
                                                               J.status, wait_ns));
                    if (!ok) break;
                }
                tc_fence_after();
                const bool clear = clear_v && t == last_tile && valid_last != 0;
                for (int blk = 0; blk < vblocks; ++blk) {
                    const int c0 = 2 * blk, s0 = v_slot(j, c0);
                    const bool pair = c0 + 1 < vc;
                    for (int c = c0; c <= c0 + (pair ? 1 : 0); ++c)
                        if (!(ok = wait_or_abort(&ms->vfull[v_slot(j, c)], v_use(j, c) & 1, ms, J.status, wait_ns)))
                            break;
                    ok = __all_sync(wm, ok);
                    if (!ok) break;
                    if (clear) {
                        for (int c = c0; c <= c0 + (pair ? 1 : 0); ++c) {
                            uint4* rows = reinterpret_cast<uint4*>(smem + v_slot(j, c) * kChunkBytes);
                            for (int i = valid_last * 8 + lane; i < kKeys * 8; i += 32) rows[i] = make_uint4(0, 0, 0, 0);
                        }
                        fence_async_shared();
                        __syncwarp(wm);
                    }
                    tc_fence_after();
                    if (leader) {
                        const uint32_t va = sbase + s0 * kChunkBytes;
                        const uint32_t o_b = o_tmem + uint32_t(blk * n_mma);
                        const uint32_t idesc = pair ? idesc_pair : idesc_one;
#pragma unroll
                        for (int ks = 0; ks < kKeys / 16; ++ks) {
                            const uint64_t ad = umma_desc_sw128(va + ks * 2048, kChunkBytes, 1024);
                            umma_bf16(o_b, ad, umma_desc_sw128(pb + ks * 2048, kChunkBytes, 1024), idesc,
                                      (t > p.t0 || ks > 0) ? 1u : 0u);
                            if (!cols)
                                umma_bf16(o_b, ad, umma_desc_sw128(p1 + ks * 2048, kChunkBytes, 1024), idesc, 1u);
                        }
                        umma_commit(&ms->vempty[s0]);
                        if (pair) umma_commit(&ms->vempty[v_slot(j, c0 + 1)]);
                    }
                    __syncwarp(wm);
                }
                if (!ok) break;
                if (leader) umma_commit(&ms->odone[j & 1]);
                __syncwarp(wm);
            }
        }
        if (leader) umma_commit(&ms->final_mma);
    } else if (warp >= 3 && warp <= 6 && cls < 2) {
        // ---- latent softmax and epilogue: thread <-> key (TMEM lane) ----
        // Instantiated per query count (class 0: one query, class 1: two), so
        // a CTA runs straight-line code for its own layout only.  S has NC =
        // 2 HQ columns per key: hi | lo products of one query (added here),
        // or (query, head) with hi and lo accumulated by the MMA (two queries
        // of 32 heads); NS scores per key, one running row state per score
        // column.
        auto latent_softmax = [&](auto nq_tag) {
            constexpr int NQ = decltype(nq_tag)::value;
            constexpr int HQ = WIDE ? kTcWideHeads : kTcHeads;
            constexpr int NC = 2 * HQ;
            constexpr int NS = NQ * HQ;
            constexpr bool cols = NQ == 1;
            // One query: each thread keeps partial row sums of its own keys
            // across the piece's tiles, reduced across the CTA once, in the
            // epilogue (no per-tile reduction or barrier for them); two
            // queries (64 columns) reduce per tile.
            constexpr bool thread_sums = NQ == 1;
            static_assert(NS <= 64 && (NQ == 1 || HQ == 32), "latent score columns per CTA");
            const int quarter = warp & 3;
            const int t_local = 32 * quarter + lane;
            const uint32_t lane_addr = uint32_t(32 * quarter) << 16;
            const int st = tid - 96;                      // 0..127
            bool failed = false;
            int s = R.s0;
            long long pos = R.r0;
            int j = 0;
            for (int k = 0; pos < R.r1 && !failed; ++k) {
                Piece p;
                next_piece(R, k, s, pos, J.kv_heads, J.split, p);
                const int ob = k % obufs;
                const uint32_t o_tmem = tbase + uint32_t(ob) * o_cols;
                const int n_keys = J.seqlens[p.b];
                const int nq_seq = J.qlens ? J.qlens[p.b] : J.length;
                // Keys of the first query's rows: an insertion step's raw query
                // excludes the new Beacon (the sequence's last key).
                const bool excl = J.causal && nq_seq == 2 && (NQ == 2 || (J.split && p.l == 0));
                const int lim0 = excl ? n_keys - 1 : n_keys;
                const int row0 = J.split ? p.l * HQ : 0;          // output row of head 0
                const int n_tiles = (max(n_keys, 0) + kKeys - 1) / kKeys;
                if (st < 64) {
                    ms->m_run[st] = -INFINITY;
                    ms->l_run[st] = 0.f;
                }
                float lsum[thread_sums ? NS : 1];
#pragma unroll
                for (int i = 0; i < (thread_sums ? NS : 1); ++i) lsum[i] = 0.f;
                named_bar(1, 128);
                // An early launch starts its first piece with a dry tile (t = t0 - 1):
                // the tile code runs once on zero scores while the prologue finishes, so
                // the real tiles find it in the instruction cache.  It waits on and
                // signals nothing; its row state is reset after it and its P write lands
                // in a buffer no MMA reads yet.
                for (int t = p.t0 - (k == 0 && early ? 1 : 0); t < p.t1; ++t) {
                    const bool dry = t < p.t0;
                    const int sb = j & 1;
                    const uint32_t s_tmem = tbase + s_col + uint32_t(sb * n_mma);
                    const int key = t * kKeys + t_local;
                    bool ok = dry || wait_or_abort(&ms->sfull[sb], (j >> 1) & 1, ms, J.status, wait_ns);
                    if (named_bar_or(1, 128, !ok)) { failed = true; break; }
                    tc_fence_after();
                    float v[NC];
                    if (dry) {
#pragma unroll
                        for (int c = 0; c < NC; ++c) v[c] = 0.f;
                    } else {
                        tmem_ld_cols<NC>(s_tmem + lane_addr, v);
                    }
                    tmem_wait_ld();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0 && !dry) mbar_arrive(&ms->sempty[sb]);
                    if constexpr (cols) {
#pragma unroll
                        for (int h = 0; h < HQ; ++h) v[h] += v[HQ + h];       // hi + lo products
                    }
                    // scale and mask
#pragma unroll
                    for (int i = 0; i < NS; ++i) v[i] = key < (i < HQ ? lim0 : n_keys) ? v[i] * J.scale_log2 : -INFINITY;
                    // Column maxima only when some score exceeds its row's running
                    // max by more than the lazy threshold (always on a piece's first
                    // tile): otherwise the max stays and every p <= 2^8.
                    bool over = t <= p.t0;
                    if (!over) {
#pragma unroll
                        for (int i = 0; i < NS; ++i) over |= v[i] > ms->m_run[i] + kLazyLog2;
                    }
                    const bool rescan = named_bar_or(1, 128, over);
                    bool need_fix = false;
                    if (rescan) {
                        transpose_reduce_to<true, NS>(v, lane, ms->red[quarter]);
                        named_bar(1, 128);
                        if (st < NS) {
                            const float tm =
                                fmaxf(fmaxf(ms->red[0][st], ms->red[1][st]), fmaxf(ms->red[2][st], ms->red[3][st]));
                            const float mo = ms->m_run[st];
                            float mn = mo, alpha = 1.f;
                            if (tm != -INFINITY && (mo == -INFINITY || tm > mo + kLazyLog2)) {
                                mn = fmaxf(mo, tm);
                                alpha = mo == -INFINITY ? 0.f : exp2f(mo - mn);
                            }
                            ms->alpha[st] = alpha;
                            ms->m_run[st] = mn;
                            ms->l_run[st] *= alpha;
                        }
                        need_fix = named_bar_or(1, 128, st < NS && t > p.t0 && ms->alpha[st] != 1.f);
                        if constexpr (thread_sums) {
#pragma unroll
                            for (int i = 0; i < NS; ++i) lsum[i] *= ms->alpha[i];
                        }
                    }
                    // P(j) overwrites the buffer P.V(j-1) reads: wait for it.
                    if (j > 0) {
                        ok = wait_or_abort(&ms->odone[(j - 1) & 1], ((j - 1) >> 1) & 1, ms, J.status, wait_ns);
                        if (named_bar_or(1, 128, !ok)) { failed = true; break; }
                        tc_fence_after();
                    }
                    // The sequence's partial last tile: V rows past the length hold
                    // whatever the cache has there; P is zero for them, and zeroing
                    // the rows too keeps a non-finite stale value from turning 0 * x
                    // into NaN.  Each thread clears its own key row once the chunk
                    // has landed (P.V(j) does not start before P(j) is released).
                    // The wide layout's P.V warp does this instead.
                    if constexpr (!WIDE) {
                        if (!dry && t == n_tiles - 1 && (n_keys & (kKeys - 1)) != 0) {
                            bool okc = true;
                            if (key >= n_keys) {
                                for (int c = 0; c < vc && okc; ++c) {
                                    const int slot = v_slot(j, c);
                                    okc = wait_or_abort(&ms->vfull[slot], v_use(j, c) & 1, ms, J.status, wait_ns);
                                    if (okc) {
                                        uint4* row = reinterpret_cast<uint4*>(smem + slot * kChunkBytes + t_local * 128);
#pragma unroll
                                        for (int u = 0; u < 8; ++u) row[u] = make_uint4(0, 0, 0, 0);
                                    }
                                }
                            }
                            if (named_bar_or(1, 128, !okc)) { failed = true; break; }
                        }
                    }
                    if (need_fix) {
                        // O^T column c of a block belongs to row c mod HQ (hi | lo)
                        // or to row c (two queries).
                        for (int blk = 0; blk < vblocks; ++blk) {
#pragma unroll
                            for (int c0 = 0; c0 < NC; c0 += 32) {
                                const uint32_t addr = o_tmem + lane_addr + uint32_t(blk * n_mma + c0);
                                if (c0 + 32 <= NC) {
                                    float o[32];
                                    tmem_ld32(addr, o);
                                    tmem_wait_ld();
#pragma unroll
                                    for (int i = 0; i < 32; ++i) o[i] *= ms->alpha[cols ? (c0 + i) % HQ : c0 + i];
                                    tmem_st32(addr, o);
                                } else {
                                    float o[16];
                                    tmem_ld16(addr, o);
                                    tmem_wait_ld();
#pragma unroll
                                    for (int i = 0; i < 16; ++i) o[i] *= ms->alpha[cols ? (c0 + i) % HQ : c0 + i];
                                    tmem_st16(addr, o);
                                }
                            }
                        }
                        tmem_wait_st();
                    }
                    // Probabilities -> P^T row of this key: column 8u of the hi part
                    // and HQ + 8u (hi | lo) or 64 + 8u (two queries: the lo buffer)
                    // of the lo part, in 64-column swizzle atoms kChunkBytes apart.
                    uint8_t* prow = smem + LY.off_p + t_local * 128;
                    float pr[NS];
#pragma unroll
                    for (int i = 0; i < NS; ++i) {
                        const float m = ms->m_run[i];
                        pr[i] = v[i] == -INFINITY ? 0.f : sfu_exp2(v[i] - m);     // finite v => finite m
                    }
#pragma unroll
                    for (int u = 0; u < NS / 8; ++u) {
                        uint4 hi, lo;
                        split_hilo(pr, u, hi, lo);
                        const int ch = 8 * u, cl = (cols ? HQ : 64) + 8 * u;
                        *reinterpret_cast<uint4*>(prow + (ch >> 6) * kChunkBytes + ((((ch & 63) >> 3) ^ (t_local & 7)) << 4)) = hi;
                        *reinterpret_cast<uint4*>(prow + (cl >> 6) * kChunkBytes + ((((cl & 63) >> 3) ^ (t_local & 7)) << 4)) = lo;
                    }
                    if constexpr (thread_sums) {
#pragma unroll
                        for (int i = 0; i < NS; ++i) lsum[i] += pr[i];
                    } else {
                        transpose_reduce_to<false, NS>(pr, lane, ms->red[quarter]);
                    }
                    fence_async_shared();
                    tc_fence_before();
                    if constexpr (!thread_sums) {
                        named_bar(1, 128);
                        if (st < NS)
                            ms->l_run[st] += ms->red[0][st] + ms->red[1][st] + ms->red[2][st] + ms->red[3][st];
                    }
                    __syncwarp();
                    if (dry) {
                        if (st < 64) {
                            ms->m_run[st] = -INFINITY;
                            ms->l_run[st] = 0.f;
                        }
#pragma unroll
                        for (int i = 0; i < (thread_sums ? NS : 1); ++i) lsum[i] = 0.f;
                        named_bar(1, 128);
                        continue;
                    }
                    if (lane == 0) mbar_arrive(&ms->pfull[j & 1]);
                    ++j;
                }
                if (failed) break;
                // ---- epilogue of the piece: normalised partial output and LSE ----
                {
                    const bool ok = wait_or_abort(&ms->odone[(j - 1) & 1], ((j - 1) >> 1) & 1, ms, J.status, wait_ns);
                    if (named_bar_or(1, 128, !ok)) { failed = true; break; }
                }
                tc_fence_after();
                if constexpr (thread_sums) {
                    transpose_reduce_to<false, NS>(lsum, lane, ms->red[quarter]);
                    named_bar(1, 128);
                    if (st < NS) ms->l_run[st] = ms->red[0][st] + ms->red[1][st] + ms->red[2][st] + ms->red[3][st];
                }
                named_bar(1, 128);                     // every thread's l_run update is in
                if (st < 64) ms->alpha[st] = (st < NS && ms->l_run[st] > 0.f) ? 1.f / ms->l_run[st] : 0.f;
                named_bar(1, 128);
                const int piece = piece_base + p.piece;
                float* out = J.part_o + (int64_t)piece * J.rows_alloc * J.out_width;
                // The row scales in registers: read between the global stores
                // through a generic pointer they would be reloaded every time.
                float al[NS];
#pragma unroll
                for (int i = 0; i < NS; ++i) al[i] = ms->alpha[i];
                for (int blk = 0; blk < vblocks; ++blk) {
                    const bool pair = 2 * blk + 1 < vc;
                    float o[NC];
                    tmem_ld_cols<NC>(o_tmem + lane_addr + uint32_t(blk * n_mma), o);
                    tmem_wait_ld();
                    // An M=128 block holds dim 32q + L of its chunk pair in lane L
                    // of quarter q; the M=64 block holds dim 16q + L in lane L < 16.
                    if (pair || lane < 16) {
                        const int d = 128 * blk + (pair ? 32 * quarter + lane : 16 * quarter + lane);
                        if constexpr (cols) {
                            float* dst = out + (int64_t)row0 * J.out_width + d;
#pragma unroll
                            for (int h = 0; h < HQ; ++h) dst[h * J.out_width] = (o[h] + o[HQ + h]) * al[h];
                        } else {
#pragma unroll
                            for (int c = 0; c < NC; ++c) out[c * J.out_width + d] = o[c] * al[c];
                        }
                    }
                }
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&ms->oempty[ob]);
                // Output row of score column i: row0 + i (head h of query l at l * HQ + h).
                if (st < NS) {
                    const float lsum = ms->l_run[st];
                    J.part_lse[(int64_t)piece * J.rows_alloc + row0 + st] =
                        lsum > 0.f ? (ms->m_run[st] + log2f(lsum)) * 0.69314718055994530942f : -INFINITY;
                }
                // A split sequence's other query has no keys in this piece.
                if (J.split && nq_seq == 2 && st < HQ)
                    J.part_lse[(int64_t)piece * J.rows_alloc + (HQ - row0) + st] = -INFINITY;
                named_bar(1, 128);                     // m_run / l_run / alpha are reset by the next piece
            }
        };
        if constexpr (WIDE) latent_softmax(std::integral_constant<int, 1>{});
        else if (cls == 0) latent_softmax(std::integral_constant<int, 1>{});
        else latent_softmax(std::integral_constant<int, 2>{});
    } else if (warp >= 3 && warp <= 6) {
        // ---- raw softmax and epilogue: thread <-> key, 16 score columns ----
        // Column l * kRawCols + h holds query l of head h of the group (Q rows
        // in that order); P^T carries the bf16 hi parts in columns 0-15 and
        // the lo parts in 16-31 of buffer j & 1, so P(j) is written while
        // P.V(j - 1) still reads the other buffer.
        const int quarter = warp & 3;
        const int t_local = 32 * quarter + lane;
        const uint32_t lane_addr = uint32_t(32 * quarter) << 16;
        const int st = tid - 96;                      // 0..127
        const int rg = J.group;
        bool failed = false;
        int s = R.s0;
        long long pos = R.r0;
        int j = 0;
        for (int k = 0; pos < R.r1 && !failed; ++k) {
            Piece p;
            next_piece(R, k, s, pos, J.kv_heads, J.split, p);
            const int ob = k & 1;
            const uint32_t o_tmem = tbase + uint32_t(ob) * o_cols;
            const int n_keys = J.seqlens[p.b];
            const int nq = J.qlens ? J.qlens[p.b] : J.length;
            const int n_tiles = (max(n_keys, 0) + kKeys - 1) / kKeys;
            if (st < kRawS) {
                ms->m_run[st] = -INFINITY;
                ms->l_run[st] = 0.f;
            }
            named_bar(1, 128);
            // A dry first tile on an early launch, as in the latent branch.
            for (int t = p.t0 - (k == 0 && early ? 1 : 0); t < p.t1; ++t) {
                const bool dry = t < p.t0;
                const int sb = j & 1;
                const uint32_t s_tmem = tbase + s_col + uint32_t(sb * n_mma);
                const int key = t * kKeys + t_local;
                bool ok = dry || wait_or_abort(&ms->sfull[sb], (j >> 1) & 1, ms, J.status, wait_ns);
                if (named_bar_or(1, 128, !ok)) { failed = true; break; }
                tc_fence_after();
                float v[kRawS];
                if (dry) {
#pragma unroll
                    for (int c = 0; c < kRawS; ++c) v[c] = 0.f;
                } else {
                    tmem_ld16(s_tmem + lane_addr, v);
                }
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0 && !dry) mbar_arrive(&ms->sempty[sb]);
#pragma unroll
                for (int c = 0; c < kRawS; ++c) v[c] = key < n_keys ? v[c] * J.scale_log2 : -INFINITY;
                bool over = t <= p.t0;
                if (!over) {
#pragma unroll
                    for (int c = 0; c < kRawS; ++c) over |= v[c] > ms->m_run[c] + kLazyLog2;
                }
                const bool rescan = named_bar_or(1, 128, over);
                bool need_fix = false;
                if (rescan) {
                    float tmp[kRawS];
#pragma unroll
                    for (int c = 0; c < kRawS; ++c) tmp[c] = v[c];
                    const float r = warp_transpose_reduce16<true>(tmp, lane);
                    if (lane < kRawS) ms->red[quarter][lane] = r;
                    named_bar(1, 128);
                    if (st < kRawS) {
                        const float tm =
                            fmaxf(fmaxf(ms->red[0][st], ms->red[1][st]), fmaxf(ms->red[2][st], ms->red[3][st]));
                        const float mo = ms->m_run[st];
                        float mn = mo, alpha = 1.f;
                        if (tm != -INFINITY && (mo == -INFINITY || tm > mo + kLazyLog2)) {
                            mn = fmaxf(mo, tm);
                            alpha = mo == -INFINITY ? 0.f : exp2f(mo - mn);
                        }
                        ms->alpha[st] = alpha;
                        ms->m_run[st] = mn;
                        ms->l_run[st] *= alpha;
                    }
                    need_fix = named_bar_or(1, 128, st < kRawS && t > p.t0 && ms->alpha[st] != 1.f);
                }
                // P(j) overwrites the buffer P.V(j - 2) read; rescaling O needs
                // P.V(j - 1) done (a commit covers every earlier MMA).
                {
                    const int w = need_fix ? j - 1 : j - 2;
                    if (w >= 0 && !dry) {
                        ok = wait_or_abort(&ms->odone[w & 1], (w >> 1) & 1, ms, J.status, wait_ns);
                        if (named_bar_or(1, 128, !ok)) { failed = true; break; }
                        tc_fence_after();
                    }
                }
                // The partial last tile: clear the V rows past the length (see
                // the latent branch).
                if (!dry && t == n_tiles - 1 && (n_keys & (kKeys - 1)) != 0) {
                    bool okc = true;
                    if (key >= n_keys) {
                        for (int c = 0; c < vc && okc; ++c) {
                            const int slot = v_slot(j, c);
                            okc = wait_or_abort(&ms->vfull[slot], v_use(j, c) & 1, ms, J.status, wait_ns);
                            if (okc) {
                                uint4* row = reinterpret_cast<uint4*>(smem + slot * kChunkBytes + t_local * 128);
#pragma unroll
                                for (int u = 0; u < 8; ++u) row[u] = make_uint4(0, 0, 0, 0);
                            }
                        }
                    }
                    if (named_bar_or(1, 128, !okc)) { failed = true; break; }
                }
                if (need_fix) {
                    // O^T columns c (hi) and 16 + c (lo) belong to score column c.
                    for (int blk = 0; blk < vblocks; ++blk) {
                        float o[32];
                        const uint32_t addr = o_tmem + lane_addr + uint32_t(blk * n_mma);
                        tmem_ld32(addr, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int c = 0; c < 32; ++c) o[c] *= ms->alpha[c & (kRawS - 1)];
                        tmem_st32(addr, o);
                    }
                    tmem_wait_st();
                }
                uint8_t* prow = smem + LY.off_p + uint32_t(j & 1) * kChunkBytes + t_local * 128;
                float pr[kRawS];
#pragma unroll
                for (int c = 0; c < kRawS; ++c) {
                    const float m = ms->m_run[c];
                    pr[c] = v[c] == -INFINITY ? 0.f : sfu_exp2(v[c] - m);     // finite v => finite m
                }
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    uint4 hi, lo;
                    split_hilo(pr, u, hi, lo);
                    *reinterpret_cast<uint4*>(prow + ((u ^ (t_local & 7)) << 4)) = hi;
                    *reinterpret_cast<uint4*>(prow + (((u + 2) ^ (t_local & 7)) << 4)) = lo;
                }
                {
                    const float r = warp_transpose_reduce16<false>(pr, lane);
                    if (lane < kRawS) ms->red[quarter][lane] = r;
                }
                fence_async_shared();
                tc_fence_before();
                named_bar(1, 128);
                if (st < kRawS)
                    ms->l_run[st] += ms->red[0][st] + ms->red[1][st] + ms->red[2][st] + ms->red[3][st];
                __syncwarp();
                if (dry) {
                    if (st < kRawS) {
                        ms->m_run[st] = -INFINITY;
                        ms->l_run[st] = 0.f;
                    }
                    named_bar(1, 128);
                    continue;
                }
                if (lane == 0) mbar_arrive(&ms->pfull[j & 1]);
                ++j;
            }
            if (failed) break;
            // ---- epilogue of the piece ----
            {
                const bool ok = wait_or_abort(&ms->odone[(j - 1) & 1], ((j - 1) >> 1) & 1, ms, J.status, wait_ns);
                if (named_bar_or(1, 128, !ok)) { failed = true; break; }
            }
            tc_fence_after();
            named_bar(1, 128);                     // every thread's l_run update is in
            if (st < kRawS) ms->alpha[st] = ms->l_run[st] > 0.f ? 1.f / ms->l_run[st] : 0.f;
            named_bar(1, 128);
            const int piece = piece_base + p.piece;
            float* out = J.part_o + (int64_t)piece * J.rows_alloc * J.out_width;
            float al[kRawS];
#pragma unroll
            for (int c = 0; c < kRawS; ++c) al[c] = ms->alpha[c];
            for (int blk = 0; blk < vblocks; ++blk) {
                const bool pair = 2 * blk + 1 < vc;
                float o[32];
                tmem_ld32(o_tmem + lane_addr + uint32_t(blk * n_mma), o);
                tmem_wait_ld();
                if (pair || lane < 16) {
                    const int d = 128 * blk + (pair ? 32 * quarter + lane : 16 * quarter + lane);
#pragma unroll
                    for (int l = 0; l < 2; ++l) {
                        if (l < nq) {
#pragma unroll
                            for (int h = 0; h < kRawCols; ++h) {
                                const int c = l * kRawCols + h;
                                if (h < rg) out[(l * rg + h) * J.out_width + d] = (o[c] + o[kRawS + c]) * al[c];
                            }
                        }
                    }
                }
            }
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&ms->oempty[ob]);
            if (st < kRawS) {
                const int l = st / kRawCols, h = st % kRawCols;
                if (l < nq && h < rg) {
                    const float lsum = ms->l_run[st];
                    J.part_lse[(int64_t)piece * J.rows_alloc + l * rg + h] =
                        lsum > 0.f ? (ms->m_run[st] + log2f(lsum)) * 0.69314718055994530942f : -INFINITY;
                }
            }
            named_bar(1, 128);                     // m_run / l_run / alpha are reset by the next piece
        }
    }
    __syncthreads();
    if (tid == 64) {
        // Both issuers committed final_mma after their last MMA: every MMA has
        // completed before TMEM is freed (bounded wait, independent of the
        // pipeline bound so that a short one cannot free TMEM under an MMA).
        mbar_wait(&ms->final_mma, 0, 2000000000ull);
    }
    if (ms->abort && tid == 0) {
        // Drain: wait (bounded) for the last copy issued into every slot.
        for (int s = 0; s < kring; ++s) {
            mbar_wait(&ms->kfull[s], 0, 100000000ull);
            mbar_wait(&ms->kfull[s], 1, 100000000ull);
        }
        for (int s = 0; s < LY.vslots; ++s) {
            mbar_wait(&ms->vfull[s], 0, 100000000ull);
            mbar_wait(&ms->vfull[s], 1, 100000000ull);
        }
        for (int s = 0; s < LY.qbufs; ++s) {
            mbar_wait(&ms->qfull[s], 0, 100000000ull);
            mbar_wait(&ms->qfull[s], 1, 100000000ull);
        }
    }
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tbase, kTmemCols);
    }
    // Every CTA issues this at its end, so the merge launch (which waits for
    // this grid's completion before reading its partials) can be set up while
    // the last CTAs finish, never ahead of a CTA that has not started.
    if (tid == 0) grid_launch_dependents();
}

namespace {

int make_side(const TcSide& S, int batch, int length, float scale, const int32_t* qlens, unsigned* status,
              uint64_t wait_ns, bool wide, TcJob& J, CUtensorMap& km, CUtensorMap& vm, CUtensorMap& qm) {
    // The wide latent branch: 40 heads, ranks <= 512 with an even number of
    // 64-column V chunks (a chunk pair takes two adjacent ring slots).
    const bool wide_lat = wide && !S.q_rows;
    const int max_dim = wide_lat ? 512 : 320;
    if (S.dim_k > max_dim || S.dim_v > max_dim || S.width < 64 || S.width % 64 || S.rows_alloc < 2 * S.group ||
        (reinterpret_cast<uintptr_t>(S.part_o) & 15) || (wide_lat ? S.group != kTcWideHeads : S.group > kTcHeads) ||
        (wide_lat && ((S.dim_v + 63) / 64) % 2))
        return fail(SLIMKV_ERR_UNSUPPORTED_SHAPE, "tensor-core decode attention: unsupported branch shape");
    int rc, box_rows = 128;
    if (S.pages) {
        // One map over the pages: (W columns, slots rows, pages);
        // K chunks at columns [0, dim_k), V chunks from dim_k.
        const int W = S.dim_k + S.dim_v;
        if (S.slots % 16 || S.dim_k % 8 || S.sink_elements % 8 || S.page_stride % 8 || S.num_pages <= 0 || !S.table ||
            (reinterpret_cast<uintptr_t>(S.pages) & 15))
            return fail(SLIMKV_ERR_UNSUPPORTED_SHAPE,
                        "paged latent attention needs 16-row-aligned pages (slots %% 16, ranks %% 8, 16-byte aligned)");
        const void* base = static_cast<const uint16_t*>(S.pages) + S.sink_elements;
        const uint64_t row = uint64_t(W) * 2, page = uint64_t(S.page_stride) * 2;
        // dims (W, 1, slots, pages), box {64, 1, box_rows, 1}: the largest
        // power of two <= 128 dividing slots, so boxes never cross pages.
        while (S.slots % box_rows) box_rows /= 2;
        if ((rc = encode_map_4d(&km, base, W, 1, S.slots, S.num_pages, row, row, page, box_rows))) return rc;
        vm = km;
    } else {
        const uint64_t head_bytes = S.kv_heads > 1 ? uint64_t(S.stride_head) * 2 : uint64_t(S.stride_row) * 2;
        if ((rc = encode_map_4d(&km, S.k, S.dim_k, S.kv_heads, S.capacity, batch, head_bytes,
                                uint64_t(S.stride_row) * 2, uint64_t(S.stride_batch) * 2, kKeys)))
            return rc;
        if ((rc = encode_map_4d(&vm, S.v, S.dim_v, S.kv_heads, S.capacity, batch, head_bytes,
                                uint64_t(S.stride_row) * 2, uint64_t(S.stride_batch) * 2, kKeys)))
            return rc;
    }
    if (S.q_rows && (S.group > kRawCols || S.causal || length > 2))
        return fail(SLIMKV_ERR_UNSUPPORTED_SHAPE, "tensor-core decode attention: raw branch needs group <= 8");
    if (S.q_rows) {
        // q_rot [B][L][H][dim] as (dim, 1, H, B * L), boxes of `group` rows.
        const uint64_t row = uint64_t(S.dim_k) * 2;
        if ((rc = encode_map_4d(&qm, S.q, S.dim_k, 1, S.heads, uint64_t(batch) * length, row, row, row * S.heads,
                                S.group)))
            return rc;
    } else if (wide_lat) {
        // q_hilo [B][160][width]: boxes of one query's 80 rows.
        const uint64_t row = uint64_t(S.width) * 2;
        if ((rc = encode_map_4d(&qm, S.q, S.width, 1, kTcWideRows, batch, row, row, row * kTcWideRows,
                                2 * kTcWideHeads)))
            return rc;
    } else {
        const uint64_t row = uint64_t(S.width) * 2;
        if ((rc = encode_map_4d(&qm, S.q, S.width, 1, 128, batch, row, row, row * 128, 64))) return rc;
    }
    J = TcJob{};
    J.kchunks = (S.dim_k + 63) / 64;
    J.vchunks = (S.dim_v + 63) / 64;
    J.kv_heads = S.kv_heads;
    J.group = S.group;
    J.causal = S.causal;
    J.q_rows = S.q_rows;
    J.split = wide_lat ? 1 : 0;
    J.seqlens = S.seqlens;
    J.qlens = qlens;
    J.length = length;
    J.scale_log2 = scale * 1.4426950408889634f;
    J.rows_alloc = S.rows_alloc;
    J.out_width = S.width;
    J.part_o = S.part_o;
    J.part_lse = S.part_lse;
    J.piece_base = 0;
    J.status = status;
    J.table = S.pages ? S.table : nullptr;
    J.table_stride = S.table_stride;
    J.slots = S.slots;
    J.v_col = S.pages ? S.dim_k : 0;
    J.box_rows = box_rows;
    J.wait_ns = wait_ns;
    return SLIMKV_OK;
}

}  // namespace

size_t tc_smem_bytes() { return kSmemBytes; }

namespace {

template <bool WIDE>
int launch_tc(const TcLaunch& L, const CUtensorMap& lk, const CUtensorMap& lv, const CUtensorMap& lq,
              const CUtensorMap& rk, const CUtensorMap& rv, const CUtensorMap& rq, const TcJob& jl, const TcJob& jr,
              cudaStream_t stream) {
    // Every class layout fits the tile area (latent K chunks for classes 0-1,
    // two for raw).
    for (int cls = 0; cls < kTcClasses; ++cls) {
        const Layout LY = class_layout<WIDE>(cls, cls == 2 ? 2 : jl.kchunks);
        if (LY.off_p + uint32_t(LY.pbufs) * kChunkBytes > kTileBytes ||
            (cls < 2 && uint32_t(jl.kchunks) * LY.qchunk > LY.qbytes))
            return fail(SLIMKV_ERR_UNSUPPORTED_SHAPE, "tensor-core decode attention: class %d layout too large", cls);
    }
    auto kernel = decode_tc_kernel<WIDE>;
    static bool configured[64] = {};
    const int dev = device_info().device;
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemBytes)) != cudaSuccess)
            return fail(SLIMKV_ERR_CUDA, "cudaFuncSetAttribute (decode tc) failed");
        configured[dev] = true;
    }
    const TcPlanLayout PL = tc_plan_layout(L.batch, L.kv_heads, WIDE ? 1 : 0);
    // An early launch may start before the previous kernel (the prologue)
    // ends; the kernel waits for it before reading what it writes.
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(L.ctas);
    cfg.blockDim = dim3(kThreads8);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = L.early ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, lk, lv, lq, rk, rv, rq, jl, jr, L.plan, PL, L.lat_pieces, L.early);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return fail(SLIMKV_ERR_CUDA, "decode tc launch failed: %s", cudaGetErrorString(e));
    return SLIMKV_OK;
}

}  // namespace

int launch_decode_tc(const TcLaunch& L, cudaStream_t stream) {
    CUtensorMap lk, lv, lq, rk, rv, rq;
    TcJob jl, jr;
    int rc;
    const uint64_t wait_ns = L.wait_ns ? L.wait_ns : 2000000000ull;
    const bool wide = L.wide != 0;
    if ((rc = make_side(L.lat, L.batch, L.length, L.scale, L.query_len, L.status, wait_ns, wide, jl, lk, lv, lq)))
        return rc;
    if (L.with_raw) {
        if ((rc = make_side(L.raw, L.batch, L.length, L.scale, L.query_len, L.status, wait_ns, wide, jr, rk, rv, rq)))
            return rc;
        if (jr.kchunks > 2 || jr.vchunks > 2)
            return fail(SLIMKV_ERR_UNSUPPORTED_SHAPE, "tensor-core decode attention: raw head dim above 128");
    } else {
        jr = jl;
        rk = lk; rv = lv; rq = lq;
    }
    return wide ? launch_tc<true>(L, lk, lv, lq, rk, rv, rq, jl, jr, stream)
                : launch_tc<false>(L, lk, lv, lq, rk, rv, rq, jl, jr, stream);
}

}  // namespace slimkv
