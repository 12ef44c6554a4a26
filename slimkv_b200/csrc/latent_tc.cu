// Latent-branch split-KV decode attention on the 5th-generation tensor cores.
//
// One CTA owns (sequence b, split): a contiguous range of 128-key tiles of
// the sequence's latent cache against all query rows of the step (32 heads x
// nq = 1 or 2 queries).  Swap-AB so the keys fill M:
//
//   S^T [128 keys x 64]        = K_tile . Q^T          (M=128, K-major A/B)
//   O^T [128 dims x 64] (x2,3) += V_pair^T . P^T       (M=128 over two 64-dim
//                                                       V chunks; M=64 for an
//                                                       odd last chunk)
//
// Q and P are split into bf16 hi + lo (x = hi + lo to ~16 mantissa bits), so
// the bf16 K/V tiles are used as stored and the result keeps fp32-level
// accuracy.  How the split uses the 64 MMA columns depends on nq:
//   nq = 1: hi and lo are separate columns (cols 0-31 hi, 32-63 lo, one MMA
//           per k-step); the softmax and the epilogue add the two halves.
//   nq = 2: columns are (query, head); hi and lo accumulate into the same
//           columns (two MMAs per k-step).
//
// Streams.  K and V chunks (16 KB, [128 keys x 64 columns], 128-byte
// swizzle) flow through two rings so the V chunks that wait for a tile's
// probabilities never hold up the K prefetch: a K ring (5 slots, 2 for
// nq = 2) and a V ring of one tile (chunk c of every tile in slot c, so the
// chunk pairs of the M=128 products are always adjacent).  Two threads issue
// MMAs: one computes S(j) as K chunks land, the other P.V(j) once P(j) is
// written; each commits the ring slots it read.  S is double-buffered in TMEM.
//
// Softmax: one key per thread reading its TMEM lane, column maxima and sums
// via warp transpose-reduce, and a lazy rescale (the running max moves only
// when a column max exceeds it by 2^8, so the TMEM read-modify-write of O^T is
// rare).  The epilogue stages the normalised partial output in shared memory
// and writes it with bulk tensor stores.
//
// Warp roles (7 warps): 0 = TMA producer, 1 = P.V issuer, 2 = TMEM allocator
// and S issuer, 3-6 = softmax / epilogue (TMEM lane quarters 3, 0, 1, 2).  No
// cluster multicast.  Every wait is bounded: on expiry the CTA reports
// SLIMKV_DEVICE_TIMEOUT, drains its copies and MMAs (bounded), frees TMEM and
// returns.
#include <algorithm>

#include "common.cuh"
#include "host_utils.h"
#include "latent_tc.h"

namespace slimkv {

namespace {

constexpr int kKeys = 128;
constexpr int kThreads7 = 224;
constexpr int kMaxChunks = 5;                        // ranks <= 320
constexpr int kKRingMax = 5;
constexpr uint32_t kChunkBytes = 128 * 128;          // [128 keys x 64 bf16], 128-byte swizzle
constexpr uint32_t kQChunkBytes = 64 * 128;          // [64 rows x 64 bf16]
constexpr float kLazyLog2 = 8.f;
constexpr uint32_t kTmemCols = 512;
constexpr int kN = 64;                               // MMA N
constexpr uint64_t kWaitNs = 2000000000ull;

// Shared memory: V ring (5 slots) | K ring (5 slots for nq = 1, 2 for nq = 2)
// | Q (nq x 40 KB) | P (nq x 16 KB) | ... | Misc at a fixed offset.
__host__ __device__ constexpr int k_ring_slots(int nq) { return nq == 1 ? 5 : 2; }
constexpr uint32_t kOffK = kMaxChunks * kChunkBytes;
constexpr uint32_t kOffMisc = kOffK + 2 * kChunkBytes + 2 * kMaxChunks * kQChunkBytes + 2 * kChunkBytes;
static_assert(kOffK + 5 * kChunkBytes + kMaxChunks * kQChunkBytes + kChunkBytes <= kOffMisc, "single-query layout");

struct Misc {
    uint64_t kfull[kKRingMax], kempty[kKRingMax], vfull[kMaxChunks], vempty[kMaxChunks];
    uint64_t qfull, sfull[2], sempty[2], pfull, odone, final_mma;
    uint32_t tmem_base;
    int abort;
    float m_run[64], l_run[64], alpha[64];
    float red[4][64];
};
constexpr uint32_t kSmemBytes = kOffMisc + sizeof(Misc) + 1024;
static_assert(kSmemBytes <= 232448, "shared memory budget");

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, Misc* ms, unsigned* status) {
    if (ms->abort) return false;
    if (mbar_wait(bar, parity, kWaitNs)) return true;
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

// Eight packed bf16 pairs of (hi, lo) for p[8u .. 8u+8).
__device__ __forceinline__ void split_hilo(const float (&p)[32], int u, uint4& hi, uint4& lo) {
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

}  // namespace

// CTAs [0, n_lat) take latent work (b, split); the rest raw work
// (b, KV head g, split).  Each branch has its own K / V / Q / partial-output
// maps and job.
__global__ void __launch_bounds__(kThreads7, 1)
decode_tc_kernel(const __grid_constant__ CUtensorMap lkmap, const __grid_constant__ CUtensorMap lvmap,
                 const __grid_constant__ CUtensorMap lqmap, const __grid_constant__ CUtensorMap lomap,
                 const __grid_constant__ CUtensorMap rkmap, const __grid_constant__ CUtensorMap rvmap,
                 const __grid_constant__ CUtensorMap rqmap, const __grid_constant__ CUtensorMap romap,
                 const __grid_constant__ TcJob jl, const __grid_constant__ TcJob jr, int n_lat) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Misc* ms = reinterpret_cast<Misc*>(smem + kOffMisc);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool is_lat = int(blockIdx.x) < n_lat;
    const TcJob& J = is_lat ? jl : jr;
    const CUtensorMap* kmap = is_lat ? &lkmap : &rkmap;
    const CUtensorMap* vmap = is_lat ? &lvmap : &rvmap;
    const CUtensorMap* qmap = is_lat ? &lqmap : &rqmap;
    const CUtensorMap* omap = is_lat ? &lomap : &romap;
    const int idx = is_lat ? int(blockIdx.x) : int(blockIdx.x) - n_lat;
    int split = idx % J.splits, bg = idx / J.splits, nsplits = J.splits;
    if (J.work) {
        // Work-list item; the whole CTA leaves on an unused entry.
        const int item = __ldg(J.work + idx);
        if (item < 0) return;
        split = item & 31;
        nsplits = (item >> 5) & 63;
        bg = (item >> 11) * J.kv_heads;
    }
    const int b = bg / J.kv_heads, g = bg - b * J.kv_heads;
    const int z = bg * J.splits + split;                     // partial-output slot
    const int n_keys = J.seqlens[b];
    const int nq = J.qlens ? J.qlens[b] : J.length;          // 1 or 2 queries
    const bool cols = nq == 1;                               // hi / lo as separate columns
    const int rows = 32 * nq;
    const int kring = k_ring_slots(nq);
    const int kc = J.kchunks, vc = J.vchunks;
    const uint32_t off_q = kOffK + uint32_t(kring) * kChunkBytes;
    const uint32_t off_p = off_q + uint32_t(nq * kMaxChunks) * kQChunkBytes;
    const int n_tiles = (max(n_keys, 0) + kKeys - 1) / kKeys;
    // Tiles spread evenly over the sequence's splits.
    const int t0 = int((int64_t)split * n_tiles / nsplits);
    const int t1 = int((int64_t)(split + 1) * n_tiles / nsplits);
    const int nt = max(0, t1 - t0);
    const int total_k = nt * kc, total_v = nt * vc;
    // K chunk n -> (tile n / kc, chunk n % kc) in ring slot n % kring.
    // V chunk n -> (tile T = n / vc, chunk c = n % vc) in V slot c; with <= 2
    // chunks per tile (the raw branch) tiles alternate between slot pairs
    // (0,1) and (2,3), so two tiles of V are in flight.
    const bool dbl = vc <= 2;
    auto v_slot = [&](int T, int c) -> int { return dbl ? 2 * (T & 1) + c : c; };
    auto v_use = [&](int T) -> int { return dbl ? T >> 1 : T; };     // earlier uses of the slot
    // Paged K/V: the page of each 16-key block of one tile, cached in
    // registers per stream (K runs ahead of V).  Keys past the length read a
    // valid page (their scores are masked and their V rows zeroed).
    // Paged K/V: the page of each 16-key block of one tile, cached in
    // registers per stream (K runs ahead of V).  Keys past the length read a
    // valid page (their scores are masked and their V rows zeroed).
    // A tile is J.box_rows-row boxes (box_rows = gcd(slots, 128) >= 16, so
    // no box crosses a page).
    struct PageCache { int tile = -1; int page[kKeys / 16]; };
    PageCache kpc, vpc;
    const int boxes = J.table ? kKeys / J.box_rows : 1;
    auto fill_pages = [&](PageCache& pc, int tile) {
        if (pc.tile == tile) return;
        pc.tile = tile;
        const int last = max(n_keys - 1, 0);
#pragma unroll
        for (int i = 0; i < kKeys / 16; ++i) {
            if (i >= boxes) break;
            const int key = min(tile * kKeys + J.box_rows * i, last);
            pc.page[i] = __ldg(J.table + b * J.table_stride + key / J.slots);
        }
    };
    // One 16 KB chunk [128 keys x 64 columns] at column col: one box of the
    // dense map, or 128 / box_rows boxes of the page map.
    auto load_chunk = [&](uint8_t* dst, const CUtensorMap* map, uint64_t* bar, int col, int tile, PageCache& pc) {
        if (!J.table) {
            tma_load_4d(dst, map, bar, col, g, tile * kKeys, b);
            return;
        }
        fill_pages(pc, tile);
        const int last = max(n_keys - 1, 0);
#pragma unroll
        for (int i = 0; i < kKeys / 16; ++i) {
            if (i >= boxes) break;
            const int key = min(tile * kKeys + J.box_rows * i, last);
            tma_load_4d(dst + i * J.box_rows * 128, map, bar, col, 0, (key % J.slots) & ~(J.box_rows - 1),
                        pc.page[i]);
        }
    };
    auto issue_k = [&](int n) {
        const int slot = n % kring;
        mbar_expect_tx(&ms->kfull[slot], kChunkBytes);
        load_chunk(smem + kOffK + slot * kChunkBytes, kmap, &ms->kfull[slot], (n % kc) * 64, t0 + n / kc, kpc);
    };
    auto issue_v = [&](int n) {
        const int c = n % vc, slot = v_slot(n / vc, c);
        mbar_expect_tx(&ms->vfull[slot], kChunkBytes);
        load_chunk(smem + slot * kChunkBytes, vmap, &ms->vfull[slot], J.v_col + c * 64, t0 + n / vc, vpc);
    };

    if (warp == 0 && J.q_rows && nt > 0) {
        // Row-mode Q fills only the valid rows of each chunk: zero the rest.
        for (int i = lane; i < kc * int(kQChunkBytes / 16); i += 32)
            reinterpret_cast<uint4*>(smem + off_q)[i] = make_uint4(0, 0, 0, 0);
        fence_async_shared();
        __syncwarp();
    }
    if (tid == 0) {
        for (int s = 0; s < kKRingMax; ++s) { mbar_init(&ms->kfull[s], 1); mbar_init(&ms->kempty[s], 1); }
        for (int s = 0; s < kMaxChunks; ++s) { mbar_init(&ms->vfull[s], 1); mbar_init(&ms->vempty[s], 1); }
        mbar_init(&ms->qfull, 1);
        for (int s = 0; s < 2; ++s) { mbar_init(&ms->sfull[s], 1); mbar_init(&ms->sempty[s], 4); }
        mbar_init(&ms->pfull, 4);
        mbar_init(&ms->odone, 1);
        mbar_init(&ms->final_mma, 2);
        ms->abort = 0;
        fence_barrier_init();
        // The streams start at once: Q, the first ring's worth of K chunks and
        // the first tile's V chunks (first use of each slot needs no wait)
        // overlap the setup below.
        if (nt > 0) {
            if (J.q_rows) {
                // The group's query heads of query l -> rows 32 l + j.
                mbar_expect_tx(&ms->qfull, uint32_t(kc * nq * J.group) * 128u);
                for (int c = 0; c < kc; ++c)
                    for (int l = 0; l < nq; ++l)
                        tma_load_4d(smem + off_q + c * kQChunkBytes + l * 32 * 128, qmap, &ms->qfull, c * 64, 0,
                                    g * J.group, b * J.length + l);
            } else {
                // Q rows of the sequence: [hi | lo] x 32 * nq (one 64-row box
                // per chunk for nq = 1, hi and lo boxes for nq = 2).
                mbar_expect_tx(&ms->qfull, uint32_t(nq * kc) * kQChunkBytes);
                for (int c = 0; c < kc; ++c)
                    for (int hl = 0; hl < nq; ++hl)
                        tma_load_4d(smem + off_q + (hl * kMaxChunks + c) * kQChunkBytes, qmap, &ms->qfull, c * 64,
                                    0, hl * 64, b);
            }
            for (int n = 0; n < kring && n < total_k; ++n) issue_k(n);
            for (int n = 0; n < (dbl ? 2 * vc : vc) && n < total_v; ++n) issue_v(n);
        }
    }
    if (warp == 2) {
        tmem_alloc(&ms->tmem_base, kTmemCols);
        tmem_relinquish();
    }
    if (tid >= 96 && tid < 160) {
        ms->m_run[tid - 96] = -INFINITY;
        ms->l_run[tid - 96] = 0.f;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = ms->tmem_base;
    const uint32_t o_tmem = tbase;                         // up to 3 blocks x 64 columns
    const uint32_t s_tmem0 = tbase + 3 * kN;               // two 64-column buffers
    const uint32_t sbase = smem_u32(smem);
    const int vblocks = (vc + 1) / 2;

    if (nt > 0) {
        if (warp == 0 && lane == 0) {
            // ---- TMA producer: K chunks first whenever a K slot is free ----
            int nk = min(kring, total_k), nv = min(dbl ? 2 * vc : vc, total_v);
            uint64_t idle_since = 0;
            while ((nk < total_k || nv < total_v) && !ms->abort) {
                bool progressed = false;
                if (nk < total_k && mbar_test(&ms->kempty[nk % kring], (nk / kring - 1) & 1)) {
                    issue_k(nk++);
                    progressed = true;
                } else if (nv < total_v &&
                           mbar_test(&ms->vempty[v_slot(nv / vc, nv % vc)], (v_use(nv / vc) - 1) & 1)) {
                    issue_v(nv++);
                    progressed = true;
                }
                if (progressed) {
                    idle_since = 0;
                    continue;
                }
                __nanosleep(64);
                if (idle_since == 0) {
                    idle_since = global_timer_ns();
                } else if (global_timer_ns() - idle_since > kWaitNs) {
                    ms->abort = 1;
                    report(J.status, SLIMKV_DEVICE_TIMEOUT);
                }
            }
        } else if (warp == 2 && lane == 0) {
            // ---- S issuer: S(j) = K(j) . Q^T as K chunks land ----
            const uint32_t idesc_s = umma_idesc_bf16(128, kN, 0, 0);
            const uint32_t q0 = sbase + off_q, q1 = q0 + kMaxChunks * kQChunkBytes;
            bool ok = wait_or_abort(&ms->qfull, 0, ms, J.status);
            for (int j = 0; j < nt && ok; ++j) {
                const int sb = j & 1;
                const uint32_t s_tmem = s_tmem0 + uint32_t(sb * kN);
                if (j >= 2 && !(ok = wait_or_abort(&ms->sempty[sb], ((j - 2) >> 1) & 1, ms, J.status))) break;
                tc_fence_after();
                for (int c = 0; c < kc; ++c) {
                    const int n = j * kc + c, slot = n % kring;
                    if (!(ok = wait_or_abort(&ms->kfull[slot], (n / kring) & 1, ms, J.status))) break;
                    tc_fence_after();
                    const uint32_t ka = sbase + kOffK + slot * kChunkBytes;
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint64_t ad = umma_desc_sw128(ka + kk * 32, 16, 1024);
                        umma_bf16(s_tmem, ad, umma_desc_sw128(q0 + c * kQChunkBytes + kk * 32, 16, 1024), idesc_s,
                                  (c | kk) != 0);
                        if (!cols && !J.q_rows)
                            umma_bf16(s_tmem, ad, umma_desc_sw128(q1 + c * kQChunkBytes + kk * 32, 16, 1024), idesc_s,
                                      1u);
                    }
                    umma_commit(&ms->kempty[slot]);
                }
                if (!ok) break;
                umma_commit(&ms->sfull[sb]);
            }
            umma_commit(&ms->final_mma);
        } else if (warp == 1 && lane == 0) {
            // ---- P.V issuer: O^T += V(j)^T . P(j)^T once P(j) is written ----
            const uint32_t idesc_pair = umma_idesc_bf16(128, kN, 1, 1);
            const uint32_t idesc_one = umma_idesc_bf16(64, kN, 1, 1);
            const uint32_t p0 = sbase + off_p, p1 = p0 + kChunkBytes;
            bool ok = true;
            for (int j = 0; j < nt && ok; ++j) {
                if (!(ok = wait_or_abort(&ms->pfull, j & 1, ms, J.status))) break;
                tc_fence_after();
                for (int blk = 0; blk < vblocks; ++blk) {
                    const int c0 = 2 * blk, s0 = v_slot(j, c0);
                    const bool pair = c0 + 1 < vc;
                    for (int c = c0; c <= c0 + (pair ? 1 : 0); ++c)
                        if (!(ok = wait_or_abort(&ms->vfull[v_slot(j, c)], v_use(j) & 1, ms, J.status))) break;
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t va = sbase + s0 * kChunkBytes;
                    const uint32_t o_b = o_tmem + uint32_t(blk * kN);
                    const uint32_t idesc = pair ? idesc_pair : idesc_one;
#pragma unroll
                    for (int ks = 0; ks < kKeys / 16; ++ks) {
                        const uint64_t ad = umma_desc_sw128(va + ks * 2048, kChunkBytes, 1024);
                        umma_bf16(o_b, ad, umma_desc_sw128(p0 + ks * 2048, kChunkBytes, 1024), idesc,
                                  (j > 0 || ks > 0) ? 1u : 0u);
                        if (!cols) umma_bf16(o_b, ad, umma_desc_sw128(p1 + ks * 2048, kChunkBytes, 1024), idesc, 1u);
                    }
                    umma_commit(&ms->vempty[s0]);
                    if (pair) umma_commit(&ms->vempty[s0 + 1]);
                }
                if (!ok) break;
                umma_commit(&ms->odone);
            }
            umma_commit(&ms->final_mma);
        } else if (warp >= 3) {
            // ---- softmax and epilogue: thread <-> key (TMEM lane) ----
            const int quarter = warp & 3;
            const int t_local = 32 * quarter + lane;
            const uint32_t lane_addr = uint32_t(32 * quarter) << 16;
            const int st = tid - 96;                      // 0..127
            bool failed = false;
            for (int i = 0; i < nt; ++i) {
                const int sb = i & 1;
                const uint32_t s_tmem = s_tmem0 + uint32_t(sb * kN);
                const int key = (t0 + i) * kKeys + t_local;
                bool ok = wait_or_abort(&ms->sfull[sb], (i >> 1) & 1, ms, J.status);
                if (named_bar_or(1, 128, !ok)) { failed = true; break; }
                tc_fence_after();
                float v[2][32];
                tmem_ld32(s_tmem + lane_addr, v[0]);
                tmem_ld32(s_tmem + lane_addr + 32, v[1]);
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&ms->sempty[sb]);
                if (cols) {
#pragma unroll
                    for (int h = 0; h < 32; ++h) v[0][h] += v[1][h];       // hi + lo products
                }
                // scale and mask (an insertion step's raw query excludes the new Beacon)
#pragma unroll
                for (int l = 0; l < 2; ++l) {
                    const int limit = (J.causal && nq == 2 && l == 0) ? n_keys - 1 : n_keys;
#pragma unroll
                    for (int h = 0; h < 32; ++h) v[l][h] = key < limit ? v[l][h] * J.scale_log2 : -INFINITY;
                }
                // Column maxima only when some score exceeds its row's running
                // max by more than the lazy threshold (always on the first
                // tile): otherwise the max stays and every p <= 2^8.
                bool over = i == 0;
                if (!over) {
#pragma unroll
                    for (int l = 0; l < 2; ++l)
                        if (l < nq) {
#pragma unroll
                            for (int h = 0; h < 32; ++h) over |= v[l][h] > ms->m_run[32 * l + h] + kLazyLog2;
                        }
                }
                const bool rescan = named_bar_or(1, 128, over);
                bool need_fix = false;
                if (rescan) {
#pragma unroll
                    for (int l = 0; l < 2; ++l) {
                        if (l < nq) {
                            float tmp[32];
#pragma unroll
                            for (int h = 0; h < 32; ++h) tmp[h] = v[l][h];
                            ms->red[quarter][32 * l + lane] = warp_transpose_reduce<true>(tmp, lane);
                        }
                    }
                    named_bar(1, 128);
                    if (st < rows) {
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
                    need_fix = named_bar_or(1, 128, st < rows && i > 0 && ms->alpha[st] != 1.f);
                }
                // P(i) overwrites the buffer P.V(i-1) reads: wait for it.
                if (i > 0) {
                    ok = wait_or_abort(&ms->odone, (i - 1) & 1, ms, J.status);
                    if (named_bar_or(1, 128, !ok)) { failed = true; break; }
                    tc_fence_after();
                }
                // The sequence's partial last tile: V rows past the length hold
                // whatever the cache has there; P is zero for them, and zeroing
                // the rows too keeps a non-finite stale value from turning 0 * x
                // into NaN.  Each thread clears its own key row once the chunk
                // has landed (P.V(i) does not start before P(i) is released).
                if (i == nt - 1 && t0 + i == n_tiles - 1 && (n_keys & (kKeys - 1)) != 0) {
                    bool okc = true;
                    if (key >= n_keys) {
                        for (int c = 0; c < vc && okc; ++c) {
                            const int slot = v_slot(i, c);
                            okc = wait_or_abort(&ms->vfull[slot], v_use(i) & 1, ms, J.status);
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
                    // O^T column group k (32 columns) belongs to row k*32 + h, or
                    // to row h for the single-query hi | lo layout.
                    for (int blk = 0; blk < vblocks; ++blk)
                        for (int k = 0; k < 2; ++k) {
                            float o[32];
                            const uint32_t addr = o_tmem + lane_addr + uint32_t(blk * kN + 32 * k);
                            tmem_ld32(addr, o);
                            tmem_wait_ld();
                            const float* al = ms->alpha + (cols ? 0 : 32 * k);
#pragma unroll
                            for (int h = 0; h < 32; ++h) o[h] *= al[h];
                            tmem_st32(addr, o);
                        }
                    tmem_wait_st();
                }
                // probabilities -> P^T rows (hi and lo), row sums
                uint8_t* prow = smem + off_p + t_local * 128;
#pragma unroll
                for (int l = 0; l < 2; ++l) {
                    if (l < nq) {
                        float p[32];
#pragma unroll
                        for (int h = 0; h < 32; ++h) {
                            const float m = ms->m_run[32 * l + h];
                            p[h] = (v[l][h] == -INFINITY || m == -INFINITY) ? 0.f : exp2f(v[l][h] - m);
                        }
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            uint4 hi, lo;
                            split_hilo(p, u, hi, lo);
                            // nq = 1: units 0-3 hi, 4-7 lo of one buffer; nq = 2:
                            // unit 4l + u of the hi and of the lo buffer.
                            const int uh = cols ? u : 4 * l + u, ul = cols ? 4 + u : 4 * l + u;
                            uint8_t* lrow = cols ? prow : prow + kChunkBytes;
                            *reinterpret_cast<uint4*>(prow + ((uh ^ (t_local & 7)) << 4)) = hi;
                            *reinterpret_cast<uint4*>(lrow + ((ul ^ (t_local & 7)) << 4)) = lo;
                        }
                        ms->red[quarter][32 * l + lane] = warp_transpose_reduce<false>(p, lane);
                    }
                }
                fence_async_shared();
                tc_fence_before();
                named_bar(1, 128);
                if (st < rows)
                    ms->l_run[st] += ms->red[0][st] + ms->red[1][st] + ms->red[2][st] + ms->red[3][st];
                __syncwarp();
                if (lane == 0) mbar_arrive(&ms->pfull);
            }
            // ---- epilogue: normalised partial output and LSE per row ----
            if (!failed) {
                const bool ok = wait_or_abort(&ms->odone, (nt - 1) & 1, ms, J.status);
                failed = named_bar_or(1, 128, !ok);
            }
            if (!failed) {
                tc_fence_after();
                // per-row 1 / l (0 for a row without mass)
                if (st < 64) ms->alpha[st] = (st < rows && ms->l_run[st] > 0.f) ? 1.f / ms->l_run[st] : 0.f;
                named_bar(1, 128);
                // Stage O / l as [chunk][row][64] fp32 in the drained V ring.  An
                // M=128 block holds dim 32q + L of its chunk pair in lane L of
                // quarter q; the M=64 block holds dim 16q + L in lane L < 16.
                // Bulk tensor stores then write whole [32 rows x 64] boxes.
                float inv0[32], inv1[32];
#pragma unroll
                for (int h = 0; h < 32; ++h) {
                    inv0[h] = ms->alpha[h];
                    inv1[h] = ms->alpha[32 + h];
                }
                float* stage = reinterpret_cast<float*>(smem);
                for (int blk = 0; blk < vblocks; ++blk) {
                    const bool pair = 2 * blk + 1 < vc;
                    float o[2][32];
                    tmem_ld32(o_tmem + lane_addr + uint32_t(blk * kN), o[0]);
                    tmem_ld32(o_tmem + lane_addr + uint32_t(blk * kN + 32), o[1]);
                    tmem_wait_ld();
                    if (pair || lane < 16) {
                        const int dd = pair ? 32 * quarter + lane : 16 * quarter + lane;   // dim in the block
                        float* dst = stage + ((2 * blk + (dd >> 6)) * 64) * 64 + (dd & 63);
                        if (cols) {
#pragma unroll
                            for (int h = 0; h < 32; ++h) dst[h * 64] = (o[0][h] + o[1][h]) * inv0[h];
                        } else {
#pragma unroll
                            for (int h = 0; h < 32; ++h) {
                                dst[h * 64] = o[0][h] * inv0[h];
                                dst[(32 + h) * 64] = o[1][h] * inv1[h];
                            }
                        }
                    }
                }
                fence_async_shared();
                named_bar(1, 128);
                const int64_t base_row = (int64_t)z * J.rows_alloc;
                if (st == 0) {
                    for (int c = 0; c < vc; ++c)
                        for (int rb = 0; rb < nq; ++rb)
                            tma_store_3d(omap, stage + (c * 64 + rb * 32) * 64, c * 64, rb * 32, z);
                    bulk_commit();
                    bulk_wait_read_all();
                }
                if (st < rows) {
                    const float lsum = ms->l_run[st];
                    J.part_lse[base_row + st] = lsum > 0.f ? (ms->m_run[st] + log2f(lsum)) * 0.69314718055994530942f
                                                           : -INFINITY;
                }
                tc_fence_before();
            }
        }
    } else if (tid >= 96) {
        // Empty split: zero mass.
        const int st = tid - 96;
        const int64_t base_row = (int64_t)z * J.rows_alloc;
        if (st < rows) J.part_lse[base_row + st] = -INFINITY;
        for (int idx = st; idx < rows * J.out_width; idx += 128)
            J.part_o[(base_row + idx / J.out_width) * J.out_width + idx % J.out_width] = 0.f;
    }
    __syncthreads();
    if (nt > 0 && tid == 64) {
        // Both issuers committed final_mma after their last MMA: every MMA has
        // completed before TMEM is freed (bounded wait).
        mbar_wait(&ms->final_mma, 0, kWaitNs);
    }
    if (ms->abort && tid == 0) {
        // Drain: wait (bounded) for the last copy issued into every slot.
        for (int s = 0; s < kring; ++s) {
            mbar_wait(&ms->kfull[s], 0, 100000000ull);
            mbar_wait(&ms->kfull[s], 1, 100000000ull);
        }
        for (int s = 0; s < (dbl ? 2 * vc : vc); ++s) {
            mbar_wait(&ms->vfull[s], 0, 100000000ull);
            mbar_wait(&ms->vfull[s], 1, 100000000ull);
        }
        mbar_wait(&ms->qfull, 0, 100000000ull);
    }
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tbase, kTmemCols);
    }
}

namespace {

int make_side(const TcSide& S, int batch, int length, float scale, const int32_t* qlens, unsigned* status, TcJob& J,
              CUtensorMap& km, CUtensorMap& vm, CUtensorMap& qm, CUtensorMap& om) {
    if (S.dim_k > 320 || S.dim_v > 320 || S.width < 64 || S.width % 64 || S.rows_alloc % 32 ||
        (reinterpret_cast<uintptr_t>(S.part_o) & 15) || S.group > 32)
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
    if (S.q_rows) {
        // q_rot [B][L][H][dim] as (dim, 1, H, B * L), boxes of `group` rows.
        const uint64_t row = uint64_t(S.dim_k) * 2;
        if ((rc = encode_map_4d(&qm, S.q, S.dim_k, 1, S.heads, uint64_t(batch) * length, row, row, row * S.heads,
                                S.group)))
            return rc;
    } else {
        const uint64_t row = uint64_t(S.width) * 2;
        if ((rc = encode_map_4d(&qm, S.q, S.width, 1, 128, batch, row, row, row * 128, 64))) return rc;
    }
    if ((rc = encode_map_f32_3d(&om, S.part_o, S.width, S.rows_alloc, uint64_t(batch) * S.kv_heads * S.splits,
                                uint64_t(S.width) * 4, uint64_t(S.width) * 4 * S.rows_alloc, 64, 32)))
        return rc;
    J = TcJob{};
    J.kchunks = (S.dim_k + 63) / 64;
    J.vchunks = (S.dim_v + 63) / 64;
    J.kv_heads = S.kv_heads;
    J.group = S.group;
    J.causal = S.causal;
    J.q_rows = S.q_rows;
    J.seqlens = S.seqlens;
    J.qlens = qlens;
    J.length = length;
    J.scale_log2 = scale * 1.4426950408889634f;
    J.splits = S.splits;
    J.rows_alloc = S.rows_alloc;
    J.out_width = S.width;
    J.part_o = S.part_o;
    J.part_lse = S.part_lse;
    J.status = status;
    J.table = S.pages ? S.table : nullptr;
    J.table_stride = S.table_stride;
    J.slots = S.slots;
    J.v_col = S.pages ? S.dim_k : 0;
    J.box_rows = box_rows;
    J.work = S.work;
    J.tps = S.tiles_per_split > 0 ? S.tiles_per_split : 1;
    return SLIMKV_OK;
}

}  // namespace

int launch_decode_tc(const TcLaunch& L, cudaStream_t stream) {
    CUtensorMap lk, lv, lq, lo, rk, rv, rq, ro;
    TcJob jl, jr;
    int rc;
    if ((rc = make_side(L.lat, L.batch, L.length, L.scale, L.query_len, L.status, jl, lk, lv, lq, lo))) return rc;
    if (L.with_raw) {
        if ((rc = make_side(L.raw, L.batch, L.length, L.scale, L.query_len, L.status, jr, rk, rv, rq, ro))) return rc;
    } else {
        jr = jl;
        rk = lk; rv = lv; rq = lq; ro = lo;
    }
    static bool configured[64] = {};
    const int dev = device_info().device;
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        if (cudaFuncSetAttribute(decode_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemBytes)) !=
            cudaSuccess)
            return fail(SLIMKV_ERR_CUDA, "cudaFuncSetAttribute (decode tc) failed");
        configured[dev] = true;
    }
    const int n_lat = L.batch * L.lat.splits;
    const int n_raw = L.with_raw ? L.batch * L.raw.kv_heads * L.raw.splits : 0;
    decode_tc_kernel<<<n_lat + n_raw, kThreads7, kSmemBytes, stream>>>(lk, lv, lq, lo, rk, rv, rq, ro, jl, jr, n_lat);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(SLIMKV_ERR_CUDA, "decode tc launch failed: %s", cudaGetErrorString(e));
    return SLIMKV_OK;
}

}  // namespace slimkv
