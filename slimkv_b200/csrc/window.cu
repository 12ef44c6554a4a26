// Prefill window projection with Beacon roles (C ABI slimkv_window_project)
// and the prefill RoPE (slimkv_prefill_rope).
//
// Projection = a grouped tcgen05 GEMM.  A group multiplies the chunk rows of
// one role (raw or Beacon rows, gathered through an index list) by one
// nn.Linear weight [N][K] and stores bf16 results to up to three targets.
// One CTA computes a 256-row x bn-column tile (bn <= 256, a multiple of 16)
// as two M=128 MMAs that share the weight tile, accumulating in TMEM:
//   warps 0-7  gather A rows with cp.async (16-byte pieces written in the
//              128-byte swizzle the MMA descriptors expect); completion is
//              signalled per stage by cp.async.mbarrier.arrive.noinc, then
//              the same warps drain TMEM in the epilogue;
//   warp 8     loads the weight tile with TMA (no multicast);
//   warp 9     owns TMEM and issues the MMAs from one thread.
// Stages of 64 reduction columns (A 32 KB + B up to 32 KB), as many as fit
// 216 KB for the widest B tile of the launch (3 at bn 256, 4 at 160).  The epilogue
// adds the bias, rounds once to bf16 and stores each row to a dense row
// (chunk output or dense cache), a page row (Beacon / raw pages through a
// block table) and / or the sink of the root Beacon page.
//
// Launches with fewer tiles than SMs split the reduction: the `splits` CTAs
// of a tile each run a slice of the K chunks and store their fp32 partial
// tile into their own workspace slot; a second kernel (finalize_kernel)
// sums the slots in slice order - deterministic, unlike atomics - adds the
// bias, rounds and stores to the same targets.
//
// Every wait is bounded: a timeout sets SLIMKV_DEVICE_TIMEOUT, the CTA winds
// down (own copies drained, MMAs retired, TMEM freed) and returns.
#include <algorithm>
#include <climits>
#include <initializer_list>

#include "common.cuh"
#include "host_utils.h"

namespace slimkv {
namespace {

constexpr int kPjHalves = 2;
constexpr int kPjTileM = 128 * kPjHalves;
constexpr int kPjMaxStages = 6;
constexpr uint32_t kPjABytes = kPjTileM * 128;
constexpr uint32_t kPjStageBudget = 221184;        // bytes of stages (216 KB): 3 x 64 KB at bn 256, 4 x 52 KB at 160
constexpr int kPjGather = 256;                       // gather / epilogue threads
constexpr int kPjThreads = kPjGather + 64;           // + TMA warp + MMA warp
constexpr uint32_t kPjTmemCols = 512;                // two 128 x 256 fp32 accumulators
constexpr int kPjMaxGroups = 6;
constexpr int kPjMaxTargets = 3;
constexpr uint64_t kPjWaitNs = 2000000000ull;

enum : int { kTargetNone = 0, kTargetDense = 1, kTargetPaged = 2, kTargetSink = 3 };

// Where the rows of a group go.  Row j of sequence b has logical row
// (idx ? idx[j] : j) + (start ? start[b] : 0); rows j < first are skipped.
//   dense: base + b * sb + row * sr, row < limit
//   paged: base + table[b][row / slots] * page_stride + sink + (row % slots) * width + col
//   sink:  base + table[b][0] * page_stride + col, only for row == 0
struct PjTarget {
    int kind;
    uint16_t* base;
    int64_t sb, sr;
    const int32_t* idx;
    const int32_t* start;
    int first, col;
    int64_t limit;
    int64_t page_stride;
    int slots, sink, width;
    const int32_t* table;
    int64_t table_stride;
    int num_pages;
};

// A group: rows j < rows of every sequence b read A row
// (a_idx ? a_idx[j] : j) + (a_start ? a_start[b] : 0) (checked against
// a_limit) of a + b * a_sb, times weight map `gi` ([n][k]).  With a_count,
// rows j >= a_count[b] of sequence b are neither read nor written.
struct PjGroup {
    const uint16_t* a;
    int64_t a_sb, a_sr;
    const int32_t* a_idx;
    const int32_t* a_start;
    const int32_t* a_count;
    int a_limit, rows, k, n, bn, tiles_m, tiles_n, tile_begin;
    int splits;                // K slices per output tile (1: no workspace)
    float* acc;                // [splits][tiles_m * tiles_n][kPjTileM][bn] fp32 partial tiles
    int strip_begin;           // first finalize block of this group
    const uint16_t* bias;
    PjTarget t[kPjMaxTargets];
};

struct PjParams {
    int batch, groups;
    int stages;                // pipeline depth: stage = A tile + the widest B tile of the launch
    uint32_t stage_bytes;
    unsigned* status;
    PjGroup g[kPjMaxGroups];
};

struct PjMaps {
    CUtensorMap m[kPjMaxGroups];
};

struct PjShared {
    uint64_t afull[kPjMaxStages], bfull[kPjMaxStages], empty[kPjMaxStages], acc_full;
    uint32_t tmem_base;
    int abort;
};
constexpr uint32_t kPjSmemBytes = kPjStageBudget + sizeof(PjShared) + 1024;
static_assert(kPjSmemBytes <= 232448, "shared memory budget");

__device__ __forceinline__ void pj_cp_async16(uint32_t dst, const void* src, uint32_t bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}
// Arrive on `bar` once every cp.async this thread issued so far has landed
// (the barrier's expected count includes this arrival).
__device__ __forceinline__ void pj_cp_async_arrive(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void pj_cp_async_drain() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ bool pj_wait(uint64_t* bar, uint32_t parity, PjShared* ps, unsigned* status) {
    if (*reinterpret_cast<volatile int*>(&ps->abort)) return false;
    if (mbar_wait(bar, parity, kPjWaitNs)) return true;
    *reinterpret_cast<volatile int*>(&ps->abort) = 1;
    report(status, SLIMKV_DEVICE_TIMEOUT);
    return false;
}

// Destination of row j of sequence b (column 0 of the group's output), or
// nullptr when the target skips the row.
__device__ __forceinline__ uint16_t* target_row(const PjTarget& T, int b, int j, unsigned* status) {
    if (T.kind == kTargetNone || j < T.first) return nullptr;
    const int64_t row = int64_t(T.idx ? __ldg(T.idx + j) : j) + (T.start ? __ldg(T.start + b) : 0);
    if (T.kind == kTargetDense) {
        if (row < 0 || row >= T.limit) {
            report(status, SLIMKV_DEVICE_BAD_LENGTH);
            return nullptr;
        }
        return T.base + b * T.sb + row * T.sr;
    }
    if (T.kind == kTargetSink && row != 0) return nullptr;
    const int64_t page_index = row < 0 ? -1 : row / T.slots;
    const int page =
        (page_index < 0 || page_index >= T.table_stride) ? -1 : __ldg(T.table + b * T.table_stride + page_index);
    if (page < 0 || page >= T.num_pages) {
        report(status, SLIMKV_DEVICE_BAD_LENGTH);
        return nullptr;
    }
    if (T.kind == kTargetSink) return T.base + int64_t(page) * T.page_stride + T.col;
    return T.base + int64_t(page) * T.page_stride + T.sink + (row % T.slots) * T.width + T.col;
}

// Per-warp staging tile of 32 rows x 128 bytes, 16-byte chunks swizzled by
// row so that both the row-per-lane writes and the row-segment reads are
// free of bank conflicts.
__device__ __forceinline__ void stage_row(uint8_t* stg, int lane, const uint32_t* w) {
#pragma unroll
    for (int u = 0; u < 8; ++u)
        *reinterpret_cast<uint4*>(stg + lane * 128 + ((u ^ (lane & 7)) << 4)) =
            make_uint4(w[4 * u], w[4 * u + 1], w[4 * u + 2], w[4 * u + 3]);
}
__device__ __forceinline__ uint4 staged_piece(const uint8_t* stg, int row, int piece) {
    return *reinterpret_cast<const uint4*>(stg + row * 128 + ((piece ^ (row & 7)) << 4));
}
// Store `cnt` (<= 8) bf16 values of a 16-byte piece.
__device__ __forceinline__ void store_piece(uint16_t* dst, uint4 v, int cnt) {
    if (cnt == 8 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
        *reinterpret_cast<uint4*>(dst) = v;
        return;
    }
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    for (int e = 0; e < cnt; ++e) dst[e] = static_cast<uint16_t>(w[e >> 1] >> ((e & 1) * 16));
}

__device__ __forceinline__ bool pj_row_live(const PjGroup& G, int b, int j) {
    return !G.a_count || j < __ldg(G.a_count + b);
}

__global__ void __launch_bounds__(kPjThreads, 1)
project_kernel(const __grid_constant__ PjMaps maps, const __grid_constant__ PjParams P) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    PjShared* ps = reinterpret_cast<PjShared*>(smem + kPjStageBudget);
    const int S = P.stages;
    const uint32_t stage_bytes = P.stage_bytes;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    int gi = 0;
    for (int g = 1; g < P.groups; ++g)
        if (int(blockIdx.x) >= P.g[g].tile_begin) gi = g;
    const PjGroup& G = P.g[gi];
    const int local = blockIdx.x - G.tile_begin;
    const int tiles_mn = G.tiles_m * G.tiles_n;
    const int tile = local % tiles_mn, split = local / tiles_mn;
    const int m0 = (tile % G.tiles_m) * kPjTileM;
    const int n0 = (tile / G.tiles_m) * G.bn;
    const int total_rows = P.batch * G.rows;
    const int nk_all = (G.k + 63) / 64;
    const int k0 = split * nk_all / G.splits;              // this CTA's K chunks [k0, k0 + nk)
    const int nk = (split + 1) * nk_all / G.splits - k0;
    if (G.a_count) {
        // A tile whose rows are all past their sequences' counts has no work
        // (uniform over the CTA, before any barrier or TMEM allocation).
        bool live = false;
        const int b_first = m0 / G.rows, b_last = (min(m0 + kPjTileM, total_rows) - 1) / G.rows;
        for (int b = b_first; b <= b_last && !live; ++b)
            live = (b == b_first ? m0 % G.rows : 0) < __ldg(G.a_count + b);
        if (!live) return;
    }

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&ps->afull[s], kPjGather);
            mbar_init(&ps->bfull[s], 1);
            mbar_init(&ps->empty[s], 1);
        }
        mbar_init(&ps->acc_full, 1);
        ps->abort = 0;
        fence_barrier_init();
    }
    if (warp == 9) {
        tmem_alloc(&ps->tmem_base, kPjTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = ps->tmem_base;

    if (tid < kPjGather) {
        // ---- A gather: thread = (row slot, 16-byte piece); rows slot + 32 q.
        const int piece = tid & 7, rslot = tid >> 3;
        const uint16_t* rowp[8];
        uint32_t valid = 0;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const int grow = m0 + rslot + 32 * q;
            rowp[q] = G.a;
            if (grow < total_rows && pj_row_live(G, grow / G.rows, grow % G.rows)) {
                const int b = grow / G.rows, j = grow % G.rows;
                const int ar = (G.a_idx ? __ldg(G.a_idx + j) : j) + (G.a_start ? __ldg(G.a_start + b) : 0);
                if (ar >= 0 && ar < G.a_limit) {
                    rowp[q] = G.a + b * G.a_sb + int64_t(ar) * G.a_sr + piece * 8;
                    valid |= 1u << q;
                } else if (piece == 0) {
                    report(P.status, SLIMKV_DEVICE_BAD_LENGTH);
                }
            }
        }
        for (int i = 0; i < nk; ++i) {
            const int s = i % S, use = i / S, kc = k0 + i;
            if (i >= S && !pj_wait(&ps->empty[s], (use - 1) & 1, ps, P.status)) break;
            const uint32_t sa = smem_u32(smem + s * stage_bytes);
            const bool kin = kc * 64 + piece * 8 < G.k;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const int r = rslot + 32 * q;
                const bool v = kin && ((valid >> q) & 1);
                pj_cp_async16(sa + r * 128 + ((piece ^ (r & 7)) << 4), v ? rowp[q] + kc * 64 : G.a, v ? 16u : 0u);
            }
            pj_cp_async_arrive(&ps->afull[s]);
        }
        pj_cp_async_drain();

        // ---- epilogue: warp w reads TMEM lanes 32 (w % 4).. of accumulator w / 4.
        bool ok = mbar_wait(&ps->acc_full, 0, kPjWaitNs) && !*reinterpret_cast<volatile int*>(&ps->abort);
        ok = __all_sync(0xffffffffu, ok);
        tc_fence_after();
        const int h = warp >> 2, quarter = warp & 3;
        const uint32_t taddr = tbase + (uint32_t(quarter * 32) << 16) + uint32_t(h * 256);
        const int grow = m0 + h * 128 + quarter * 32 + lane;
        // Staging: each warp turns its 32 rows x 128 bytes (thread = row, as
        // TMEM delivers them) around through shared memory (stage 0 is free
        // once every MMA has retired) so lanes store whole row segments.
        uint8_t* stg = smem + warp * 4096;
        const int srow = lane >> 3;     // with piece = lane & 7: 4 rows x 8 pieces per store
        if (G.splits > 1) {
            // Store this slice's fp32 partial tile into its workspace slot.
            float* acc_tile = G.acc + (int64_t(split) * tiles_mn + tile) * kPjTileM * G.bn;
            const int row0 = h * 128 + quarter * 32;
            const int valid_rows = min(32, total_rows - (m0 + row0));
            if (ok) {
                for (int c0 = 0; c0 < G.bn; c0 += 32) {
                    float v[32];
                    tmem_ld32(taddr + c0, v);
                    tmem_wait_ld();
                    stage_row(stg, lane, reinterpret_cast<const uint32_t*>(v));
                    __syncwarp();
                    const int cnt = min(32, G.bn - c0);
#pragma unroll
                    for (int rr = 0; rr < 8; ++rr) {
                        const int r = rr * 4 + srow;
                        if (r < valid_rows && piece * 4 < cnt)
                            __stcg(reinterpret_cast<uint4*>(acc_tile + int64_t(row0 + r) * G.bn + c0 + piece * 4),
                                   staged_piece(stg, r, piece));
                    }
                    __syncwarp();
                }
            }
            ok = false;
        }
        if (ok) {
            uint16_t* dst[kPjMaxTargets] = {nullptr, nullptr, nullptr};
            if (grow < total_rows && pj_row_live(G, grow / G.rows, grow % G.rows)) {
                const int b = grow / G.rows, j = grow % G.rows;
                const int ar = (G.a_idx ? __ldg(G.a_idx + j) : j) + (G.a_start ? __ldg(G.a_start + b) : 0);
                if (ar >= 0 && ar < G.a_limit) {
#pragma unroll
                    for (int t = 0; t < kPjMaxTargets; ++t) dst[t] = target_row(G.t[t], b, j, P.status);
                }
            }
            for (int c0 = 0; c0 < G.bn; c0 += 64) {
                const int n = n0 + c0;
                const int cnt = min(64, min(G.bn - c0, G.n - n));
                if (cnt <= 0) break;
                uint32_t packed[32];
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    float v[32];
                    tmem_ld32(taddr + c0 + half * 32, v);
                    tmem_wait_ld();
                    if (G.bias) {
#pragma unroll
                        for (int e = 0; e < 32; ++e)
                            if (half * 32 + e < cnt) v[e] += __uint_as_float(uint32_t(__ldg(G.bias + n + half * 32 + e)) << 16);
                    }
#pragma unroll
                    for (int e = 0; e < 16; ++e) packed[half * 16 + e] = pack_bf16x2(v[2 * e], v[2 * e + 1]);
                }
                stage_row(stg, lane, packed);
                __syncwarp();
#pragma unroll
                for (int t = 0; t < kPjMaxTargets; ++t) {
#pragma unroll
                    for (int rr = 0; rr < 8; ++rr) {
                        const int r = rr * 4 + srow;
                        uint16_t* d = reinterpret_cast<uint16_t*>(
                            __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(dst[t]), r));
                        if (d && piece * 8 < cnt) store_piece(d + n + piece * 8, staged_piece(stg, r, piece),
                                                              min(8, cnt - piece * 8));
                    }
                }
                __syncwarp();
            }
        }
    } else if (warp == 8) {
        // ---- weight tiles by TMA: rows [n0, n0 + bn), 64 columns per stage.
        if (lane == 0) {
            const CUtensorMap* map = &maps.m[gi];
            tma_prefetch_desc(map);
            int i = 0;
            for (; i < nk; ++i) {
                const int s = i % S, use = i / S;
                if (i >= S && !pj_wait(&ps->empty[s], (use - 1) & 1, ps, P.status)) break;
                mbar_expect_tx(&ps->bfull[s], uint32_t(G.bn) * 128u);
                tma_load_4d(smem + s * stage_bytes + kPjABytes, map, &ps->bfull[s], (k0 + i) * 64, 0, n0, 0);
            }
            if (*reinterpret_cast<volatile int*>(&ps->abort)) {
                // Drain: the last load issued into each stage lands before exit.
                for (int c = max(0, i - S); c < i; ++c) mbar_wait(&ps->bfull[c % S], (c / S) & 1, 100000000ull);
            }
        }
    } else if (lane == 0) {
        // ---- MMA issue (warp 9): two M=128 accumulators share each B tile.
        const uint32_t idesc = umma_idesc_bf16(128, G.bn, 0, 0);
        for (int i = 0; i < nk; ++i) {
            const int s = i % S, use = i / S;
            if (!pj_wait(&ps->afull[s], use & 1, ps, P.status) || !pj_wait(&ps->bfull[s], use & 1, ps, P.status))
                break;
            // cp.async wrote A through the generic proxy; the MMA reads it
            // through the async proxy.
            fence_async_shared();
            tc_fence_after();
            const uint32_t a0 = smem_u32(smem + s * stage_bytes), b0 = a0 + kPjABytes;
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                const uint64_t bd = umma_desc_sw128(b0 + ks * 32, 16, 1024);
#pragma unroll
                for (int h = 0; h < kPjHalves; ++h)
                    umma_bf16(tbase + h * 256, umma_desc_sw128(a0 + h * 16384 + ks * 32, 16, 1024), bd, idesc,
                              (i | ks) != 0);
            }
            umma_commit(&ps->empty[s]);
        }
        umma_commit(&ps->acc_full);
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 9) {
        // Every MMA has retired before TMEM is freed (the epilogue waited for
        // acc_full; after an abort wait here, bounded).
        if (lane == 0 && *reinterpret_cast<volatile int*>(&ps->abort)) mbar_wait(&ps->acc_full, 0, 100000000ull);
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tbase, kPjTmemCols);
    }
}

// Split-K finish: one block per 8-row strip of a split tile; every thread
// sums 4 columns of one row over the slices in slice order, adds the bias,
// rounds to bf16 and stores to the group's targets.
constexpr int kFinRows = 8;

__global__ void __launch_bounds__(256) finalize_kernel(const __grid_constant__ PjParams P) {
    int gi = -1;
    for (int g = 0; g < P.groups; ++g)
        if (P.g[g].splits > 1 && int(blockIdx.x) >= P.g[g].strip_begin) gi = g;
    if (gi < 0) return;
    const PjGroup& G = P.g[gi];
    const int strips = kPjTileM / kFinRows;
    const int local = blockIdx.x - G.strip_begin;
    const int tiles_mn = G.tiles_m * G.tiles_n;
    const int tile = local / strips, strip = local % strips;
    const int m0 = (tile % G.tiles_m) * kPjTileM, n0 = (tile / G.tiles_m) * G.bn;
    const int total_rows = P.batch * G.rows;
    const int per_row = G.bn / 4;
    for (int item = threadIdx.x; item < kFinRows * per_row; item += blockDim.x) {
        const int r = strip * kFinRows + item / per_row, c = (item % per_row) * 4;
        const int grow = m0 + r, n = n0 + c;
        if (grow >= total_rows || n >= G.n) continue;
        const int b = grow / G.rows, j = grow % G.rows;
        if (!pj_row_live(G, b, j)) continue;
        const int ar = (G.a_idx ? __ldg(G.a_idx + j) : j) + (G.a_start ? __ldg(G.a_start + b) : 0);
        if (ar < 0 || ar >= G.a_limit) continue;
        const float* src = G.acc + (int64_t(tile) * kPjTileM + r) * G.bn + c;
        const int64_t slot = int64_t(tiles_mn) * kPjTileM * G.bn;
        // All slices in flight at once, then summed in slice order.
        float4 part[16];
#pragma unroll
        for (int sp = 0; sp < 16; ++sp)
            if (sp < G.splits) part[sp] = __ldcg(reinterpret_cast<const float4*>(src + sp * slot));
        float4 acc = part[0];
#pragma unroll
        for (int sp = 1; sp < 16; ++sp)
            if (sp < G.splits) acc.x += part[sp].x, acc.y += part[sp].y, acc.z += part[sp].z, acc.w += part[sp].w;
        const int cnt = min(4, G.n - n);
        float v[4] = {acc.x, acc.y, acc.z, acc.w};
        if (G.bias) {
#pragma unroll
            for (int e = 0; e < 4; ++e)
                if (e < cnt) v[e] += __uint_as_float(uint32_t(__ldg(G.bias + n + e)) << 16);
        }
        const uint32_t lo = pack_bf16x2(v[0], v[1]), hi = pack_bf16x2(v[2], v[3]);
#pragma unroll
        for (int t = 0; t < kPjMaxTargets; ++t) {
            uint16_t* dst = target_row(G.t[t], b, j, P.status);
            if (!dst) continue;
            dst += n;
            if (cnt == 4 && (reinterpret_cast<uintptr_t>(dst) & 7) == 0) {
                *reinterpret_cast<uint2*>(dst) = make_uint2(lo, hi);
            } else {
                const uint32_t w[2] = {lo, hi};
                for (int e = 0; e < cnt; ++e) dst[e] = static_cast<uint16_t>(w[e >> 1] >> ((e & 1) * 16));
            }
        }
    }
}

// ------------------------------------------------------------ prefill RoPE --
struct RopeArgs {
    const uint16_t* q;
    const uint16_t* k;
    int64_t qs[3], ks[3], qos[3], kos[3];
    uint16_t* q_out;
    uint16_t* k_out;
    const float* cos;
    const float* sin;
    int rope_positions;
    const int64_t* pos;
    int64_t pos_stride;
    const int64_t* roles;
    int role_count, sink, batch, heads, kv_heads, queries, keys, dim;
    unsigned* status;
};

__device__ __forceinline__ float bfv(uint16_t x) { return __uint_as_float(uint32_t(x) << 16); }
__device__ __forceinline__ uint16_t bfr(float x) {
    __nv_bfloat16 h = __float2bfloat16_rn(x);
    return *reinterpret_cast<uint16_t*>(&h);
}

// One thread rotates V consecutive pairs (d, d + D/2) of one row.
template <int V>
__global__ void prefill_rope_kernel(RopeArgs A) {
    const int half = A.dim / 2, groups = half / V;
    const int64_t q_items = int64_t(A.batch) * A.heads * A.queries * groups;
    const int64_t k_items = int64_t(A.batch) * A.kv_heads * A.keys * groups;
    for (int64_t it = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; it < q_items + k_items;
         it += int64_t(gridDim.x) * blockDim.x) {
        const bool is_q = it < q_items;
        int64_t r = is_q ? it : it - q_items;
        const int d0 = int(r % groups) * V;
        r /= groups;
        const int seq = is_q ? A.queries : A.keys, nh = is_q ? A.heads : A.kv_heads;
        const int s = int(r % seq);
        r /= seq;
        const int h = int(r % nh);
        const int b = int(r / nh);
        const uint16_t* x = is_q ? A.q + b * A.qs[0] + h * A.qs[1] + s * A.qs[2]
                                 : A.k + b * A.ks[0] + h * A.ks[1] + s * A.ks[2];
        uint16_t* o = is_q ? A.q_out + b * A.qos[0] + h * A.qos[1] + s * A.qos[2]
                           : A.k_out + b * A.kos[0] + h * A.kos[1] + s * A.kos[2];
        bool beacon = false;
        int64_t p;
        if (is_q) {
            p = A.pos[b * A.pos_stride + A.keys - A.queries + s];
        } else {
            p = A.pos[b * A.pos_stride + s];
            const int prefix = A.keys - A.role_count;
            const int64_t role = s >= prefix ? A.roles[s - prefix] : 0;
            beacon = (s < prefix && s >= A.sink) || role == 1 || role == 2;
        }
        uint16_t lo[V], hi[V];
        if (V == 8) {
            *reinterpret_cast<uint4*>(lo) = *reinterpret_cast<const uint4*>(x + d0);
            *reinterpret_cast<uint4*>(hi) = *reinterpret_cast<const uint4*>(x + d0 + half);
        } else {
#pragma unroll
            for (int e = 0; e < V; ++e) lo[e] = x[d0 + e], hi[e] = x[d0 + half + e];
        }
        uint16_t out_lo[V], out_hi[V];
        if (!beacon && (p < 0 || p >= A.rope_positions)) {
            report(A.status, SLIMKV_DEVICE_BAD_LENGTH);
            beacon = true;
        }
        if (beacon) {
#pragma unroll
            for (int e = 0; e < V; ++e) out_lo[e] = lo[e], out_hi[e] = hi[e];
        } else {
            const float* cr = A.cos + p * A.dim;
            const float* sr = A.sin + p * A.dim;
#pragma unroll
            for (int e = 0; e < V; ++e) {
                const float xl = bfv(lo[e]), xh = bfv(hi[e]);
                const float cl = bf16_round(__ldg(cr + d0 + e)), ch = bf16_round(__ldg(cr + d0 + half + e));
                const float sl = bf16_round(__ldg(sr + d0 + e)), sh = bf16_round(__ldg(sr + d0 + half + e));
                out_lo[e] = bfr(bf16_round(xl * cl) + bf16_round(-xh * sl));
                out_hi[e] = bfr(bf16_round(xh * ch) + bf16_round(xl * sh));
            }
        }
        if (V == 8) {
            *reinterpret_cast<uint4*>(o + d0) = *reinterpret_cast<const uint4*>(out_lo);
            *reinterpret_cast<uint4*>(o + d0 + half) = *reinterpret_cast<const uint4*>(out_hi);
        } else {
#pragma unroll
            for (int e = 0; e < V; ++e) o[d0 + e] = out_lo[e], o[d0 + half + e] = out_hi[e];
        }
    }
}

// -------------------------------------------------------------------- host --
int launched(const char* what) {
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? SLIMKV_OK : fail(SLIMKV_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(e));
}

// Tile width for n output columns: fewest tiles of at most 256, then the
// narrowest multiple of 16.
int tile_width(int n) {
    const int tiles = (n + 255) / 256;
    return ((n + tiles - 1) / tiles + 15) / 16 * 16;
}

PjTarget dense_target(void* base, int64_t sb, int64_t sr, int64_t limit, const int32_t* idx, const int32_t* start,
                      int first = 0) {
    PjTarget t{};
    if (!base) return t;
    t.kind = kTargetDense;
    t.limit = limit;
    t.base = static_cast<uint16_t*>(base);
    t.sb = sb;
    t.sr = sr;
    t.idx = idx;
    t.start = start;
    t.first = first;
    return t;
}

PjTarget beacon_target(const slimkv_beacon_pages* p, const int32_t* start, int col) {
    PjTarget t{};
    t.kind = kTargetPaged;
    t.base = static_cast<uint16_t*>(p->pages);
    t.start = start;
    t.col = col;
    t.page_stride = p->page_stride;
    t.slots = p->slots;
    t.sink = p->sink_elements;
    t.width = p->rank_k + p->rank_v;
    t.table = p->table;
    t.table_stride = p->table_stride;
    t.num_pages = p->num_pages;
    return t;
}

PjTarget raw_page_target(const slimkv_raw_pages* p, const int32_t* start, int first, int col) {
    PjTarget t{};
    const int kvd = p->kv_heads * p->head_dim;
    t.kind = kTargetPaged;
    t.base = static_cast<uint16_t*>(p->pages);
    t.start = start;
    t.first = first;
    t.col = col;
    t.page_stride = int64_t(p->block_size) * 2 * kvd;
    t.slots = p->block_size;
    t.sink = 0;
    t.width = 2 * kvd;
    t.table = p->table;
    t.table_stride = p->table_stride;
    t.num_pages = p->num_blocks;
    return t;
}

struct Launch {
    PjParams p{};
    PjMaps maps{};
    const void* weight[kPjMaxGroups] = {};
    int tiles = 0;
};

// Append a group computing rows x weight[n][k]^T; no-op when it has no target.
int add_group(Launch& L, const void* a, int64_t a_sb, int64_t a_sr, const int32_t* a_idx, const int32_t* a_start,
              int a_limit, int rows, const void* weight, int k, int n, const void* bias,
              std::initializer_list<PjTarget> targets, int batch, const int32_t* a_count = nullptr) {
    bool any = false;
    for (const PjTarget& t : targets) any |= t.kind != kTargetNone;
    if (!any || rows == 0 || batch == 0) return SLIMKV_OK;
    if (!weight) return fail(SLIMKV_ERR_INVALID_ARGUMENT, "window projection: a requested output has no weight");
    if (!aligned16(weight) || k % 8 || k <= 0 || n <= 0)
        return fail(SLIMKV_ERR_ALIGNMENT, "window projection: weights must be [out][in] with in %% 8 == 0, 16-byte aligned");
    if (L.p.groups == kPjMaxGroups) return fail(SLIMKV_ERR_INVALID_ARGUMENT, "window projection: too many groups");
    PjGroup& G = L.p.g[L.p.groups];
    G = PjGroup{};
    G.a = static_cast<const uint16_t*>(a);
    G.a_sb = a_sb;
    G.a_sr = a_sr;
    G.a_idx = a_idx;
    G.a_start = a_start;
    G.a_count = a_count;
    G.a_limit = a_limit;
    G.rows = rows;
    G.k = k;
    G.n = n;
    G.bn = tile_width(n);
    G.tiles_m = int((int64_t(batch) * rows + kPjTileM - 1) / kPjTileM);
    G.tiles_n = (n + G.bn - 1) / G.bn;
    G.splits = 1;
    G.bias = static_cast<const uint16_t*>(bias);
    int i = 0;
    for (const PjTarget& t : targets) G.t[i++] = t;
    L.weight[L.p.groups++] = weight;
    return SLIMKV_OK;
}

// K split of each group: a launch with fewer output tiles than SMs splits
// every reduction into power-of-two slices (at least 4 chunks of 64 each) so
// the launch fills the machine.  Returns the workspace bytes the slices'
// fp32 partial tiles need; with `ws` (at least that many bytes, 256-byte
// aligned) the splits are applied.
size_t plan_splits(Launch& L, int sms, uint8_t* ws) {
    int tiles_mn = 0;
    for (int g = 0; g < L.p.groups; ++g) tiles_mn += L.p.g[g].tiles_m * L.p.g[g].tiles_n;
    int S = 1;
    while (tiles_mn > 0 && tiles_mn * S * 2 <= sms && S < 16) S *= 2;
    size_t bytes = 0;
    for (int g = 0; g < L.p.groups; ++g) {
        PjGroup& G = L.p.g[g];
        int sg = S;
        while (sg > 1 && (G.k + 63) / 64 / sg < 4) sg /= 2;
        if (sg == 1) continue;
        if (ws) {
            G.splits = sg;
            G.acc = reinterpret_cast<float*>(ws + bytes);
        }
        bytes += (size_t(sg) * G.tiles_m * G.tiles_n * kPjTileM * G.bn * 4 + 255) & ~size_t(255);
    }
    return bytes;
}

int run(Launch& L, int batch, void* ws, size_t ws_bytes, cudaStream_t stream) {
    if (L.p.groups == 0) return SLIMKV_OK;
    const int sms = device_info().sm_count;
    const size_t need = plan_splits(L, sms, nullptr);
    if (need && ws && ws_bytes >= need && aligned16(ws)) plan_splits(L, sms, static_cast<uint8_t*>(ws));
    L.tiles = 0;
    for (int g = 0; g < L.p.groups; ++g) {
        PjGroup& G = L.p.g[g];
        G.tile_begin = L.tiles;
        L.tiles += G.tiles_m * G.tiles_n * G.splits;
        const uint64_t row_bytes = uint64_t(G.k) * 2;
        if (int rc = encode_map_4d(&L.maps.m[g], L.weight[g], G.k, 1, G.n, 1, row_bytes, row_bytes,
                                   row_bytes * G.n, G.bn))
            return rc;
    }
    static bool attr_set = false;
    if (!attr_set) {
        if (cudaFuncSetAttribute(project_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPjSmemBytes) !=
            cudaSuccess)
            return fail(SLIMKV_ERR_CUDA, "window projection: cannot reserve %u bytes of shared memory", kPjSmemBytes);
        attr_set = true;
    }
    int max_bn = 16;
    for (int g = 0; g < L.p.groups; ++g) max_bn = std::max(max_bn, L.p.g[g].bn);
    L.p.stage_bytes = (kPjABytes + uint32_t(max_bn) * 128 + 1023) & ~1023u;
    L.p.stages = std::min<int>(kPjMaxStages, kPjStageBudget / L.p.stage_bytes);
    L.p.batch = batch;
    L.p.status = status_word();
    int strips = 0;
    for (int g = 0; g < L.p.groups; ++g) {
        PjGroup& G = L.p.g[g];
        G.strip_begin = strips;
        if (G.splits > 1) strips += G.tiles_m * G.tiles_n * (kPjTileM / kFinRows);
    }
    project_kernel<<<L.tiles, kPjThreads, kPjSmemBytes, stream>>>(L.maps, L.p);
    if (int rc = launched("window projection")) return rc;
    if (strips == 0) return SLIMKV_OK;
    finalize_kernel<<<strips, 256, 0, stream>>>(L.p);
    return launched("window projection finish");
}

bool rows_ok(const void* p, int64_t sb, int64_t sr) { return aligned16(p) && sb % 8 == 0 && sr % 8 == 0; }

}  // namespace
}  // namespace slimkv

using namespace slimkv;

namespace slimkv {
namespace {

// Validate the arguments and describe both launches (no device work).
int build(const slimkv_window_project_args* a, Launch& L1, Launch& L2) {
    if (!a) return fail(SLIMKV_ERR_INVALID_ARGUMENT, "null arguments");
    if (a->batch < 0 || a->rows < 0 || a->raw_count < 0 || a->beacon_count < 0 || a->raw_count > a->rows ||
        a->beacon_count > a->rows)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "window projection: invalid batch, rows or role counts");
    if (a->batch == 0 || a->rows == 0) return SLIMKV_OK;
    if (a->heads <= 0 || a->kv_heads <= 0 || a->head_dim <= 0 || a->rank_k <= 0 || a->rank_v <= 0 || a->hidden <= 0)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "window projection: dimensions must be positive");
    if (a->hidden % 8 || !a->hidden_states || !rows_ok(a->hidden_states, a->hidden_stride_batch, a->hidden_stride_row))
        return fail(SLIMKV_ERR_ALIGNMENT,
                    "window projection: hidden rows must be 16-byte aligned with hidden %% 8 == 0");
    if ((a->raw_count && !a->raw_rows) || (a->beacon_count && !a->beacon_rows))
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "window projection: missing role index list");
    const int qd = a->heads * a->head_dim, kvd = a->kv_heads * a->head_dim;
    const bool want_lat_cache = a->beacon_pages != nullptr;
    const bool want_raw_cache = a->raw_pages || a->raw_key_cache || a->raw_value_cache;
    if (want_lat_cache && !a->beacon_start)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "window projection: Beacon pages need beacon_start");
    if ((want_raw_cache || a->write_sink) && !a->raw_start)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "window projection: raw cache writes need raw_start");
    if (a->raw_pages && (a->raw_key_cache || a->raw_value_cache))
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "window projection: give raw pages or a dense raw cache, not both");
    if (a->beacon_count && ((a->key && !a->key_latent) || (a->value && !a->value_latent)))
        return fail(SLIMKV_ERR_INVALID_ARGUMENT,
                    "window projection: Beacon key/value rows are up-projected from key_latent/value_latent");
    if (a->beacon_pages) {
        const slimkv_beacon_pages* p = a->beacon_pages;
        if (!p->pages || !p->table || p->slots <= 0 || p->table_stride <= 0 || p->num_pages <= 0 ||
            p->rank_k != a->rank_k || p->rank_v != a->rank_v || p->sink_elements < 0 ||
            p->page_stride < int64_t(p->sink_elements) + int64_t(p->slots) * (p->rank_k + p->rank_v))
            return fail(SLIMKV_ERR_INVALID_ARGUMENT, "window projection: Beacon page geometry does not match the ranks");
    }
    if (a->write_sink && (!a->beacon_pages || a->beacon_pages->sink_elements != 2 * kvd))
        return fail(SLIMKV_ERR_INVALID_ARGUMENT,
                    "Sink cache must retain the original raw K/V dimensions.");
    if (a->raw_pages) {
        const slimkv_raw_pages* p = a->raw_pages;
        if (!p->pages || !p->table || p->block_size <= 0 || p->table_stride <= 0 || p->num_blocks <= 0 ||
            p->kv_heads != a->kv_heads || p->head_dim != a->head_dim)
            return fail(SLIMKV_ERR_INVALID_ARGUMENT, "Raw cache dimensions differ from the engine allocation.");
    }
    if ((a->raw_key_cache || a->raw_value_cache) && a->raw_cache_rows <= 0)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "window projection: a dense raw cache needs raw_cache_rows");
    if ((a->key_latent || a->value_latent) && a->latent_start && a->latent_rows <= 0)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "window projection: latent rows at latent_start need latent_rows");
    const int64_t lat_rows = a->latent_rows > 0 ? a->latent_rows : a->beacon_count;
    if (a->w_k_up && a->rank_k % 8) return fail(SLIMKV_ERR_UNSUPPORTED_SHAPE, "window projection: rank_k %% 8 != 0");
    if (a->w_v_up && a->rank_v % 8) return fail(SLIMKV_ERR_UNSUPPORTED_SHAPE, "window projection: rank_v %% 8 != 0");

    const int B = a->batch;
    const int32_t* rr = a->raw_rows;
    const int32_t* br = a->beacon_rows;
    const PjTarget none{};
    int rc;
    // Raw rows: q, k, v (+ raw cache, sink).
    rc = add_group(L1, a->hidden_states, a->hidden_stride_batch, a->hidden_stride_row, rr, nullptr, a->rows,
                   a->raw_count, a->w_q, a->hidden, qd, a->b_q,
                   {dense_target(a->query, a->query_stride_batch, a->query_stride_row, a->rows, rr, nullptr)}, B);
    if (rc) return rc;
    // Beacon rows: beacon_q.
    if ((rc = add_group(L1, a->hidden_states, a->hidden_stride_batch, a->hidden_stride_row, br, nullptr, a->rows,
                        a->beacon_count, a->w_bq, a->hidden, qd, a->b_bq,
                        {dense_target(a->query, a->query_stride_batch, a->query_stride_row, a->rows, br, nullptr)}, B)))
        return rc;
    for (int kind = 0; kind < 2; ++kind) {
        void* chunk_out = kind ? a->value : a->key;
        const int64_t csb = kind ? a->value_stride_batch : a->key_stride_batch;
        const int64_t csr = kind ? a->value_stride_row : a->key_stride_row;
        void* cache = kind ? a->raw_value_cache : a->raw_key_cache;
        PjTarget cache_t = a->raw_pages ? raw_page_target(a->raw_pages, a->raw_start, a->raw_first, kind * kvd)
                                        : dense_target(cache, a->raw_cache_stride_batch, a->raw_cache_stride_row,
                                                       a->raw_cache_rows, nullptr, a->raw_start, a->raw_first);
        PjTarget sink_t = none;
        if (a->write_sink) {
            sink_t = beacon_target(a->beacon_pages, a->raw_start, kind * kvd);
            sink_t.kind = kTargetSink;
        }
        if ((rc = add_group(L1, a->hidden_states, a->hidden_stride_batch, a->hidden_stride_row, rr, nullptr, a->rows,
                            a->raw_count, kind ? a->w_v : a->w_k, a->hidden, kvd, kind ? a->b_v : a->b_k,
                            {dense_target(chunk_out, csb, csr, a->rows, rr, nullptr), cache_t, sink_t}, B)))
            return rc;
    }
    // Beacon rows: latents (+ Beacon pages).
    for (int kind = 0; kind < 2; ++kind) {
        const int rank = kind ? a->rank_v : a->rank_k;
        void* lat = kind ? a->value_latent : a->key_latent;
        const int64_t lsb = kind ? a->value_latent_stride_batch : a->key_latent_stride_batch;
        const int64_t lsr = kind ? a->value_latent_stride_row : a->key_latent_stride_row;
        PjTarget page_t = want_lat_cache ? beacon_target(a->beacon_pages, a->beacon_start, kind * a->rank_k) : none;
        if ((rc = add_group(L1, a->hidden_states, a->hidden_stride_batch, a->hidden_stride_row, br, nullptr, a->rows,
                            a->beacon_count, kind ? a->w_v_down : a->w_k_down, a->hidden, rank, nullptr,
                            {dense_target(lat, lsb, lsr, lat_rows, nullptr, a->latent_start), page_t}, B)))
            return rc;
    }
    // Beacon key/value rows (second launch): up-projection of the bf16
    // latents the first launch wrote.
    for (int kind = 0; kind < 2; ++kind) {
        void* out = kind ? a->value : a->key;
        if (!out || !a->beacon_count) continue;
        const void* lat = kind ? a->value_latent : a->key_latent;
        const int64_t lsb = kind ? a->value_latent_stride_batch : a->key_latent_stride_batch;
        const int64_t lsr = kind ? a->value_latent_stride_row : a->key_latent_stride_row;
        if (!rows_ok(lat, lsb, lsr))
            return fail(SLIMKV_ERR_ALIGNMENT, "window projection: latent rows must be 16-byte aligned");
        if ((rc = add_group(L2, lat, lsb, lsr, nullptr, a->latent_start, int(std::min<int64_t>(lat_rows, INT_MAX)),
                            a->beacon_count,
                            kind ? a->w_v_up : a->w_k_up, kind ? a->rank_v : a->rank_k, kvd,
                            kind ? a->b_v_up : a->b_k_up,
                            {dense_target(out, kind ? a->value_stride_batch : a->key_stride_batch,
                                          kind ? a->value_stride_row : a->key_stride_row, a->rows, br, nullptr)},
                            B)))
            return rc;
    }
    return SLIMKV_OK;
}

}  // namespace
}  // namespace slimkv

extern "C" size_t slimkv_window_project_workspace_size(const slimkv_window_project_args* a) {
    Launch L1, L2;
    if (build(a, L1, L2) != SLIMKV_OK) return 0;
    const int sms = device_info().sm_count;
    return std::max(plan_splits(L1, sms, nullptr), plan_splits(L2, sms, nullptr));
}

extern "C" int slimkv_window_project(const slimkv_window_project_args* a, void* stream) {
    Launch L1, L2;
    if (int rc = build(a, L1, L2)) return rc;
    if (a->batch == 0 || a->rows == 0) return SLIMKV_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (int rc = run(L1, a->batch, a->workspace, a->workspace_bytes, st)) return rc;
    return run(L2, a->batch, a->workspace, a->workspace_bytes, st);
}

namespace slimkv {
namespace {

// The two up-projection groups of a Beacon K/V reconstruction.
int build_reconstruct(const slimkv_reconstruct_args* a, Launch& L) {
    if (!a) return fail(SLIMKV_ERR_INVALID_ARGUMENT, "null arguments");
    if (a->batch < 0 || a->rows < 0 || a->kv_heads <= 0 || a->head_dim <= 0 || a->rank_k <= 0 || a->rank_v <= 0)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "reconstruct: invalid shape");
    if (a->batch == 0 || a->rows == 0) return SLIMKV_OK;
    if (a->rows > a->lat_capacity || a->out_rows <= 0)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "reconstruct: rows exceed the latent capacity or out_rows is empty");
    if (!a->lat_k || !a->lat_v || !a->w_k_up || !a->w_v_up || !a->key || !a->value)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "reconstruct: null tensor pointer");
    if (a->rank_k % 8 || a->rank_v % 8 || !rows_ok(a->lat_k, a->lat_stride_batch, a->lat_stride_row) ||
        !rows_ok(a->lat_v, a->lat_stride_batch, a->lat_stride_row) ||
        !rows_ok(a->key, a->out_stride_batch, a->out_stride_row) ||
        !rows_ok(a->value, a->out_stride_batch, a->out_stride_row))
        return fail(SLIMKV_ERR_ALIGNMENT, "reconstruct: rows must be 16-byte aligned with strides and ranks %% 8 == 0");
    const int kvd = a->kv_heads * a->head_dim;
    if (a->out_stride_row < kvd || a->lat_stride_row < std::max(a->rank_k, a->rank_v))
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "reconstruct: row stride smaller than a row");
    int rc;
    if ((rc = add_group(L, a->lat_k, a->lat_stride_batch, a->lat_stride_row, nullptr, nullptr, a->lat_capacity,
                        a->rows, a->w_k_up, a->rank_k, kvd, a->b_k_up,
                        {dense_target(a->key, a->out_stride_batch, a->out_stride_row, a->out_rows, nullptr,
                                      a->out_start)},
                        a->batch, a->row_count)))
        return rc;
    return add_group(L, a->lat_v, a->lat_stride_batch, a->lat_stride_row, nullptr, nullptr, a->lat_capacity, a->rows,
                     a->w_v_up, a->rank_v, kvd, a->b_v_up,
                     {dense_target(a->value, a->out_stride_batch, a->out_stride_row, a->out_rows, nullptr,
                                   a->out_start)},
                     a->batch, a->row_count);
}

}  // namespace
}  // namespace slimkv

extern "C" size_t slimkv_reconstruct_kv_workspace_size(const slimkv_reconstruct_args* a) {
    Launch L;
    if (build_reconstruct(a, L) != SLIMKV_OK) return 0;
    return plan_splits(L, device_info().sm_count, nullptr);
}

extern "C" int slimkv_reconstruct_kv(const slimkv_reconstruct_args* a, void* stream) {
    Launch L;
    if (int rc = build_reconstruct(a, L)) return rc;
    if (a->batch == 0 || a->rows == 0) return SLIMKV_OK;
    return run(L, a->batch, a->workspace, a->workspace_bytes, static_cast<cudaStream_t>(stream));
}

extern "C" int slimkv_prefill_rope(const void* q, const int64_t q_stride[3], const void* k, const int64_t k_stride[3],
                                   const float* cos, const float* sin, int rope_positions, const int64_t* positions,
                                   int64_t positions_stride, const int64_t* roles, int role_count, int sink, int batch,
                                   int heads, int kv_heads, int queries, int keys, int head_dim, void* q_out,
                                   const int64_t q_out_stride[3], void* k_out, const int64_t k_out_stride[3],
                                   void* stream) {
    if (!q || !k || !cos || !sin || !positions || !q_out || !k_out || !q_stride || !k_stride || !q_out_stride ||
        !k_out_stride)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "prefill rope: null argument");
    if (batch < 0 || heads <= 0 || kv_heads <= 0 || queries < 0 || keys < 0 || queries > keys || head_dim <= 0 ||
        head_dim % 2 || role_count < 0 || role_count > keys || (role_count && !roles) || sink < 0 ||
        rope_positions <= 0)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "prefill rope: invalid shape");
    if (batch == 0 || keys == 0) return SLIMKV_OK;
    RopeArgs A{};
    A.q = static_cast<const uint16_t*>(q);
    A.k = static_cast<const uint16_t*>(k);
    for (int i = 0; i < 3; ++i) {
        A.qs[i] = q_stride[i];
        A.ks[i] = k_stride[i];
        A.qos[i] = q_out_stride[i];
        A.kos[i] = k_out_stride[i];
    }
    A.q_out = static_cast<uint16_t*>(q_out);
    A.k_out = static_cast<uint16_t*>(k_out);
    A.cos = cos;
    A.sin = sin;
    A.rope_positions = rope_positions;
    A.pos = positions;
    A.pos_stride = positions_stride;
    A.roles = roles;
    A.role_count = role_count;
    A.sink = sink;
    A.batch = batch;
    A.heads = heads;
    A.kv_heads = kv_heads;
    A.queries = queries;
    A.keys = keys;
    A.dim = head_dim;
    A.status = status_word();
    bool vec = (head_dim / 2) % 8 == 0;
    for (int i = 0; i < 3; ++i)
        vec = vec && A.qs[i] % 8 == 0 && A.ks[i] % 8 == 0 && A.qos[i] % 8 == 0 && A.kos[i] % 8 == 0;
    vec = vec && aligned16(q) && aligned16(k) && aligned16(q_out) && aligned16(k_out);
    const int V = vec ? 8 : 1;
    const int64_t items =
        (int64_t(batch) * heads * queries + int64_t(batch) * kv_heads * keys) * (head_dim / 2 / V);
    const int sms = std::max(device_info().sm_count, 1);
    const int grid = int(std::max<int64_t>(1, std::min<int64_t>((items + 255) / 256, int64_t(sms) * 16)));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (vec)
        prefill_rope_kernel<8><<<grid, 256, 0, st>>>(A);
    else
        prefill_rope_kernel<1><<<grid, 256, 0, st>>>(A);
    return launched("prefill rope");
}
