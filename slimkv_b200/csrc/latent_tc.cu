// Latent-branch split-KV decode attention on the 5th-generation tensor cores.
//
// One CTA owns (sequence b, split): a contiguous range of 128-key tiles of
// the sequence's latent cache, against all query rows of the step (32 heads x
// 1 or 2 queries).  Swap-AB so the keys fill the MMA's M = 128:
//
//   S^T [128 keys x Np]  = K_tile [128 x Rk] . Q^T           (K-major A and B)
//   O^T [Rv x Np]       += V_tile^T [Rv x 128] . P^T          (MN-major A and B)
//
// Q and P are carried as bf16 hi/lo pairs (q = hi + lo to ~16 mantissa bits)
// so the bf16 tensor cores keep fp32-level accuracy without converting the
// bf16 K/V tiles: Np = 64 per query (32 heads hi | 32 heads lo).  Scores and
// the output accumulate in tensor memory (TMEM); softmax runs with one key per
// thread reading its TMEM lane, column maxima/sums via warp transpose-reduce,
// and a lazy rescale (the running max only moves when a column max exceeds it
// by 2^8), so O^T rarely needs a TMEM read-modify-write.
//
// Warp roles (7 warps): 0 = K TMA producer (ring of 3 [128 x 64] chunks),
// 1 = Q + V TMA producer (ring of 2 [128 x 128] blocks), 2 = TMEM allocator and
// single-thread MMA issuer, 3-6 = softmax / epilogue (TMEM lane quarters
// 3, 0, 1, 2).  TMA loads use the 128-byte swizzle and no cluster multicast.
// Every wait is bounded: on expiry the CTA reports SLIMKV_DEVICE_TIMEOUT,
// drains its copies and MMAs (bounded), frees TMEM and returns.
#include <algorithm>

#include "common.cuh"
#include "host_utils.h"
#include "latent_tc.h"

namespace slimkv {

namespace {

constexpr int kKeys = 128;
constexpr int kThreads7 = 224;
constexpr int kKSlots = 3;
constexpr int kVSlots = 2;
constexpr uint32_t kChunkBytes = 128 * 128;          // one [128 rows x 64 bf16] swizzled box
constexpr int kMaxKChunks = 5;                      // rank_k <= 320
constexpr float kLazyLog2 = 8.f;
constexpr uint32_t kTmemCols = 512;

constexpr uint32_t kOffK = 0;
constexpr uint32_t kOffV = kOffK + kKSlots * kChunkBytes;
constexpr uint32_t kOffQ = kOffV + kVSlots * 2 * kChunkBytes;
constexpr uint32_t kOffP = kOffQ + kMaxKChunks * kChunkBytes;
constexpr uint32_t kOffMisc = kOffP + 2 * kChunkBytes;

struct Misc {
    uint64_t kfull[kKSlots], kempty[kKSlots], vfull[kVSlots], vempty[kVSlots];
    uint64_t qfull, sfull, sempty, pfull, odone, final_mma;
    uint32_t tmem_base;
    int abort;
    float m_run[64], l_run[64], alpha[64];
    float red[4][64];
    int fix;
};
constexpr uint32_t kSmemBytes = kOffMisc + sizeof(Misc) + 1024;
static_assert(kSmemBytes <= 232448, "shared memory budget");

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, Misc* ms, unsigned* status) {
    if (ms->abort) return false;
    if (mbar_wait(bar, parity)) return true;
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

// After this, lane `l` holds the reduction over the warp's 32 lanes of the
// value v[c] with c = l (a transpose-reduce: 31 shuffles for 32 columns).
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

}  // namespace

__global__ void __launch_bounds__(kThreads7, 1)
latent_tc_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                 const __grid_constant__ CUtensorMap qmap, TcJob J) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Misc* ms = reinterpret_cast<Misc*>(smem + kOffMisc);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int b = blockIdx.x / J.splits, split = blockIdx.x % J.splits;
    const int n_keys = J.seqlens[b];
    const int nq = J.qlens ? J.qlens[b] : J.length;          // 1 or 2 queries
    const int np = 64 * nq;                                   // MMA N (hi/lo per query)
    const int rows = 32 * nq;
    const int n_tiles = (max(n_keys, 0) + kKeys - 1) / kKeys;
    const int t0 = split * J.tiles_per_split;
    const int t1 = split == J.splits - 1 ? n_tiles : min(n_tiles, t0 + J.tiles_per_split);
    const int nt = max(0, t1 - t0);

    if (tid == 0) {
        for (int s = 0; s < kKSlots; ++s) { mbar_init(&ms->kfull[s], 1); mbar_init(&ms->kempty[s], 1); }
        for (int s = 0; s < kVSlots; ++s) { mbar_init(&ms->vfull[s], 1); mbar_init(&ms->vempty[s], 1); }
        mbar_init(&ms->qfull, 1);
        mbar_init(&ms->sfull, 1);
        mbar_init(&ms->sempty, 4);
        mbar_init(&ms->pfull, 4);
        mbar_init(&ms->odone, 1);
        mbar_init(&ms->final_mma, 1);
        ms->abort = 0;
        fence_barrier_init();
        tma_prefetch_desc(&kmap);
        tma_prefetch_desc(&vmap);
        tma_prefetch_desc(&qmap);
    }
    if (warp == 2) {
        tmem_alloc(&ms->tmem_base, kTmemCols);
        tmem_relinquish();
    }
    if (tid >= 96) {
        const int r = tid - 96;
        if (r < 64) { ms->m_run[r] = -INFINITY; ms->l_run[r] = 0.f; }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = ms->tmem_base;
    const uint32_t o_tmem = tbase;                            // vblocks x np columns
    const uint32_t s_tmem = tbase + uint32_t(J.vblocks * np); // np columns
    const uint32_t sbase = smem_u32(smem);

    if (nt > 0) {
        if (warp == 0 && lane == 0) {
            // ---- K producer ----
            int kc = 0;
            for (int i = 0; i < nt && !ms->abort; ++i) {
                for (int c = 0; c < J.kchunks; ++c, ++kc) {
                    const int slot = kc % kKSlots, use = kc / kKSlots;
                    if (use > 0 && !wait_or_abort(&ms->kempty[slot], (use - 1) & 1, ms, J.status)) break;
                    mbar_expect_tx(&ms->kfull[slot], kChunkBytes);
                    tma_load_4d(smem + kOffK + slot * kChunkBytes, &kmap, &ms->kfull[slot], c * 64, 0,
                                (t0 + i) * kKeys, b);
                }
            }
        } else if (warp == 1 && lane == 0) {
            // ---- Q + V producer ----
            mbar_expect_tx(&ms->qfull, J.kchunks * kChunkBytes);
            for (int c = 0; c < J.kchunks; ++c)
                tma_load_4d(smem + kOffQ + c * kChunkBytes, &qmap, &ms->qfull, c * 64, 0, 0, b);
            int vc = 0;
            for (int i = 0; i < nt && !ms->abort; ++i) {
                for (int mb = 0; mb < J.vblocks; ++mb, ++vc) {
                    const int slot = vc % kVSlots, use = vc / kVSlots;
                    if (use > 0 && !wait_or_abort(&ms->vempty[slot], (use - 1) & 1, ms, J.status)) break;
                    uint8_t* dst = smem + kOffV + slot * 2 * kChunkBytes;
                    mbar_expect_tx(&ms->vfull[slot], 2 * kChunkBytes);
                    tma_load_4d(dst, &vmap, &ms->vfull[slot], mb * 128, 0, (t0 + i) * kKeys, b);
                    tma_load_4d(dst + kChunkBytes, &vmap, &ms->vfull[slot], mb * 128 + 64, 0, (t0 + i) * kKeys, b);
                }
            }
        } else if (warp == 2 && lane == 0) {
            // ---- MMA issuer ----
            const uint32_t idesc_s = umma_idesc_bf16(128, np, 0, 0);
            const uint32_t idesc_pv = umma_idesc_bf16(128, np, 1, 1);
            int kc = 0, vc = 0;
            if (wait_or_abort(&ms->qfull, 0, ms, J.status)) {
                for (int i = 0; i < nt; ++i) {
                    if (i > 0 && !wait_or_abort(&ms->sempty, (i - 1) & 1, ms, J.status)) break;
                    tc_fence_after();
                    bool ok = true;
                    for (int c = 0; c < J.kchunks && ok; ++c, ++kc) {
                        const int slot = kc % kKSlots;
                        if (!wait_or_abort(&ms->kfull[slot], (kc / kKSlots) & 1, ms, J.status)) { ok = false; break; }
                        tc_fence_after();
                        const uint32_t ka = sbase + kOffK + slot * kChunkBytes;
                        const uint32_t qa = sbase + kOffQ + c * kChunkBytes;
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            umma_bf16(s_tmem, umma_desc_sw128(ka + kk * 32, 16, 1024),
                                      umma_desc_sw128(qa + kk * 32, 16, 1024), idesc_s, (c | kk) != 0);
                        umma_commit(&ms->kempty[slot]);
                    }
                    if (!ok) break;
                    umma_commit(&ms->sfull);
                    if (!wait_or_abort(&ms->pfull, i & 1, ms, J.status)) break;
                    tc_fence_after();
                    for (int mb = 0; mb < J.vblocks && ok; ++mb, ++vc) {
                        const int slot = vc % kVSlots;
                        if (!wait_or_abort(&ms->vfull[slot], (vc / kVSlots) & 1, ms, J.status)) { ok = false; break; }
                        tc_fence_after();
                        const uint32_t va = sbase + kOffV + slot * 2 * kChunkBytes;
                        const uint32_t pa = sbase + kOffP;
#pragma unroll
                        for (int ks = 0; ks < kKeys / 16; ++ks)
                            umma_bf16(o_tmem + uint32_t(mb * np), umma_desc_sw128(va + ks * 2048, kChunkBytes, 1024),
                                      umma_desc_sw128(pa + ks * 2048, kChunkBytes, 1024), idesc_pv,
                                      (i > 0 || ks > 0) ? 1u : 0u);
                        umma_commit(&ms->vempty[slot]);
                    }
                    if (!ok) break;
                    umma_commit(&ms->odone);
                }
            }
            // All issued MMAs complete before TMEM is read back or freed.
            umma_commit(&ms->final_mma);
            mbar_wait(&ms->final_mma, 0);
        } else if (warp >= 3) {
            // ---- softmax and epilogue: thread <-> key (TMEM lane) ----
            const int quarter = warp & 3;
            const int t_local = 32 * quarter + lane;
            const uint32_t lane_addr = uint32_t(32 * quarter) << 16;
            const int st = tid - 96;                      // 0..127
            bool failed = false;
            for (int i = 0; i < nt; ++i) {
                const int key = (t0 + i) * kKeys + t_local;
                bool ok = wait_or_abort(&ms->sfull, i & 1, ms, J.status);
                if (named_bar_or(1, 128, !ok)) { failed = true; break; }
                tc_fence_after();
                float v[2][32];
#pragma unroll
                for (int l = 0; l < 2; ++l) {
                    if (l < nq) {
                        float lo[32];
                        tmem_ld32(s_tmem + lane_addr + 64 * l, v[l]);
                        tmem_ld32(s_tmem + lane_addr + 64 * l + 32, lo);
                        tmem_wait_ld();
#pragma unroll
                        for (int h = 0; h < 32; ++h) v[l][h] += lo[h];
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&ms->sempty);
                // scale, mask (a Beacon-insertion step's raw query excludes the new Beacon)
#pragma unroll
                for (int l = 0; l < 2; ++l) {
                    const int limit = (nq == 2 && l == 0) ? n_keys - 1 : n_keys;
#pragma unroll
                    for (int h = 0; h < 32; ++h) v[l][h] = key < limit ? v[l][h] * J.scale_log2 : -INFINITY;
                }
                // column maxima of this tile
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
                    const float tm = fmaxf(fmaxf(ms->red[0][st], ms->red[1][st]), fmaxf(ms->red[2][st], ms->red[3][st]));
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
                const bool need_fix = named_bar_or(1, 128, st < rows && ms->alpha[st] != 1.f && i > 0);
                // P(i) reuses the buffer read by PV(i-1); PV(i-1) precedes S(i)
                // on the tensor pipe, so it has finished, but wait for it anyway.
                if (i > 0) {
                    ok = wait_or_abort(&ms->odone, (i - 1) & 1, ms, J.status);
                    if (named_bar_or(1, 128, !ok)) { failed = true; break; }
                    tc_fence_after();
                }
                if (need_fix) {
                    // rescale the O^T columns whose running max moved
                    for (int mb = 0; mb < J.vblocks; ++mb)
                        for (int l = 0; l < nq; ++l)
                            for (int half = 0; half < 2; ++half) {
                                float o[32];
                                const uint32_t addr = o_tmem + lane_addr + uint32_t(mb * np + 64 * l + 32 * half);
                                tmem_ld32(addr, o);
                                tmem_wait_ld();
#pragma unroll
                                for (int h = 0; h < 32; ++h) o[h] *= ms->alpha[32 * l + h];
                                tmem_st32(addr, o);
                            }
                    tmem_wait_st();
                }
                // probabilities -> P^T (hi | lo per query), row sums
#pragma unroll
                for (int l = 0; l < 2; ++l) {
                    if (l < nq) {
                        float p[32];
#pragma unroll
                        for (int h = 0; h < 32; ++h) {
                            const float m = ms->m_run[32 * l + h];
                            p[h] = (v[l][h] == -INFINITY || m == -INFINITY) ? 0.f : exp2f(v[l][h] - m);
                        }
                        uint8_t* prow = smem + kOffP + l * kChunkBytes + t_local * 128;
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            uint32_t hi[4], lo[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const float a0 = p[8 * u + 2 * e], a1 = p[8 * u + 2 * e + 1];
                                const float h0 = bf16_round(a0), h1 = bf16_round(a1);
                                hi[e] = pack_bf16x2(h0, h1);
                                lo[e] = pack_bf16x2(a0 - h0, a1 - h1);
                            }
                            *reinterpret_cast<uint4*>(prow + (((u) ^ (t_local & 7)) << 4)) =
                                make_uint4(hi[0], hi[1], hi[2], hi[3]);
                            *reinterpret_cast<uint4*>(prow + (((u + 4) ^ (t_local & 7)) << 4)) =
                                make_uint4(lo[0], lo[1], lo[2], lo[3]);
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
                named_bar(1, 128);
                const int64_t base_row = ((int64_t)b * J.splits + split) * J.rows_alloc;
                for (int mb = 0; mb < J.vblocks; ++mb) {
                    const int d = mb * 128 + t_local;
                    for (int l = 0; l < nq; ++l) {
                        float hi[32], lo[32];
                        tmem_ld32(o_tmem + lane_addr + uint32_t(mb * np + 64 * l), hi);
                        tmem_ld32(o_tmem + lane_addr + uint32_t(mb * np + 64 * l + 32), lo);
                        tmem_wait_ld();
                        if (d < J.out_width) {
#pragma unroll
                            for (int h = 0; h < 32; ++h) {
                                const float lsum = ms->l_run[32 * l + h];
                                J.part_o[(base_row + 32 * l + h) * J.out_width + d] =
                                    lsum > 0.f ? (hi[h] + lo[h]) / lsum : 0.f;
                            }
                        }
                    }
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
        const int64_t base_row = ((int64_t)b * J.splits + split) * J.rows_alloc;
        if (st < rows) J.part_lse[base_row + st] = -INFINITY;
        for (int idx = st; idx < rows * J.out_width; idx += 128)
            J.part_o[(base_row + idx / J.out_width) * J.out_width + idx % J.out_width] = 0.f;
    }
    __syncthreads();
    if (ms->abort && tid == 0) {
        // Drain: wait (bounded) for the last copy issued into every slot.
        for (int s = 0; s < kKSlots; ++s) { mbar_wait(&ms->kfull[s], 0, 100000000ull); mbar_wait(&ms->kfull[s], 1, 100000000ull); }
        for (int s = 0; s < kVSlots; ++s) { mbar_wait(&ms->vfull[s], 0, 100000000ull); mbar_wait(&ms->vfull[s], 1, 100000000ull); }
        mbar_wait(&ms->qfull, 0, 100000000ull);
    }
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tbase, kTmemCols);
    }
}

int launch_latent_tc(const TcLaunch& L, cudaStream_t stream) {
    if (L.rank_k > 320 || L.rank_v > 320 || L.width < 64 || L.width % 64)
        return fail(SLIMKV_ERR_UNSUPPORTED_SHAPE, "latent tensor-core path needs ranks <= 320");
    CUtensorMap km, vm, qm;
    int rc;
    if ((rc = encode_map_4d(&km, L.lat_k, L.rank_k, 1, L.lat_capacity, L.batch, L.lat_stride_row * 2,
                            L.lat_stride_row * 2, L.lat_stride_batch * 2, kKeys)))
        return rc;
    if ((rc = encode_map_4d(&vm, L.lat_v, L.rank_v, 1, L.lat_capacity, L.batch, L.lat_stride_row * 2,
                            L.lat_stride_row * 2, L.lat_stride_batch * 2, kKeys)))
        return rc;
    if ((rc = encode_map_4d(&qm, L.q_hilo, L.width, 1, 128, L.batch, uint64_t(L.width) * 2, uint64_t(L.width) * 2,
                            uint64_t(L.width) * 2 * 128, 128)))
        return rc;
    TcJob J{};
    J.rank_k = L.rank_k;
    J.rank_v = L.rank_v;
    J.kchunks = (L.rank_k + 63) / 64;
    J.vblocks = (L.rank_v + 127) / 128;
    J.seqlens = L.latent_len;
    J.qlens = L.query_len;
    J.length = L.length;
    J.scale_log2 = L.scale * 1.4426950408889634f;
    J.splits = L.splits;
    J.tiles_per_split = L.tiles_per_split;
    J.rows_alloc = L.rows_alloc;
    J.out_width = L.width;
    J.part_o = L.part_o;
    J.part_lse = L.part_lse;
    J.status = L.status;
    static bool configured[64] = {};
    const int dev = device_info().device;
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        if (cudaFuncSetAttribute(latent_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemBytes)) !=
            cudaSuccess)
            return fail(SLIMKV_ERR_CUDA, "cudaFuncSetAttribute (latent tc) failed");
        configured[dev] = true;
    }
    latent_tc_kernel<<<L.batch * L.splits, kThreads7, kSmemBytes, stream>>>(km, vm, qm, J);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(SLIMKV_ERR_CUDA, "latent tc launch failed: %s", cudaGetErrorString(e));
    return SLIMKV_OK;
}

}  // namespace slimkv
