// Prefill attention on the 5th-generation tensor cores (C ABI
// slimkv_prefill_attention): one flash-attention forward used for both parts
// of a prefill chunk's attention when the history is kept as Beacon latents.
//
// The reference joins the chunk's attention by materialising every history
// latent into full keys and values each window (ReconstructionCache.
// materialize, slimkv/llama3/memory.py:26-48, called from the prefill
// forward at modeling_llama.py:1650-1681) and running one causal flash
// attention over [sinks, history, current].  Beacon keys carry no rotary, so
// the history part can instead run in latent space: each query row absorbed
// into the latent key space (q . U_k[g], all heads of the chunk sharing the
// one latent "head"), attended against the latents themselves, and the
// latent output up-projected once per row (U_v[g]); the sinks and the
// chunk's own rows are attended in full dimension with the causal mask; the
// two parts are merged by their LSEs.  Both are this kernel:
//   history: rows (token, head) over all H heads, dim = the latent ranks,
//            no mask but the sequence's latent count;
//   current: rows (token, head of the KV group) per KV head, dim 128, key k
//            visible to token t when k <= causal_offset + t (the bottom-right
//            alignment of a causal attention whose queries are the last
//            tokens of the key sequence).
//
// One CTA per (one or two 128-row Q tiles, KV head, sequence): Q staged once
// by TMA; keys in 128-key tiles through K and V rings of 16 KB chunks ([128
// keys x 64 columns], 128-byte swizzle, no multicast), each key / value tile
// used by every Q tile of the CTA (two when both dims are <= 128: the chunk
// part, with one softmax warpgroup per Q tile);
//   S [128 rows x 128 keys] = Q . K^T   (tcgen05, M=128, N=128, fp32 in TMEM)
//   O [128 rows x dim_v]   += P . V     (M=128, N=64 per V chunk)
// with P in bf16 (as flash attention keeps it).  Softmax: one thread per row
// (its TMEM lane), all 128 scores in registers, row max and sum without any
// cross-thread reduction, lazy rescale of O (only when the row max grows by
// more than 2^8).  Warp roles: 0 = Q and K producer, 3 = V producer, 1 = MMA
// issuer (lane 0; the warp zeroes the V rows past a sequence's keys in its
// last tile, whose contents the cache does not define), 2 = TMEM owner,
// 4-7 (and 8-11) = softmax and epilogue of Q tile 0 (1).  Every wait is
// bounded.
#include <algorithm>

#include "common.cuh"
#include "host_utils.h"

namespace slimkv {
namespace {

constexpr int kRows = 128;
constexpr int kKeys = 128;
constexpr uint32_t kChunk = 128 * 128;           // [128 x 64] bf16
constexpr uint32_t kTileArea = 224 * 1024;
constexpr int kMaxChunks = 5;                    // dims <= 320
constexpr int kMaxRing = 8;
constexpr float kLazyLog2 = 8.f;

struct Bars {
    uint64_t kfull[kMaxRing], kempty[kMaxRing], vfull[kMaxRing], vempty[kMaxRing];
    // [Q tile][buffer]
    uint64_t qfull, sfull[2][2], sempty[2][2], pfull[2][2], odone[2][2], final_mma;
    uint32_t tmem_base;
    int abort;
};
constexpr uint32_t kSmemBytes = 1024 + kTileArea + uint32_t(sizeof(Bars));
static_assert(kSmemBytes <= 232448, "shared memory budget");

struct Job {
    int kc, vc;                 // 64-column chunks of a key / value row
    int dim_v;
    int kring, vring, sbufs;    // ring slots, S buffers per Q tile in TMEM
    int vpair;                  // V chunk pairs in adjacent ring slots: one N=128 P.V MMA per pair
    int rpt;                    // query rows per token (per CTA's KV head)
    int tokens;                 // query tokens per sequence
    int kv_heads;
    const int32_t* kv_len;
    int kv_capacity;
    int causal, causal_offset;
    float scale_log2;
    __nv_bfloat16* out;
    int64_t o_sb, o_st, o_sh;
    float* lse;
    int64_t l_sb, l_st;
    unsigned int* status;
    uint64_t wait_ns;
};

__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, Bars* bs, const Job& J) {
    if (bs->abort) return false;
    if (mbar_wait(bar, parity, J.wait_ns)) return true;
    bs->abort = 1;
    report(J.status, SLIMKV_DEVICE_TIMEOUT);
    return false;
}

// NQ Q tiles of 128 rows per CTA (2: dims <= 128, every key / value tile
// feeds twice the MMA work; one softmax warpgroup per Q tile).
template <int NQ>
__global__ void __launch_bounds__(128 + 128 * NQ, 1)
prefill_attention_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                         const __grid_constant__ CUtensorMap vmap, const __grid_constant__ Job J) {
    constexpr int kThreadsNQ = 128 + 128 * NQ;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Bars* bs = reinterpret_cast<Bars*>(smem + kTileArea);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // Heaviest (last, for a causal job) row tiles first.
    const int pair = int(gridDim.x) - 1 - int(blockIdx.x);
    const int g = blockIdx.y, b = blockIdx.z;
    // A Q tile is tpt whole tokens: rows r < tpt * rpt (token t_first + r / rpt,
    // head r % rpt of the KV group); the rows past them are idle.  Q tile q of
    // the CTA starts at token (pair * NQ + q) * tpt.
    const int tpt = kRows / J.rpt, tile_rows = tpt * J.rpt;
    const int t_first = pair * NQ * tpt, t_last = t_first + NQ * tpt - 1;
    const int n_keys = min(max(J.kv_len[b], 0), J.kv_capacity);
    const int vis_keys = J.causal ? min(n_keys, max(J.causal_offset + t_last + 1, 0)) : n_keys;
    const int tiles = (vis_keys + kKeys - 1) / kKeys;
    // Layout: Q (NQ x kc chunks) | P (NQ x 2 chunks) | K ring | V ring.
    const uint32_t off_p = uint32_t(NQ * J.kc) * kChunk;
    const uint32_t off_k = off_p + uint32_t(NQ * 2) * kChunk;
    const uint32_t off_v = off_k + uint32_t(J.kring) * kChunk;
    // TMEM: O of Q tile q at q * o_cols, then its S buffers.
    const uint32_t o_cols = 64u * uint32_t(J.vc);
    auto s_col = [&](int q, int sb) -> uint32_t { return NQ * o_cols + uint32_t((q * J.sbufs + sb) * kKeys); };

    if (tile_rows < kRows) {
        // The idle rows of Q read as zero (the TMA box fills the rest).
        const int per = (kRows - tile_rows) * 8;
        for (int i = tid; i < NQ * J.kc * per; i += kThreadsNQ) {
            const int c = i / per, w = i - c * per;
            reinterpret_cast<uint4*>(smem + c * kChunk + tile_rows * 128)[w] = make_uint4(0, 0, 0, 0);
        }
        fence_async_shared();
    }
    if (tid == 0) {
        for (int s = 0; s < kMaxRing; ++s) {
            mbar_init(&bs->kfull[s], 1); mbar_init(&bs->kempty[s], 1);
            mbar_init(&bs->vfull[s], 1); mbar_init(&bs->vempty[s], 1);
        }
        mbar_init(&bs->qfull, 1);
        for (int q = 0; q < 2; ++q)
            for (int s = 0; s < 2; ++s) {
                mbar_init(&bs->sfull[q][s], 1);
                mbar_init(&bs->sempty[q][s], 4);
                mbar_init(&bs->pfull[q][s], 4);
                mbar_init(&bs->odone[q][s], 1);
            }
        mbar_init(&bs->final_mma, 1);
        bs->abort = 0;
        fence_barrier_init();
    }
    if (warp == 2) {
        tmem_alloc(&bs->tmem_base, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = bs->tmem_base;
    const uint32_t sbase = smem_u32(smem);

    if (warp == 0 && lane == 0 && tiles > 0) {
        // ---- Q, then the K chunks of every tile ----
        mbar_expect_tx(&bs->qfull, uint32_t(NQ * J.kc) * uint32_t(tile_rows) * 128u);
        for (int q = 0; q < NQ; ++q)
            for (int c = 0; c < J.kc; ++c)
                tma_load_4d(smem + (q * J.kc + c) * kChunk, &qmap, &bs->qfull, c * 64, g * J.rpt, t_first + q * tpt,
                            b);
        bool ok = true;
        for (int n = 0; n < tiles * J.kc && ok; ++n) {
            const int j = n / J.kc, c = n - j * J.kc, slot = n % J.kring;
            if (n >= J.kring && !(ok = wait_bar(&bs->kempty[slot], ((n / J.kring) - 1) & 1, bs, J))) break;
            mbar_expect_tx(&bs->kfull[slot], kChunk);
            tma_load_4d(smem + off_k + slot * kChunk, &kmap, &bs->kfull[slot], c * 64, g, j * kKeys, b);
        }
    } else if (warp == 3 && lane == 0 && tiles > 0) {
        // ---- the V chunks of every tile ----
        bool ok = true;
        for (int n = 0; n < tiles * J.vc && ok; ++n) {
            const int j = n / J.vc, c = n - j * J.vc, slot = n % J.vring;
            if (n >= J.vring && !(ok = wait_bar(&bs->vempty[slot], ((n / J.vring) - 1) & 1, bs, J))) break;
            mbar_expect_tx(&bs->vfull[slot], kChunk);
            tma_load_4d(smem + off_v + slot * kChunk, &vmap, &bs->vfull[slot], c * 64, g, j * kKeys, b);
        }
    } else if (warp == 1) {
        // ---- MMA issuer: S(j) of every Q tile, then P.V(j - 1) of each Q
        // tile as its probabilities land (overlapping the softmax of tile j) ----
        const bool leader = lane == 0;
        const uint32_t idesc_s = umma_idesc_bf16(128, kKeys, 0, 0);
        const uint32_t idesc_o = umma_idesc_bf16(128, 64, 0, 1);
        const uint32_t idesc_pair = umma_idesc_bf16(128, 128, 0, 1);
        bool ok = tiles == 0 || __all_sync(0xffffffffu, wait_bar(&bs->qfull, 0, bs, J));
        auto issue_pv = [&](int jj) {
            const int valid = n_keys - jj * kKeys;          // < 128 only in the sequence's last tile
            for (int q = 0; q < NQ && ok; ++q) {
                ok = __all_sync(0xffffffffu, wait_bar(&bs->pfull[q][jj & 1], (jj >> 1) & 1, bs, J));
                if (!ok) return;
                tc_fence_after();
                const uint32_t pbase = sbase + off_p + uint32_t(q * 2) * kChunk;
                // V chunks one at a time (N=64), or as adjacent pairs in the ring
                // (N=128 over two 64-column atoms kChunk apart).
                const int step = J.vpair ? 2 : 1;
                for (int c = 0; c < J.vc && ok; c += step) {
                    const int n = jj * J.vc + c, slot = n % J.vring;
                    if (q == 0) {
                        for (int cc = 0; cc < step && ok; ++cc) {
                            const int sl = (n + cc) % J.vring;
                            ok = __all_sync(0xffffffffu, wait_bar(&bs->vfull[sl], ((n + cc) / J.vring) & 1, bs, J));
                            if (ok && valid < kKeys) {
                                uint4* rows = reinterpret_cast<uint4*>(smem + off_v + sl * kChunk);
                                for (int i = max(valid, 0) * 8 + lane; i < kKeys * 8; i += 32)
                                    rows[i] = make_uint4(0, 0, 0, 0);
                                fence_async_shared();
                                __syncwarp();
                            }
                        }
                        if (!ok) break;
                        tc_fence_after();
                    }
                    if (leader) {
                        const uint32_t va = sbase + off_v + slot * kChunk;
#pragma unroll
                        for (int ks = 0; ks < kKeys / 16; ++ks)
                            umma_bf16(tbase + q * o_cols + 64u * c,
                                      umma_desc_sw128(pbase + (ks >> 2) * kChunk + (ks & 3) * 32, 16, 1024),
                                      umma_desc_sw128(va + ks * 2048, kChunk, 1024), step == 2 ? idesc_pair : idesc_o,
                                      (jj > 0 || ks > 0) ? 1u : 0u);
                        if (q == NQ - 1)
                            for (int cc = 0; cc < step; ++cc) umma_commit(&bs->vempty[(n + cc) % J.vring]);
                    }
                    __syncwarp();
                }
                if (ok && leader) umma_commit(&bs->odone[q][jj & 1]);
                __syncwarp();
            }
        };
        for (int j = 0; j < tiles && ok; ++j) {
            const int sb = j % J.sbufs;
            if (j >= J.sbufs)
                for (int q = 0; q < NQ && ok; ++q)
                    ok = __all_sync(0xffffffffu, wait_bar(&bs->sempty[q][sb], ((j / J.sbufs) - 1) & 1, bs, J));
            if (!ok) break;
            tc_fence_after();
            for (int c = 0; c < J.kc && ok; ++c) {
                const int n = j * J.kc + c, slot = n % J.kring;
                ok = __all_sync(0xffffffffu, wait_bar(&bs->kfull[slot], (n / J.kring) & 1, bs, J));
                if (!ok) break;
                tc_fence_after();
                if (leader) {
                    const uint32_t ka = sbase + off_k + slot * kChunk;
#pragma unroll
                    for (int q = 0; q < NQ; ++q)
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            umma_bf16(tbase + s_col(q, sb),
                                      umma_desc_sw128(sbase + (q * J.kc + c) * kChunk + kk * 32, 16, 1024),
                                      umma_desc_sw128(ka + kk * 32, 16, 1024), idesc_s, (c | kk) != 0);
                    umma_commit(&bs->kempty[slot]);
                }
                __syncwarp();
            }
            if (!ok) break;
            if (leader)
                for (int q = 0; q < NQ; ++q) umma_commit(&bs->sfull[q][sb]);
            __syncwarp();
            if (j >= 1) issue_pv(j - 1);
        }
        if (ok && tiles > 0) issue_pv(tiles - 1);
        if (leader) umma_commit(&bs->final_mma);
    } else if (warp >= 4) {
        // ---- softmax and epilogue of Q tile qt: thread <-> query row (TMEM lane) ----
        const int qt = (warp - 4) >> 2;
        const int quarter = warp & 3;
        const int r = 32 * quarter + lane;
        const uint32_t lane_addr = uint32_t(32 * quarter) << 16;
        const uint32_t o_base = tbase + lane_addr + uint32_t(qt) * o_cols;
        const int t = t_first + qt * tpt + r / J.rpt, jh = r % J.rpt;
        const bool live = r < tile_rows && t < J.tokens;
        // Keys this row may see.
        const int row_keys = J.causal ? min(n_keys, max(J.causal_offset + t + 1, 0)) : n_keys;
        float m_run = -INFINITY, l_run = 0.f;
        bool failed = false;
        for (int j = 0; j < tiles; ++j) {
            const int sb = j % J.sbufs;
            const bool ok = wait_bar(&bs->sfull[qt][sb], (j / J.sbufs) & 1, bs, J);
            if (!__all_sync(0xffffffffu, ok)) { failed = true; break; }
            tc_fence_after();
            // One Q tile: the row's 128 scores held in registers.  Two (384
            // threads, 168 registers each): two passes over them in TMEM, 32 at a
            // time, the row max and then the probabilities.
            const uint32_t s_addr = tbase + lane_addr + s_col(qt, sb);
            const int lim = row_keys - j * kKeys;
            float vall[NQ == 1 ? kKeys : 1];
            float mx = -INFINITY;
            if constexpr (NQ == 1) {
#pragma unroll
                for (int c = 0; c < kKeys / 32; ++c) tmem_ld32(s_addr + uint32_t(32 * c), vall + 32 * c);
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bs->sempty[qt][sb]);
#pragma unroll
                for (int i = 0; i < kKeys; ++i)
                    if (i < lim) mx = fmaxf(mx, vall[i]);
            } else {
#pragma unroll
                for (int c = 0; c < kKeys / 32; ++c) {
                    float v[32];
                    tmem_ld32(s_addr + uint32_t(32 * c), v);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (32 * c + i < lim) mx = fmaxf(mx, v[i]);
                }
            }
            mx *= J.scale_log2;                                // scale > 0: the max of the scaled scores
            float alpha = 1.f;
            if (mx != -INFINITY && (m_run == -INFINITY || mx > m_run + kLazyLog2)) {
                const float mn = fmaxf(m_run, mx);
                alpha = m_run == -INFINITY ? 0.f : exp2f(m_run - mn);
                m_run = mn;
                l_run *= alpha;
            }
            // P(j) overwrites the P that P.V(j - 1) reads; a rescale of O needs it done.
            if (j > 0) {
                const bool okd = wait_bar(&bs->odone[qt][(j - 1) & 1], ((j - 1) >> 1) & 1, bs, J);
                if (!__all_sync(0xffffffffu, okd)) { failed = true; break; }
                tc_fence_after();
                if (__any_sync(0xffffffffu, alpha != 1.f)) {
                    for (int c = 0; c < 2 * J.vc; ++c) {
                        float o[32];
                        tmem_ld32(o_base + uint32_t(32 * c), o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] *= alpha;
                        tmem_st32(o_base + uint32_t(32 * c), o);
                    }
                    tmem_wait_st();
                }
            }
            float sum = 0.f;
            uint8_t* prow = smem + off_p + uint32_t(qt * 2) * kChunk + r * 128;
#pragma unroll
            for (int c = 0; c < kKeys / 32; ++c) {
                float v[32];
                if constexpr (NQ == 1) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = vall[32 * c + i];
                } else {
                    tmem_ld32(s_addr + uint32_t(32 * c), v);
                    tmem_wait_ld();
                }
#pragma unroll
                for (int uu = 0; uu < 4; ++uu) {
                    const int u = 4 * c + uu;                  // 8-key unit of the row
                    float p[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        p[e] = 8 * u + e < lim ? sfu_exp2(v[8 * uu + e] * J.scale_log2 - m_run) : 0.f;
                    // The row sum of the probabilities as the MMA sees them (bf16).
                    uint4 w;
                    w.x = pack_bf16x2(p[0], p[1]); w.y = pack_bf16x2(p[2], p[3]);
                    w.z = pack_bf16x2(p[4], p[5]); w.w = pack_bf16x2(p[6], p[7]);
                    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        sum += __uint_as_float(ws[e] << 16) + __uint_as_float(ws[e] & 0xffff0000u);
                    *reinterpret_cast<uint4*>(prow + (u >> 3) * kChunk + (((u & 7) ^ (r & 7)) << 4)) = w;
                }
            }
            if constexpr (NQ != 1) {
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bs->sempty[qt][sb]);
            }
            l_run += sum;
            fence_async_shared();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bs->pfull[qt][j & 1]);
        }
        // ---- epilogue: O / l in bf16, the row's natural-log LSE ----
        if (!failed && tiles > 0) {
            const bool okd = wait_bar(&bs->odone[qt][(tiles - 1) & 1], ((tiles - 1) >> 1) & 1, bs, J);
            failed = !__all_sync(0xffffffffu, okd);
            tc_fence_after();
        }
        if (!failed) {
            const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
            __nv_bfloat16* dst = J.out + b * J.o_sb + int64_t(t) * J.o_st + int64_t(g * J.rpt + jh) * J.o_sh;
            for (int c = 0; c < 2 * J.vc; ++c) {
                float o[32];
                if (tiles > 0) {
                    tmem_ld32(o_base + uint32_t(32 * c), o);
                    tmem_wait_ld();
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = 0.f;
                }
                if (live) {
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int d = 32 * c + 8 * u;
                        uint4 w;
                        w.x = pack_bf16x2(o[8 * u] * inv, o[8 * u + 1] * inv);
                        w.y = pack_bf16x2(o[8 * u + 2] * inv, o[8 * u + 3] * inv);
                        w.z = pack_bf16x2(o[8 * u + 4] * inv, o[8 * u + 5] * inv);
                        w.w = pack_bf16x2(o[8 * u + 6] * inv, o[8 * u + 7] * inv);
                        if (d < J.dim_v) *reinterpret_cast<uint4*>(dst + d) = w;
                    }
                }
            }
            if (live && J.lse)
                J.lse[b * J.l_sb + int64_t(t) * J.l_st + g * J.rpt + jh] =
                    l_run > 0.f ? (m_run + log2f(l_run)) * 0.69314718055994530942f : -INFINITY;
        }
        tmem_wait_ld();
        tc_fence_before();
    }
    __syncthreads();
    if (tid == 64 && tiles > 0) mbar_wait(&bs->final_mma, 0, 2000000000ull);
    if (bs->abort && tid == 0) {
        for (int s = 0; s < J.kring; ++s) {
            mbar_wait(&bs->kfull[s], 0, 100000000ull);
            mbar_wait(&bs->kfull[s], 1, 100000000ull);
        }
        for (int s = 0; s < J.vring; ++s) {
            mbar_wait(&bs->vfull[s], 0, 100000000ull);
            mbar_wait(&bs->vfull[s], 1, 100000000ull);
        }
        mbar_wait(&bs->qfull, 0, 100000000ull);
    }
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tbase, 512);
    }
}

template <int NQ>
int launch_prefill_attention(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm, const Job& J,
                             dim3 grid, cudaStream_t stream) {
    auto kernel = prefill_attention_kernel<NQ>;
    static bool configured[64] = {};
    const int dev = device_info().device;
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemBytes)) != cudaSuccess)
            return fail(SLIMKV_ERR_CUDA, "cudaFuncSetAttribute (prefill attention) failed");
        configured[dev] = true;
    }
    kernel<<<grid, 128 + 128 * NQ, kSmemBytes, stream>>>(qm, km, vm, J);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? SLIMKV_OK
                            : fail(SLIMKV_ERR_CUDA, "prefill attention launch failed: %s", cudaGetErrorString(e));
}

}  // namespace
}  // namespace slimkv

using namespace slimkv;

extern "C" int slimkv_prefill_attention(const slimkv_prefill_attention_args* a, void* stream) {
    if (!a || !a->q || !a->k || !a->v || !a->kv_len || !a->out) return fail(SLIMKV_ERR_INVALID_ARGUMENT, "null pointer");
    if (a->batch <= 0 || a->kv_heads <= 0 || a->tokens <= 0 || a->rows_per_token <= 0 || a->kv_capacity <= 0)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "invalid sizes");
    if (a->rows_per_token > kRows)
        return fail(SLIMKV_ERR_UNSUPPORTED_SHAPE, "prefill attention: at most 128 rows per token");
    if (a->dim_qk <= 0 || a->dim_qk > 64 * kMaxChunks || a->dim_qk % 8 || a->dim_v <= 0 ||
        a->dim_v > 64 * kMaxChunks || a->dim_v % 8)
        return fail(SLIMKV_ERR_UNSUPPORTED_SHAPE, "prefill attention: dims must be multiples of 8 up to 320");
    for (int i = 0; i < 3; ++i)
        if (a->q_stride[i] % 8 || a->kv_stride[i] % 8 || a->out_stride[i] % 8)
            return fail(SLIMKV_ERR_ALIGNMENT, "prefill attention: strides must be multiples of 8 elements");
    if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->out))
        return fail(SLIMKV_ERR_ALIGNMENT, "prefill attention: 16-byte aligned tensors");
    const int heads = a->kv_heads * a->rows_per_token;
    CUtensorMap qm, km, vm;
    int rc;
    // q [B][T][H][dq] (element strides {batch, token, head}) as (dq, H, T, B):
    // a box of rows_per_token heads x floor(128 / rows_per_token) tokens.
    const int tpt = kRows / a->rows_per_token;
    if ((rc = encode_map_4d_box(&qm, a->q, a->dim_qk, heads, a->tokens, a->batch, uint64_t(a->q_stride[2]) * 2,
                                uint64_t(a->q_stride[1]) * 2, uint64_t(a->q_stride[0]) * 2, a->rows_per_token,
                                tpt)))
        return rc;
    // k, v [B][keys][Hkv][d] as (d, Hkv, keys, B), boxes of 128 keys of one head.
    const uint64_t sk = uint64_t(a->kv_stride[1]) * 2, sb = uint64_t(a->kv_stride[0]) * 2;
    const uint64_t sh = a->kv_heads > 1 ? uint64_t(a->kv_stride[2]) * 2 : sk;   // one head: any valid stride
    if ((rc = encode_map_4d(&km, a->k, a->dim_qk, a->kv_heads, a->kv_capacity, a->batch, sh, sk, sb, kKeys))) return rc;
    if ((rc = encode_map_4d(&vm, a->v, a->dim_v, a->kv_heads, a->kv_capacity, a->batch, sh, sk, sb, kKeys))) return rc;
    Job J{};
    J.kc = (a->dim_qk + 63) / 64;
    J.vc = (a->dim_v + 63) / 64;
    J.dim_v = a->dim_v;
    // Two Q tiles per CTA when both dims fit two chunks (their Q, P, O and S
    // then fill shared memory and TMEM: O 2 x 128, S 2 x 128 columns) and the
    // chunk has more than one tile of tokens.
    const int nq = (J.kc <= 2 && J.vc <= 2 && a->tokens > tpt) ? 2 : 1;
    const int slots = int((kTileArea - uint32_t(nq * (J.kc + 2)) * kChunk) / kChunk);
    J.kring = std::min(kMaxRing, slots / 2);
    J.vring = std::min(kMaxRing, slots - J.kring);
#ifndef SLIMKV_PREFILL_VPAIR
#define SLIMKV_PREFILL_VPAIR 1
#endif
    // An even V ring and chunk count keep every chunk pair in adjacent slots.
    if (SLIMKV_PREFILL_VPAIR && J.vc % 2 == 0 && J.vring % 2) {
        if (J.kring > 2) { --J.kring; ++J.vring; }
        else --J.vring;
    }
    J.vpair = SLIMKV_PREFILL_VPAIR && J.vc % 2 == 0 && J.vring % 2 == 0 ? 1 : 0;
    J.sbufs = nq * (64 * J.vc + 2 * kKeys) <= 512 ? 2 : 1;
    J.rpt = a->rows_per_token;
    J.tokens = a->tokens;
    J.kv_heads = a->kv_heads;
    J.kv_len = a->kv_len;
    J.kv_capacity = a->kv_capacity;
    J.causal = a->causal;
    J.causal_offset = a->causal_offset;
    J.scale_log2 = a->scale * 1.4426950408889634f;
    J.out = static_cast<__nv_bfloat16*>(a->out);
    J.o_sb = a->out_stride[0]; J.o_st = a->out_stride[1]; J.o_sh = a->out_stride[2];
    J.lse = a->lse;
    J.l_sb = a->lse_stride[0]; J.l_st = a->lse_stride[1];
    J.status = status_word();
    J.wait_ns = a->wait_limit_ns ? a->wait_limit_ns : 2000000000ull;
    const dim3 grid((a->tokens + nq * tpt - 1) / (nq * tpt), a->kv_heads, a->batch);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    return nq == 2 ? launch_prefill_attention<2>(qm, km, vm, J, grid, st)
                   : launch_prefill_attention<1>(qm, km, vm, J, grid, st);
}
