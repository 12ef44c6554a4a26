// Split-KV flash-decoding body shared by the drop-in attention forward and
// the fused latent decode.
//
// One CTA owns one (batch row b, KV head g, split) work item: the
// `group * queries` query rows that read KV head g (GQA packing: row
// r = l * group + j is query l of head g * group + j), and a contiguous range
// of 64-key tiles.  K/V tiles stream HBM -> shared memory through TMA 4-D
// tensor loads with the 128-byte swizzle (no cluster multicast) into a
// STAGES-deep ring guarded by mbarriers.  Scores and P.V run on the tensor
// cores (m16n8k16, fp32 accumulate) in fp16: bf16 K/V fragments are widened
// to fp16 after ldmatrix (exact inside the fp16 range), so the absorbed
// query and the probabilities keep 11 mantissa bits instead of bf16's 8.
// The online softmax runs in the log2 domain; the CTA writes its normalised
// partial output and natural-log LSE per row, which a combine kernel merges
// across splits.
//
// Warp roles (8 warps): for Q.K^T warp w owns m-tile (w % MT) and the
// w / MT-th slice of each tile's keys; for P.V warp w owns output columns
// [w * W/8, (w+1) * W/8) of every row.  Row maxima cross warps through
// shared memory (two CTA barriers per tile).
#pragma once

#include "common.cuh"

namespace slimkv {

constexpr int kTile = 64;
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kStageBudget = 160 * 1024;
constexpr float kLn2 = 0.69314718055994530942f;

struct AttnJob {
    const void* q;                 // [B, Q, H, D] (element strides below)
    int q_fp16;                    // 1: q holds fp16 values, 0: bf16
    int64_t q_sb, q_sl, q_sh;
    const CUtensorMap* kmap;       // 4-D map {D, Hkv, N, B} over K
    const CUtensorMap* vmap;       // 4-D map {Dv, Hkv, N, B} over V
    int k_bcast, v_bcast;          // batch coordinate forced to 0 (stride-0 caches)
    const int32_t* seqlens;        // keys per batch row (nullable)
    int keys;                      // keys when seqlens is null
    const int32_t* qlens;          // queries per batch row (nullable)
    int queries;                   // queries when qlens is null
    int group;                     // query heads per KV head
    int kv_heads;
    int dk;                        // real key width; Q columns >= dk read as 0
    float scale_log2;              // softmax scale * log2(e)
    int causal;                    // bottom-right causal mask
    int splits, tiles_per_split;
    int rows_alloc;                // row pitch of the partial buffers
    int out_width;                 // column pitch of part_o
    float* part_o;                 // [B][Hkv][splits][rows_alloc][out_width]
    float* part_lse;               // [B][Hkv][splits][rows_alloc]
    unsigned int* status;          // device status word
};

// TILE keys per pipeline stage: 64, or 32 for the widest latents (W = 512)
// so that two stages of K and V still fit beside Q.
template <int W, int MT, int BUDGET = kStageBudget, int TILE = kTile>
struct AttnCfg {
    static constexpr int ROWS = 16 * MT;
    static constexpr int KG = kWarps / MT;      // key groups in Q.K^T
    static constexpr int KPW = TILE / KG;       // keys per warp in Q.K^T
    static constexpr int NTQ = KPW / 8;
    static constexpr int KS = W / 16;
    static constexpr int CH = W / 64;
    static constexpr int DPW = W / kWarps;      // output columns per warp in P.V
    static constexpr int NTV = DPW / 8;
    static constexpr bool QREG = MT <= 2 && W <= 320;   // Q fragments held in registers
    static constexpr int TILE_BYTES = TILE * W * 2;
    static constexpr int STAGE_BYTES = 2 * TILE_BYTES;
    static constexpr int STAGES = (BUDGET / STAGE_BYTES) < 4 ? (BUDGET / STAGE_BYTES) : 4;
    static constexpr int Q_BYTES = QREG ? 0 : ROWS * W * 2;
    static constexpr int P_BYTES = ROWS * 128;
    static constexpr int RED_FLOATS = 2 * KG * ROWS;
    static constexpr int SMEM = STAGES * STAGE_BYTES + Q_BYTES + P_BYTES + RED_FLOATS * 4 +
                                2 * STAGES * 8 + 1024;
    static_assert(W % 64 == 0 && (W <= 320 || (W == 512 && TILE == 32)), "width");
    static_assert(KPW % 8 == 0, "keys per warp");
    static_assert(DPW % 8 == 0, "P.V column split");
    static_assert(STAGES >= 2, "pipeline depth");
    static_assert(SMEM <= 232448, "shared memory");
};

__device__ __forceinline__ uint32_t load_q_pair(const AttnJob& J, int b, int g, int row0, int row,
                                                int col, int rows_valid) {
    if (row >= rows_valid || col >= J.dk) return 0u;
    const int gr = row0 + row;
    const int l = gr / J.group, j = gr - l * J.group;
    const uint16_t* p = static_cast<const uint16_t*>(J.q) + b * J.q_sb + l * J.q_sl +
                        (int64_t)(g * J.group + j) * J.q_sh + col;
    const uint32_t v = *reinterpret_cast<const uint32_t*>(p);
    return J.q_fp16 ? v : bf16x2_to_f16x2(v);
}

// `rb` selects the block of ROWS query rows this CTA owns (row blocks let a
// GQA group wider than 64 query rows be split across CTAs).
template <int W, int MT, int BUDGET = kStageBudget, int TILE = kTile>
__device__ __forceinline__ void attn_body(const AttnJob& J, int b, int g, int split, int rb,
                                          uint8_t* smem) {
    using C = AttnCfg<W, MT, BUDGET, TILE>;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint8_t* stages = smem;
    uint8_t* qs = smem + C::STAGES * C::STAGE_BYTES;
    uint8_t* ps = qs + C::Q_BYTES;
    float* red_m = reinterpret_cast<float*>(ps + C::P_BYTES);
    float* red_l = red_m + C::KG * C::ROWS;
    uint64_t* bars = reinterpret_cast<uint64_t*>(red_l + C::KG * C::ROWS);

    const int n_keys = J.seqlens ? J.seqlens[b] : J.keys;
    const int qlen = J.qlens ? J.qlens[b] : J.queries;
    const int row0 = rb * C::ROWS;                       // first global row of this CTA
    const int rows_valid = min(qlen * J.group - row0, C::ROWS);
    const int n_tiles = (max(n_keys, 0) + TILE - 1) / TILE;
    // The last split runs to the end, so lengths beyond the planning bound
    // are still covered (only slower).
    const int t0 = split * J.tiles_per_split;
    const int t1 = split == J.splits - 1 ? n_tiles : min(n_tiles, t0 + J.tiles_per_split);

    if (tid == 0) {
        for (int s = 0; s < 2 * C::STAGES; ++s) mbar_init(&bars[s], 1);
        fence_barrier_init();
    }
    __syncthreads();

    const int bk = J.k_bcast ? 0 : b, bv = J.v_bcast ? 0 : b;
    auto issue = [&](int t, int s) {
        uint8_t* kd = stages + s * C::STAGE_BYTES;
        uint8_t* vd = kd + C::TILE_BYTES;
        mbar_expect_tx(&bars[s], C::TILE_BYTES);
#pragma unroll
        for (int c = 0; c < C::CH; ++c) tma_load_4d(kd + c * TILE * 128, J.kmap, &bars[s], c * 64, g, t * TILE, bk);
        mbar_expect_tx(&bars[C::STAGES + s], C::TILE_BYTES);
#pragma unroll
        for (int c = 0; c < C::CH; ++c)
            tma_load_4d(vd + c * TILE * 128, J.vmap, &bars[C::STAGES + s], c * 64, g, t * TILE, bv);
    };
    if (tid == 0) {
        for (int s = 0; s < C::STAGES && t0 + s < t1; ++s) issue(t0 + s, s);
    }

    const int mq = warp % MT, kg = warp / MT;
    const int rq0 = 16 * mq + (lane >> 2);

    // ---- Q fragments (A operand, 16 x W per warp) ----
    uint32_t qa[C::QREG ? C::KS : 1][4];
    if constexpr (C::QREG) {
#pragma unroll
        for (int ks = 0; ks < C::KS; ++ks) {
            const int col = ks * 16 + (lane & 3) * 2;
            qa[ks][0] = load_q_pair(J, b, g, row0, rq0, col, rows_valid);
            qa[ks][1] = load_q_pair(J, b, g, row0, rq0 + 8, col, rows_valid);
            qa[ks][2] = load_q_pair(J, b, g, row0, rq0, col + 8, rows_valid);
            qa[ks][3] = load_q_pair(J, b, g, row0, rq0 + 8, col + 8, rows_valid);
        }
    } else {
        // Q staged once in shared memory as CH swizzled [ROWS x 64] chunks.
        for (int idx = tid; idx < C::ROWS * (W / 8); idx += kThreads) {
            const int row = idx / (W / 8), u = idx % (W / 8);
            uint4 val = make_uint4(0, 0, 0, 0);
            if (row < rows_valid && u * 8 < J.dk) {
                const int l = (row0 + row) / J.group, j = (row0 + row) - l * J.group;
                const uint16_t* p = static_cast<const uint16_t*>(J.q) + b * J.q_sb + l * J.q_sl +
                                    (int64_t)(g * J.group + j) * J.q_sh + u * 8;
                val = *reinterpret_cast<const uint4*>(p);
                if (!J.q_fp16) {
                    val.x = bf16x2_to_f16x2(val.x); val.y = bf16x2_to_f16x2(val.y);
                    val.z = bf16x2_to_f16x2(val.z); val.w = bf16x2_to_f16x2(val.w);
                }
            }
            *reinterpret_cast<uint4*>(qs + (u >> 3) * (C::ROWS * 128) + sw128(row, (u & 7) * 8)) = val;
        }
        __syncthreads();
    }

    float o[MT][C::NTV][4];
#pragma unroll
    for (int i = 0; i < MT; ++i)
#pragma unroll
        for (int j = 0; j < C::NTV; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) o[i][j][e] = 0.f;
    float m_qk[2] = {-INFINITY, -INFINITY}, l_qk[2] = {0.f, 0.f};
    float m_pv[2 * MT];
#pragma unroll
    for (int i = 0; i < 2 * MT; ++i) m_pv[i] = -INFINITY;

    const int causal_shift = n_keys - qlen;   // query l sees keys < causal_shift + l + 1
    const uint32_t ps_addr = smem_u32(ps);
    const uint32_t qs_addr = smem_u32(qs);
    bool wait_failed = false, aborted = false;
    int t = t0;
    for (; t < t1; ++t) {
        const int it = t - t0, s = it % C::STAGES;
        const uint32_t par = (it / C::STAGES) & 1;
        if (!mbar_wait(&bars[s], par)) wait_failed = true;
        const uint32_t kt = smem_u32(stages + s * C::STAGE_BYTES);
        const uint32_t vt = kt + C::TILE_BYTES;

        // ---- S = Q K^T for this warp's 16 rows x KPW keys ----
        float sc[C::NTQ][4];
#pragma unroll
        for (int nt = 0; nt < C::NTQ; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) sc[nt][e] = 0.f;
        const int kbase = kg * C::KPW;
#pragma unroll
        for (int ks = 0; ks < C::KS; ++ks) {
            uint32_t a[4];
            if constexpr (C::QREG) {
                a[0] = qa[ks][0]; a[1] = qa[ks][1]; a[2] = qa[ks][2]; a[3] = qa[ks][3];
            } else {
                const int mi = lane >> 3;
                const int row = 16 * mq + (lane & 7) + (mi & 1) * 8;
                const int unit = (ks & 3) * 2 + (mi >> 1);
                ldsm_x4(qs_addr + (ks >> 2) * (C::ROWS * 128) + row * 128 + (((unit ^ row) & 7) << 4),
                        a[0], a[1], a[2], a[3]);
            }
            const uint32_t chunk = kt + (ks >> 2) * (TILE * 128);
            const int u0 = (ks & 3) * 2;
            if constexpr (C::NTQ >= 2) {
#pragma unroll
                for (int nt = 0; nt < C::NTQ; nt += 2) {
                    const int mi = lane >> 3;
                    const int key = kbase + nt * 8 + (mi >> 1) * 8 + (lane & 7);
                    const int unit = u0 + (mi & 1);
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4(chunk + key * 128 + (((unit ^ key) & 7) << 4), b0, b1, b2, b3);
                    mma_f16(sc[nt], a, bf16x2_to_f16x2(b0), bf16x2_to_f16x2(b1));
                    mma_f16(sc[nt + 1], a, bf16x2_to_f16x2(b2), bf16x2_to_f16x2(b3));
                }
            } else {
                const int mi = (lane >> 3) & 1;
                const int key = kbase + (lane & 7);
                const int unit = u0 + mi;
                uint32_t b0, b1;
                ldsm_x2(chunk + key * 128 + (((unit ^ key) & 7) << 4), b0, b1);
                mma_f16(sc[0], a, bf16x2_to_f16x2(b0), bf16x2_to_f16x2(b1));
            }
        }
        // ---- scale, mask, per-warp row maxima ----
        const int key0 = t * TILE + kbase + (lane & 3) * 2;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int row = rq0 + 8 * hh;
            const int limit = row < rows_valid
                                  ? (J.causal ? min(n_keys, causal_shift + (row0 + row) / J.group + 1) : n_keys)
                                  : 0;
            float mx = -INFINITY;
#pragma unroll
            for (int nt = 0; nt < C::NTQ; ++nt)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int key = key0 + nt * 8 + e;
                    const float v = key < limit ? sc[nt][2 * hh + e] * J.scale_log2 : -INFINITY;
                    sc[nt][2 * hh + e] = v;
                    mx = fmaxf(mx, v);
                }
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            if ((lane & 3) == 0) red_m[kg * C::ROWS + row] = mx;
        }
        // Barrier A: maxima visible; every warp finished the previous tile,
        // so its stage can be refilled.
        if (__syncthreads_or(wait_failed)) { aborted = true; break; }
        if (tid == 0 && t > t0 && t - 1 + C::STAGES < t1) issue(t - 1 + C::STAGES, (it - 1) % C::STAGES);

        // ---- probabilities of this warp's keys -> shared memory ----
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int row = rq0 + 8 * hh;
            float mn = m_qk[hh];
#pragma unroll
            for (int k = 0; k < C::KG; ++k) mn = fmaxf(mn, red_m[k * C::ROWS + row]);
            const float alpha = mn == -INFINITY ? 1.f : fast_exp2(m_qk[hh] - mn);
            float sum = 0.f;
#pragma unroll
            for (int nt = 0; nt < C::NTQ; ++nt) {
                const float p0 = mn == -INFINITY ? 0.f : f16_round(fast_exp2(sc[nt][2 * hh] - mn));
                const float p1 = mn == -INFINITY ? 0.f : f16_round(fast_exp2(sc[nt][2 * hh + 1] - mn));
                sum += p0 + p1;
                const int col = kbase + nt * 8 + (lane & 3) * 2;
                *reinterpret_cast<uint32_t*>(ps + sw128(row, col)) = pack_f16x2(p0, p1);
            }
            l_qk[hh] = l_qk[hh] * alpha + sum;
            m_qk[hh] = mn;
        }
        // ---- rescale the P.V accumulators of every row ----
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const int row = 16 * mt + (lane >> 2) + 8 * hh;
                float mn = m_pv[2 * mt + hh];
#pragma unroll
                for (int k = 0; k < C::KG; ++k) mn = fmaxf(mn, red_m[k * C::ROWS + row]);
                const float alpha = mn == -INFINITY ? 1.f : fast_exp2(m_pv[2 * mt + hh] - mn);
                m_pv[2 * mt + hh] = mn;
#pragma unroll
                for (int nt = 0; nt < C::NTV; ++nt) {
                    o[mt][nt][2 * hh] *= alpha;
                    o[mt][nt][2 * hh + 1] *= alpha;
                }
            }
        __syncthreads();  // Barrier B: P visible.
        if (!mbar_wait(&bars[C::STAGES + s], par)) wait_failed = true;

        // ---- O += P V for this warp's columns ----
        // V rows past the sequence length hold whatever the cache has there;
        // their P is zero, and zeroing the operand as well keeps a non-finite
        // stale value from turning 0 * x into NaN.
        const int d0 = warp * C::DPW;
        const int vlim = n_keys - t * TILE;
#pragma unroll
        for (int kk = 0; kk < TILE / 16; ++kk) {
            const int kq = kk * 16 + (lane & 3) * 2;
            const uint32_t m_lo = (kq < vlim ? 0xffffu : 0u) | (kq + 1 < vlim ? 0xffff0000u : 0u);
            const uint32_t m_hi = (kq + 8 < vlim ? 0xffffu : 0u) | (kq + 9 < vlim ? 0xffff0000u : 0u);
            uint32_t a[MT][4];
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                const int mi = lane >> 3;
                const int row = 16 * mt + (lane & 7) + (mi & 1) * 8;
                const int unit = 2 * kk + (mi >> 1);
                ldsm_x4(ps_addr + row * 128 + (((unit ^ row) & 7) << 4), a[mt][0], a[mt][1], a[mt][2], a[mt][3]);
            }
#pragma unroll
            for (int nt = 0; nt + 1 < C::NTV; nt += 2) {
                const int mi = lane >> 3;
                const int key = kk * 16 + (lane & 7) + (mi & 1) * 8;
                const int dim = d0 + nt * 8 + (mi >> 1) * 8;
                const int unit = (dim & 63) >> 3;
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(vt + (dim >> 6) * (TILE * 128) + key * 128 + (((unit ^ key) & 7) << 4), b0, b1, b2, b3);
                b0 = bf16x2_to_f16x2(b0) & m_lo; b1 = bf16x2_to_f16x2(b1) & m_hi;
                b2 = bf16x2_to_f16x2(b2) & m_lo; b3 = bf16x2_to_f16x2(b3) & m_hi;
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    mma_f16(o[mt][nt], a[mt], b0, b1);
                    mma_f16(o[mt][nt + 1], a[mt], b2, b3);
                }
            }
            if constexpr (C::NTV % 2) {
                constexpr int nt = C::NTV - 1;
                const int mi = (lane >> 3) & 1;
                const int key = kk * 16 + (lane & 7) + mi * 8;
                const int dim = d0 + nt * 8;
                const int unit = (dim & 63) >> 3;
                uint32_t b0, b1;
                ldsm_x2_t(vt + (dim >> 6) * (TILE * 128) + key * 128 + (((unit ^ key) & 7) << 4), b0, b1);
                b0 = bf16x2_to_f16x2(b0) & m_lo; b1 = bf16x2_to_f16x2(b1) & m_hi;
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) mma_f16(o[mt][nt], a[mt], b0, b1);
            }
        }
    }
    if (!aborted && __syncthreads_or(wait_failed)) aborted = true;
    if (aborted) {
        // A TMA wait timed out: report, wait (bounded) for the copies this CTA
        // issued, and leave without writing results.
        if (tid == 0) {
            report(J.status, SLIMKV_DEVICE_TIMEOUT);
            const int issued_end = min(t1, max(t0 + C::STAGES, t + C::STAGES - 1));
            for (int tt = max(t0, issued_end - C::STAGES); tt < issued_end; ++tt) {
                const int s2 = (tt - t0) % C::STAGES;
                const uint32_t p2 = ((tt - t0) / C::STAGES) & 1;
                mbar_wait(&bars[s2], p2);
                mbar_wait(&bars[C::STAGES + s2], p2);
            }
        }
        __syncthreads();
        return;
    }

    // ---- row sums across quads and key groups; write normalised partials ----
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        float l = l_qk[hh];
        l += __shfl_xor_sync(0xffffffffu, l, 1);
        l += __shfl_xor_sync(0xffffffffu, l, 2);
        if ((lane & 3) == 0) red_l[kg * C::ROWS + rq0 + 8 * hh] = l;
    }
    __syncthreads();
    const int64_t base_row = ((int64_t)(b * J.kv_heads + g) * J.splits + split) * J.rows_alloc + row0;
    const int d0 = warp * C::DPW;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int row = 16 * mt + (lane >> 2) + 8 * hh;
            if (row >= rows_valid) continue;
            float l = 0.f;
#pragma unroll
            for (int k = 0; k < C::KG; ++k) l += red_l[k * C::ROWS + row];
            const float inv = l > 0.f ? 1.f / l : 0.f;
            float* dst = J.part_o + (base_row + row) * J.out_width;
#pragma unroll
            for (int nt = 0; nt < C::NTV; ++nt) {
                const int col = d0 + nt * 8 + (lane & 3) * 2;
                if (col < J.out_width) {
                    *reinterpret_cast<float2*>(dst + col) =
                        make_float2(o[mt][nt][2 * hh] * inv, o[mt][nt][2 * hh + 1] * inv);
                }
            }
            if (warp == 0 && (lane & 3) == 0)
                J.part_lse[base_row + row] = l > 0.f ? (m_pv[2 * mt + hh] + log2f(l)) * kLn2 : -INFINITY;
        }
}

}  // namespace slimkv
