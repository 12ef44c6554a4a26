// Prologue and merge kernels of the fused latent decode step.
//
// Both are small tensor-core GEMMs around the attention kernel:
//   prologue: q_lat[r, :] = rope(q)[r, :] . U_k[g]      (fa2_decode.py:41-46)
//   merge:    out[r, :]   = o_lat[r, :] . U_v[g]^T      (fa2_decode.py:49-54)
// Operands are staged in shared memory with vector loads issued in parallel
// (the loops carry no load->use dependency chains) and multiplied with
// m16n8k16 fp16 MMAs (bf16 weights widen to fp16 exactly), fp32 accumulate.
#pragma once

#include "common.cuh"
#include "latent_tc.h"
#include "latent_tc_plan.cuh"

namespace slimkv {

constexpr int kMaxRows = 16;      // query rows per KV head (group * length)
constexpr int kProRows = 64;      // query rows per prologue CTA (four m-tiles)

struct PrologueArgs {
    const __nv_bfloat16* q;
    int64_t q_sb, q_sl, q_sh;
    int batch, length, heads, kv_heads, dim, rank_k, rank_v, width, group, seq_per_cta;
    const int32_t* qpos;
    const int32_t* qlens;
    const float* cos;
    const float* sin;
    int rope_positions;
    const __nv_bfloat16* uk;
    __nv_bfloat16* q_rot;   // [B, L, H, D]
    __half* q_lat;          // [B, L, H, width] fp16 (split-KV path), or
    __nv_bfloat16* q_hilo;  // [B][hilo_rows][width] bf16 hi/lo rows (tensor-memory path)
    int hilo;
    int hilo_rows;          // 128: row hl*H*nq + l*H + h; 160 (split): row l*2H + hl*H + h
    int hilo_split;
    const __nv_bfloat16* new_k;
    const __nv_bfloat16* new_v;
    int64_t new_stride;
    __nv_bfloat16* raw_k_rot;
    __nv_bfloat16* raw_v;
    __nv_bfloat16* raw_k_pre;
    int64_t raw_sb, raw_st, raw_sh;
    const int32_t* raw_len;
    int raw_capacity;
    const __nv_bfloat16* new_lat_k;
    const __nv_bfloat16* new_lat_v;
    int64_t new_lat_stride;
    __nv_bfloat16* lat_k;
    __nv_bfloat16* lat_v;
    int64_t lat_sb, lat_sr;
    const int32_t* latent_len;
    int lat_capacity;
    // Latent and raw rows per sequence the attention launch covers: a longer
    // sequence is flagged SLIMKV_DEVICE_BAD_LENGTH (its extra rows would be
    // outside every split).
    int lat_cover, raw_cover;
    // Paged latent cache (lat_pages != nullptr): row n of sequence b at
    // lat_pages + table[b][n / slots] * page_stride + sink + (n % slots) * W.
    __nv_bfloat16* lat_pages;
    int64_t lat_page_stride, lat_table_stride;
    int lat_slots, lat_sink, lat_num_pages;
    const int32_t* lat_table;
    // Plan of the tensor-memory attention (latent_tc_plan.cuh), written by
    // block (0, 0, gridDim.z - 1) when do_plan is set (that z-slice does
    // nothing else).
    TcPlanArgs plan;
    int do_plan;
    unsigned int* status;
};

__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

// Rotate dims [d0, d0+8) of one head row with the reference's BF16 rounding:
// out = bf16(bf16(x*bf16(cos)) + bf16(rotate_half(x)*bf16(sin)))
// (slimkv/llama3/decode_kernels.py:40-51).  `half` is dim/2, a multiple of 8.
__device__ __forceinline__ void rope8(const __nv_bfloat16* row, int d0, int half, const float* cos_row,
                                      const float* sin_row, float out[8]) {
    const int pd = d0 < half ? d0 + half : d0 - half;
    // Read-only loads (ld.global.nc): the compiler may issue them ahead of
    // the caller's stores.
    const uint4 xv = __ldg(reinterpret_cast<const uint4*>(row + d0));
    const uint4 pv = __ldg(reinterpret_cast<const uint4*>(row + pd));
    const float4 c0 = __ldg(reinterpret_cast<const float4*>(cos_row + d0));
    const float4 c1 = __ldg(reinterpret_cast<const float4*>(cos_row + d0 + 4));
    const float4 s0 = __ldg(reinterpret_cast<const float4*>(sin_row + d0));
    const float4 s1 = __ldg(reinterpret_cast<const float4*>(sin_row + d0 + 4));
    const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w}, pw[4] = {pv.x, pv.y, pv.z, pv.w};
    const float cs[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float sn[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    const float sign = d0 < half ? -1.f : 1.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const float x = (e & 1) ? bf16_hi(xw[e >> 1]) : bf16_lo(xw[e >> 1]);
        const float p = (e & 1) ? bf16_hi(pw[e >> 1]) : bf16_lo(pw[e >> 1]);
        const float first = bf16_round(__fmul_rn(x, bf16_round(cs[e])));
        const float second = bf16_round(__fmul_rn(sign * p, bf16_round(sn[e])));
        out[e] = bf16_round(__fadd_rn(first, second));
    }
}

__device__ __forceinline__ uint4 pack8_bf16(const float v[8]) {
    return make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                      pack_bf16x2(v[6], v[7]));
}
__device__ __forceinline__ uint4 pack8_f16(const float v[8]) {
    return make_uint4(pack_f16x2(v[0], v[1]), pack_f16x2(v[2], v[3]), pack_f16x2(v[4], v[5]),
                      pack_f16x2(v[6], v[7]));
}
__device__ __forceinline__ uint4 widen8(uint4 v) {
    return make_uint4(bf16x2_to_f16x2(v.x), bf16x2_to_f16x2(v.y), bf16x2_to_f16x2(v.z), bf16x2_to_f16x2(v.w));
}

// grid (Hkv, width / 64, ceil(B / seq_per_cta) [+ 1 planning slice]), 256
// threads.  CTA (g, cc, bb)
// absorbs the 64 query rows of KV head g for sequences [bb*spc, (bb+1)*spc)
// into latent columns [cc*64, cc*64 + 64); the cc == 0 CTAs also write q_rot
// and append this step's raw token (and, for g == 0, the Beacon latents).
__global__ void __launch_bounds__(256) decode_prologue_kernel(PrologueArgs a) {
    __shared__ __align__(1024) uint8_t s_ab[kProRows * 128 * 2 + 128 * 64 * 2];
    uint8_t* s_a = s_ab;                                // rope(q): 2 chunks [64 x 64] fp16
    uint8_t* s_b = s_ab + kProRows * 128 * 2;           // U_k[g][:, cc*64 : +64] fp16
    const int g = blockIdx.x, cc = blockIdx.y, bb = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // An attention launch that depends on this one may start as soon as every
    // block here has started (it waits for this grid's end before reading
    // what it writes): all of this grid is resident by then, so it can only
    // take SMs these blocks leave.
    if (tid == 0) grid_launch_dependents();
    if (a.do_plan && bb == int(gridDim.z) - 1) {
        // The last z-slice only plans the attention (one block, in parallel
        // with the absorb blocks), in this block's shared memory when it fits.
        if (g == 0 && cc == 0)
            plan_tc_work(a.plan, reinterpret_cast<int32_t*>(s_ab), int(sizeof(s_ab) / sizeof(int32_t)));
        return;
    }
    const int rps = a.length * a.group;                 // rows per sequence
    const int b0 = bb * a.seq_per_cta;
    const int half = a.dim / 2;
    if (g == 0 && cc == 0) {
        for (int s = tid; s < a.seq_per_cta; s += 256) {
            const int b = b0 + s;
            if (b < a.batch && (a.latent_len[b] > a.lat_cover || a.raw_len[b] > a.raw_cover))
                report(a.status, SLIMKV_DEVICE_BAD_LENGTH);
        }
    }

    // 1. U_k column chunk -> shared (fp16).
#pragma unroll
    for (int i = tid; i < 128 * 8; i += 256) {
        const int d = i >> 3, u = i & 7, col = cc * 64 + u * 8;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (col < a.rank_k) v = widen8(__ldg(reinterpret_cast<const uint4*>(a.uk + ((int64_t)g * a.dim + d) * a.rank_k + col)));
        *reinterpret_cast<uint4*>(s_b + sw128(d, u * 8)) = v;
    }
    // 2. RoPE of the CTA's query rows -> shared (fp16, exact copies of bf16).
#pragma unroll
    for (int i = tid; i < kProRows * 16; i += 256) {
        const int r = i >> 4, d0 = (i & 15) * 8;
        const int s = r / rps, rr = r - s * rps, l = rr / a.group, j = rr - l * a.group;
        const int b = b0 + s, h = g * a.group + j;
        float o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (s < a.seq_per_cta && b < a.batch && l < (a.qlens ? a.qlens[b] : a.length)) {
            int pos = a.qpos[b * a.length + l];
            if (pos < 0 || pos >= a.rope_positions) {
                report(a.status, SLIMKV_DEVICE_BAD_LENGTH);
                pos = 0;
            }
            rope8(a.q + b * a.q_sb + l * a.q_sl + h * a.q_sh, d0, half, a.cos + (int64_t)pos * a.dim,
                  a.sin + (int64_t)pos * a.dim, o);
            if (cc == 0)
                *reinterpret_cast<uint4*>(a.q_rot + (((int64_t)b * a.length + l) * a.heads + h) * a.dim + d0) =
                    pack8_bf16(o);
        }
        *reinterpret_cast<uint4*>(s_a + (d0 >> 6) * (kProRows * 128) + sw128(r, d0 & 63)) = pack8_f16(o);
    }
    __syncthreads();
    // 3. [64 x 128] . [128 x 64] on the tensor cores: warp -> m-tile (warp & 3),
    //    32 output columns (warp >> 2).
    const int mt = warp & 3, nh = warp >> 2, mi = lane >> 3;
    float acc[4][4];
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[n][e] = 0.f;
    const uint32_t a_base = smem_u32(s_a), b_base = smem_u32(s_b);
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
        uint32_t af[4];
        const int row = 16 * mt + (lane & 7) + (mi & 1) * 8;
        const int unit = (ks & 3) * 2 + (mi >> 1);
        ldsm_x4(a_base + (ks >> 2) * (kProRows * 128) + row * 128 + (((unit ^ row) & 7) << 4), af[0], af[1], af[2],
                af[3]);
#pragma unroll
        for (int np = 0; np < 2; ++np) {
            const int krow = ks * 16 + (lane & 7) + (mi & 1) * 8;
            const int col = nh * 32 + np * 16 + (mi >> 1) * 8;
            uint32_t b0, b1, b2, b3;
            ldsm_x4_t(b_base + krow * 128 + ((((col >> 3) ^ krow) & 7) << 4), b0, b1, b2, b3);
            mma_f16(acc[2 * np], af, b0, b1);
            mma_f16(acc[2 * np + 1], af, b2, b3);
        }
    }
    // 4. q_lat for the valid rows: fp16, or a bf16 hi/lo pair (q = hi + lo)
    //    at rows l*H + h (hi) and H*nq + l*H + h (lo) of the sequence's
    //    block, nq being the sequence's query count; split: l*2H + h (hi) and
    //    l*2H + H + h (lo), each query's pair contiguous.
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        const int r = 16 * mt + (lane >> 2) + 8 * hh;
        const int s = r / rps, rr = r - s * rps, l = rr / a.group, j = rr - l * a.group;
        const int b = b0 + s;
        if (s >= a.seq_per_cta || b >= a.batch) continue;
        const int nq = a.qlens ? a.qlens[b] : a.length;
        if (l >= nq) continue;
        const int col = cc * 64 + nh * 32 + (lane & 3) * 2;
        if (a.hilo) {
            const int h = g * a.group + j;
            const int hrow = a.hilo_split ? l * 2 * a.heads + h : l * a.heads + h;
            __nv_bfloat16* hi = a.q_hilo + ((int64_t)b * a.hilo_rows + hrow) * a.width + col;
            __nv_bfloat16* lo = hi + int64_t(a.hilo_split ? a.heads : a.heads * nq) * a.width;
#pragma unroll
            for (int n = 0; n < 4; ++n) {
                const float x0 = acc[n][2 * hh], x1 = acc[n][2 * hh + 1];
                const float h0 = bf16_round(x0), h1 = bf16_round(x1);
                *reinterpret_cast<uint32_t*>(hi + n * 8) = pack_bf16x2(h0, h1);
                *reinterpret_cast<uint32_t*>(lo + n * 8) = pack_bf16x2(x0 - h0, x1 - h1);
            }
        } else {
            __half* dst = a.q_lat + (((int64_t)b * a.length + l) * a.heads + g * a.group + j) * a.width + col;
#pragma unroll
            for (int n = 0; n < 4; ++n)
                *reinterpret_cast<uint32_t*>(dst + n * 8) = pack_f16x2(acc[n][2 * hh], acc[n][2 * hh + 1]);
        }
    }
    if (cc != 0) return;
    // 5. Append this step's raw token of head g: rotated key, value, pre-RoPE key.
    if (a.new_k) {
        for (int i = tid; i < a.seq_per_cta * 16; i += 256) {
            const int s = i >> 4, d0 = (i & 15) * 8, b = b0 + s;
            if (b >= a.batch) continue;
            const int row = a.raw_len[b] - 1;
            if (row < 0 || row >= a.raw_capacity) {
                report(a.status, SLIMKV_DEVICE_BAD_LENGTH);
                continue;
            }
            int pos = a.qpos[b * a.length];
            if (pos < 0 || pos >= a.rope_positions) pos = 0;
            const __nv_bfloat16* k = a.new_k + b * a.new_stride + (int64_t)g * a.dim;
            const __nv_bfloat16* v = a.new_v + b * a.new_stride + (int64_t)g * a.dim;
            float o[8];
            rope8(k, d0, half, a.cos + (int64_t)pos * a.dim, a.sin + (int64_t)pos * a.dim, o);
            const int64_t dst = b * a.raw_sb + row * a.raw_st + g * a.raw_sh + d0;
            *reinterpret_cast<uint4*>(a.raw_k_rot + dst) = pack8_bf16(o);
            *reinterpret_cast<uint4*>(a.raw_v + dst) = __ldg(reinterpret_cast<const uint4*>(v + d0));
            if (a.raw_k_pre) *reinterpret_cast<uint4*>(a.raw_k_pre + dst) = __ldg(reinterpret_cast<const uint4*>(k + d0));
        }
    }
    // 6. Append the Beacon latent pair of rows that insert one this step.
    if (g == 0 && a.new_lat_k) {
        const int ku = a.rank_k / 8, vu = a.rank_v / 8;
        for (int i = tid; i < a.seq_per_cta * (ku + vu); i += 256) {
            const int s = i / (ku + vu), u = i - s * (ku + vu), b = b0 + s;
            if (b >= a.batch || (a.qlens ? a.qlens[b] : a.length) != 2) continue;
            const int row = a.latent_len[b] - 1;
            const uint4 val = u < ku ? *reinterpret_cast<const uint4*>(a.new_lat_k + b * a.new_lat_stride + u * 8)
                                     : *reinterpret_cast<const uint4*>(a.new_lat_v + b * a.new_lat_stride + (u - ku) * 8);
            if (a.lat_pages) {
                // BeaconPages.append of one row (paged_cache.py:78-87).
                const int64_t pi = row / a.lat_slots;
                const int page = (row < 0 || pi >= a.lat_table_stride) ? -1 : a.lat_table[b * a.lat_table_stride + pi];
                if (page < 0 || page >= a.lat_num_pages) {
                    report(a.status, SLIMKV_DEVICE_BAD_LENGTH);
                    continue;
                }
                *reinterpret_cast<uint4*>(a.lat_pages + int64_t(page) * a.lat_page_stride + a.lat_sink +
                                          int64_t(row % a.lat_slots) * (a.rank_k + a.rank_v) + u * 8) = val;
                continue;
            }
            if (row < 0 || row >= a.lat_capacity) {
                report(a.status, SLIMKV_DEVICE_BAD_LENGTH);
                continue;
            }
            if (u < ku) *reinterpret_cast<uint4*>(a.lat_k + b * a.lat_sb + row * a.lat_sr + u * 8) = val;
            else *reinterpret_cast<uint4*>(a.lat_v + b * a.lat_sb + row * a.lat_sr + (u - ku) * 8) = val;
        }
    }
}

struct MergeArgs {
    const float* lat_o; const float* lat_lse; int lat_splits, lat_rows, lat_width;
    // Tensor-memory route (plan != nullptr): the partials of a segment are the
    // pieces [seg_piece[s], seg_piece[s + 1]) of its class; class 1's latent
    // pieces follow lat_pieces slots after class 0's.  Otherwise sequence b
    // (and KV head g) has lat_splits (raw_splits) consecutive partials.
    const int32_t* plan;
    TcPlanLayout PL;
    int lat_pieces;
    const float* raw_o; const float* raw_lse; int raw_splits, raw_rows;
    int raw_l_pitch;        // raw partial row of (query l, head j): l * raw_l_pitch + j
    const __nv_bfloat16* q_rot;
    const __nv_bfloat16* uv; const __nv_bfloat16* uk_bias; const __nv_bfloat16* uv_bias;
    const int32_t* qlens;
    int batch, length, heads, kv_heads, dim, rank_v, rank_v_pad, group, seq_per_cta;
    float scale;
    void* out; int out_fp32; int64_t o_sb, o_sl;
    float* out_lse;                // [B][L][H] merged LSE (nullable)
};

// Most CTAs of a split-KV attention launch (the tensor-memory route sizes its
// launch below this).
constexpr int kMergeMaxSplits = 160;

// Dynamic shared memory of decode_merge_kernel for a padded value rank:
// U_v[g] bf16 [128 x rvp], o_lat hi and lo bf16 [16 x rvp] each, raw rows
// fp32 [16 x dim], LSEs [2][16], latent LSE shifts [16].
__host__ __device__ constexpr size_t merge_smem_bytes(int rank_v_pad, int dim) {
    return 1024 + size_t(128 + 32) * rank_v_pad * 2 + size_t(16) * dim * 4 + 48 * 4;
}

// out[c:c+4] = sum_s w_s part_s[c:c+4] / sum_s w_s with w_s = exp(lse_s - max
// lse), over the n partials at src + s * pitch (LSE at lse + s * lse_pitch),
// in one pass (running max); *row_lse = log sum_s exp(lse_s) (-inf if none).
__device__ __forceinline__ float4 combine_partials(const float* src, int64_t pitch, const float* lse, int64_t lse_pitch,
                                                   int n, float* row_lse) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    float m = -INFINITY, tot = 0.f;
    for (int s0 = 0; s0 < n; s0 += 8) {
        float4 x[8];
        float ls[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            ls[u] = -INFINITY;
            if (s0 + u < n) {
                x[u] = __ldg(reinterpret_cast<const float4*>(src + (s0 + u) * pitch));
                ls[u] = __ldg(lse + (s0 + u) * lse_pitch);
            }
        }
        float mn = m;
#pragma unroll
        for (int u = 0; u < 8; ++u) mn = fmaxf(mn, ls[u]);
        if (mn == -INFINITY) continue;
        const float sc = m == -INFINITY ? 0.f : expf(m - mn);
        acc.x *= sc; acc.y *= sc; acc.z *= sc; acc.w *= sc;
        tot *= sc;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            if (ls[u] == -INFINITY) continue;
            const float w = expf(ls[u] - mn);
            acc.x = fmaf(w, x[u].x, acc.x); acc.y = fmaf(w, x[u].y, acc.y);
            acc.z = fmaf(w, x[u].z, acc.z); acc.w = fmaf(w, x[u].w, acc.w);
            tot += w;
        }
        m = mn;
    }
    if (tot > 0.f) {
        const float inv = 1.f / tot;
        acc.x *= inv; acc.y *= inv; acc.z *= inv; acc.w *= inv;
    }
    *row_lse = tot > 0.f ? m + logf(tot) : -INFINITY;
    return acc;
}

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit_wait_all() {
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// First partial and partial count of sequence b's latent branch.
__device__ __forceinline__ void lat_parts(const MergeArgs& a, int b, int& p0, int& n) {
    if (a.plan) {
        const int2 r = *reinterpret_cast<const int2*>(a.plan + a.PL.lat_range + 2 * b);
        p0 = (r.x & 0xffffff) + ((r.x >> 24) ? a.lat_pieces : 0);
        n = r.y;
    } else {
        p0 = b * a.lat_splits;
        n = a.lat_splits;
    }
}
// First partial and partial count of the raw branch of (sequence b, KV head g).
__device__ __forceinline__ void raw_parts(const MergeArgs& a, int b, int g, int& p0, int& n) {
    const int s = b * a.kv_heads + g;
    if (a.plan) {
        const int32_t* pc = a.plan + a.PL.seg_piece[2];
        p0 = pc[s];
        n = pc[s + 1] - pc[s];
    } else {
        p0 = s * a.raw_splits;
        n = a.raw_splits;
    }
}

// grid (Hkv, ceil(B / seq_per_cta), row split), 256 threads,
// merge_smem_bytes() of dynamic shared memory.  CTAs (g, bb, *) merge the
// (<= 16) query rows (seq_per_cta sequences x L x group) of KV head g, each
// CTA an equal share of them.
//   1. U_v[g] -> shared with asynchronous copies (bf16 as stored, the MMA's
//      column-major B operand), overlapping steps 2-3.
//   2. One warp per row: lane s holds the LSEs of splits s, s+32, s+64 and
//      s+96 of each branch and turns them into normalised weights (splits <=
//      kMergeMaxSplits); the row's LSEs (latent one shifted by scale * q .
//      b_k) go to shared memory.
//   3. All threads: weighted split sums over (row, 4-column) items of the
//      valid rows, every split's load independent of the others; the latent
//      rows are kept as a bf16 pair hi + lo (fp32-level accuracy through the
//      bf16 tensor cores).
//   4. Up-projection (two MMAs per k-step: hi and lo rows), bias, LSE merge,
//      store.
__global__ void __launch_bounds__(256) decode_merge_kernel(MergeArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int rvp = a.rank_v_pad;                       // multiple of 64
    uint8_t* s_b = smem;                                // U_v[g]: rvp/64 chunks [128 x 64] bf16
    uint8_t* s_hi = s_b + 128 * rvp * 2;                // o_lat hi: rvp/64 chunks [16 x 64] bf16
    uint8_t* s_lo = s_hi + 16 * rvp * 2;                // o_lat lo
    float* s_raw = reinterpret_cast<float*>(s_lo + 16 * rvp * 2);   // [16][D]
    float* s_lse = s_raw + 16 * a.dim;                  // [2][16]: latent, raw (then [16] shifts)
    const int g = blockIdx.x, bb = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rps = a.length * a.group, b0 = bb * a.seq_per_cta;
    const int nrows = min(16, a.seq_per_cta * rps);
    // gridDim.z CTAs share the rows: this one takes [row0, row0 + part) as its
    // local rows 0 .. part - 1.
    const int part = (nrows + int(gridDim.z) - 1) / int(gridDim.z), row0 = int(blockIdx.z) * part;
    // rr: the row's index in the raw branch partials.
    auto row_info = [&](int r, int& b, int& l, int& h, int& rr) -> bool {
        const int rg = r + row0;
        const int s = rg / rps, rs = rg - s * rps;
        l = rs / a.group;
        b = b0 + s;
        const int j = rs - l * a.group;
        h = g * a.group + j;
        rr = l * a.raw_l_pitch + j;
        return r < part && rg < nrows && b < a.batch && l < (a.qlens ? a.qlens[b] : a.length);
    };

    // 0. (Before the attention launch completes.)  Each row's partial ranges
    //    (latent, raw) from the plan, U_v[g] (rows d, columns c) -> shared
    //    asynchronously with zero columns past the rank, the zero rows of the
    //    A operand; then (after the attention grid) the latent LSE shift
    //    scale * q . b_k of each row (fa2_decode.py:157-160).
    __shared__ int s_parts[16][4];
    float* s_shift = s_lse + 32;                        // [16]
    if (tid < 16) {
        int b, l, h, rr, p0 = 0, n = 0, q0 = 0, m = 0;
        if (row_info(tid, b, l, h, rr)) {
            lat_parts(a, b, p0, n);
            raw_parts(a, b, g, q0, m);
        }
        s_parts[tid][0] = p0; s_parts[tid][1] = n; s_parts[tid][2] = q0; s_parts[tid][3] = m;
    }
    const int units = rvp / 8;
    for (int i = tid; i < 128 * units; i += 256) {
        const int d = i / units, u = i - d * units, col = u * 8;
        uint8_t* dst = s_b + (u >> 3) * (128 * 128) + sw128(d, (u & 7) * 8);
        if (col < a.rank_v) cp_async16(dst, a.uv + ((int64_t)g * a.dim + d) * a.rank_v + col);
        else *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
    }
    cp_async_commit();
    for (int i = tid; i < 2 * 16 * rvp / 8; i += 256) reinterpret_cast<uint4*>(s_hi)[i] = make_uint4(0, 0, 0, 0);
    grid_dependency_wait();
    for (int r = warp; r < 16; r += 8) {
        int b, l, h, rr;
        float dot = 0.f;
        if (a.uk_bias && row_info(r, b, l, h, rr)) {
            const __nv_bfloat16* q = a.q_rot + (((int64_t)b * a.length + l) * a.heads + h) * a.dim;
            const __nv_bfloat16* bk = a.uk_bias + (int64_t)g * a.dim;
            for (int d = lane; d < a.dim; d += 32) dot += __bfloat162float(q[d]) * __bfloat162float(bk[d]);
#pragma unroll
            for (int off = 16; off; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
        }
        if (lane == 0) s_shift[r] = dot * a.scale;
    }
    __syncthreads();
    // 1. Latent branch: o_lat[r, c:c+4] combined over the row's pieces in one
    //    pass -> bf16 hi / lo (fp32-level accuracy through the bf16 tensor
    //    cores); the column-0 item also records the row's LSE (shifted).
    {
        const int c4n = rvp / 4;
        const int64_t pitch = (int64_t)a.lat_rows * a.lat_width;
        for (int it = tid; it < part * c4n; it += 256) {
            const int r = it / c4n, c = (it - r * c4n) * 4;
            int b, l, h, rr;
            if (!row_info(r, b, l, h, rr) || c >= a.lat_width) continue;
            const int p0 = s_parts[r][0], nsp = s_parts[r][1];
            const int64_t row = (int64_t)p0 * a.lat_rows + l * a.heads + h;
            float lse;
            const float4 acc = combine_partials(a.lat_o + row * a.lat_width + c, pitch, a.lat_lse + row, a.lat_rows,
                                                nsp, &lse);
            if (c == 0) s_lse[r] = lse == -INFINITY ? lse : lse + s_shift[r];
            const float hx = bf16_round(acc.x), hy = bf16_round(acc.y), hz = bf16_round(acc.z), hw = bf16_round(acc.w);
            const int off = (c >> 6) * (16 * 128) + sw128(r, c & 63);
            *reinterpret_cast<uint2*>(s_hi + off) = make_uint2(pack_bf16x2(hx, hy), pack_bf16x2(hz, hw));
            *reinterpret_cast<uint2*>(s_lo + off) =
                make_uint2(pack_bf16x2(acc.x - hx, acc.y - hy), pack_bf16x2(acc.z - hz, acc.w - hw));
        }
    }
    // 2. Raw branch: fp32 combined output rows and their LSE.
    {
        const int c4n = a.dim / 4;
        const int64_t pitch = (int64_t)a.raw_rows * a.dim;
        for (int it = tid; it < 16 * c4n; it += 256) {
            const int r = it / c4n, c = (it - r * c4n) * 4;
            int b, l, h, rr;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            float lse = -INFINITY;
            if (row_info(r, b, l, h, rr)) {
                const int p0 = s_parts[r][2], nsp = s_parts[r][3];
                const int64_t row = (int64_t)p0 * a.raw_rows + rr;
                acc = combine_partials(a.raw_o + row * a.dim + c, pitch, a.raw_lse + row, a.raw_rows, nsp, &lse);
            }
            if (c == 0) s_lse[16 + r] = lse;
            *reinterpret_cast<float4*>(s_raw + r * a.dim + c) = acc;
        }
    }
    cp_async_wait_all();
    __syncthreads();
    // 4. [16 x Rvp] . [Rvp x 128] with A = hi + lo: warp -> output columns
    //    [16*warp, 16*warp + 16).
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    const uint32_t hi_base = smem_u32(s_hi), lo_base = smem_u32(s_lo), b_base = smem_u32(s_b);
    const int mi = lane >> 3;
    for (int ks = 0; ks < rvp / 16; ++ks) {
        uint32_t ah[4], al[4];
        const int row = (lane & 7) + (mi & 1) * 8;
        const int unit = (ks & 3) * 2 + (mi >> 1);
        const uint32_t aoff = (ks >> 2) * (16 * 128) + row * 128 + (((unit ^ row) & 7) << 4);
        ldsm_x4(hi_base + aoff, ah[0], ah[1], ah[2], ah[3]);
        ldsm_x4(lo_base + aoff, al[0], al[1], al[2], al[3]);
        const int n = 16 * warp + (mi >> 1) * 8 + (lane & 7);
        const int bunit = (ks & 3) * 2 + (mi & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(b_base + (ks >> 2) * (128 * 128) + n * 128 + (((bunit ^ n) & 7) << 4), b0, b1, b2, b3);
        mma_bf16(acc[0], ah, b0, b1);
        mma_bf16(acc[1], ah, b2, b3);
        mma_bf16(acc[0], al, b0, b1);
        mma_bf16(acc[1], al, b2, b3);
    }
    // 5. Bias, LSE merge (fa2_decode.py:57-66) and store.
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        const int r = (lane >> 2) + 8 * hh;
        int b, l, h, rr;
        if (!row_info(r, b, l, h, rr)) continue;
        const float ll = s_lse[r], lr = s_lse[16 + r];
        float wr = 0.f, wl = 0.f, total = -INFINITY;
        if (!(ll == -INFINITY && lr == -INFINITY)) {
            total = fmaxf(lr, ll) + log1pf(expf(-fabsf(lr - ll)));
            wr = lr == -INFINITY ? 0.f : expf(lr - total);
            wl = ll == -INFINITY ? 0.f : expf(ll - total);
        }
        if (a.out_lse && warp == 0 && (lane & 3) == 0) a.out_lse[((int64_t)b * a.length + l) * a.heads + h] = total;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int d = 16 * warp + nt * 8 + (lane & 3) * 2 + e;
                const float bv = a.uv_bias ? __bfloat162float(a.uv_bias[(int64_t)g * a.dim + d]) : 0.f;
                const float value = wr * s_raw[r * a.dim + d] + wl * (acc[nt][2 * hh + e] + bv);
                const int64_t o = b * a.o_sb + l * a.o_sl + (int64_t)h * a.dim + d;
                if (a.out_fp32) static_cast<float*>(a.out)[o] = value;
                else static_cast<__nv_bfloat16*>(a.out)[o] = __float2bfloat16_rn(value);
            }
    }
}

}  // namespace slimkv
