// Fused SlimKV latent decode step (C ABI slimkv_latent_decode).
//
// Replaces steps 3-8 of the reference `fa2_decode.decode`
// (slimkv/llama3/fa2_decode.py:77-166) with three launches:
//   1. prologue  — BF16-exact RoPE of q (decode_kernels.py:8-51), q-absorb
//                  into Beacon-K latent space (fa2_decode.py:41-46), and the
//                  append of the new raw K (rotated and pre-RoPE) / V and of a
//                  new Beacon latent pair (llama3/memory.py:233-278);
//   2. attention — one launch whose first CTAs stream the latent cache (one
//                  shared latent "head", all H query heads per CTA, causal on
//                  Beacon-insertion rows) and whose remaining CTAs stream the
//                  raw sink+tail per KV head (fa2_decode.py:146-154);
//   3. merge     — split combine of both branches, V up-projection with its
//                  bias (fa2_decode.py:49-54, 157-163), the K-bias LSE shift
//                  and the LSE merge (fa2_decode.py:57-66).
#include <algorithm>

#include "attn_body.cuh"
#include "host_utils.h"
#include "latent_decode_aux.cuh"
#include "latent_tc.h"

namespace slimkv {

int make_bshd_map(CUtensorMap* map, const void* base, int batch, int keys, int kv_heads, int dim,
                  const int64_t stride[3], int* bcast, int box_rows);

// Latent key tile of the split-KV route: 64 keys, 32 for ranks above 320.
constexpr int lat_tile_keys(int width) { return width > 320 ? 32 : kTile; }

// One launch: CTAs [0, n_latent) take latent work items, the rest raw ones.
template <int WL, int MTL>
__global__ void __launch_bounds__(kThreads, 1)
decode_attention_kernel(const __grid_constant__ CUtensorMap lk, const __grid_constant__ CUtensorMap lv,
                        const __grid_constant__ CUtensorMap rk, const __grid_constant__ CUtensorMap rv,
                        AttnJob jl, AttnJob jr, int latent_row_blocks, int n_latent) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    int idx = blockIdx.x;
    if (idx < n_latent) {
        if (threadIdx.x == 0) { tma_prefetch_desc(&lk); tma_prefetch_desc(&lv); }
        jl.kmap = &lk;
        jl.vmap = &lv;
        const int split = idx % jl.splits;
        const int rest = idx / jl.splits;
        attn_body<WL, MTL, kStageBudget, lat_tile_keys(WL)>(jl, rest / latent_row_blocks, 0, split,
                                                            rest % latent_row_blocks, smem);
    } else {
        idx -= n_latent;
        if (threadIdx.x == 0) { tma_prefetch_desc(&rk); tma_prefetch_desc(&rv); }
        jr.kmap = &rk;
        jr.vmap = &rv;
        const int split = idx % jr.splits;
        const int bg = idx / jr.splits;
        attn_body<128, 1>(jr, bg / jr.kv_heads, bg % jr.kv_heads, split, 0, smem);
    }
}

namespace {

struct DecodePlan {
    int wl = 0, mtl = 0, lat_row_blocks = 0, lat_rows = 0, lat_splits = 0, lat_tps = 0;
    int raw_rows = 0, raw_splits = 0, raw_tps = 0, group = 0, rvp = 0;
    bool tc = false;   // both branches on the persistent tensor-memory kernel (32 or 40 query heads)
    bool wide = false; // its 40-head layout (latent ranks <= 512, one query per latent CTA)
    int ctas = 0, raw_ctas = 0, lat_pieces = 0;          // tensor-memory route
    int lat_cover = 0, raw_cover = 0;                    // rows per sequence the launch attends to
    size_t q_rot = 0, q_lat = 0, lat_o = 0, lat_lse = 0, raw_o = 0, raw_lse = 0, plan = 0;
};

// Prologue CTAs resident at once on this device (one wave).
int prologue_wave() {
    static int wave[64] = {};
    const int dev = device_info().device;
    if (dev < 0 || dev >= 64) return 0;
    if (!wave[dev]) {
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_prologue_kernel, 256, 0) != cudaSuccess)
            per_sm = 1;
        wave[dev] = std::max(per_sm, 1) * std::max(device_info().sm_count, 1);
    }
    return wave[dev];
}

int plan_decode(const slimkv_latent_decode_args* a, DecodePlan& p) {
    if (!a) return fail(SLIMKV_ERR_INVALID_ARGUMENT, "null arguments");
    if (a->batch <= 0 || a->heads <= 0 || a->kv_heads <= 0 || a->heads % a->kv_heads)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "invalid head counts");
    if (a->length != 1 && a->length != 2) return fail(SLIMKV_ERR_INVALID_ARGUMENT, "length must be 1 or 2");
    if (a->head_dim != 128) return fail(SLIMKV_ERR_UNSUPPORTED_SHAPE, "fused decode needs head_dim 128");
    if (a->rank_k <= 0 || a->rank_k > 512 || a->rank_k % 8 || a->rank_v <= 0 || a->rank_v > 512 || a->rank_v % 8)
        return fail(SLIMKV_ERR_UNSUPPORTED_SHAPE, "latent ranks must be multiples of 8 in [8, 512]");
    if (a->raw_capacity <= 0 || a->lat_capacity <= 0) return fail(SLIMKV_ERR_INVALID_ARGUMENT, "empty cache");
    p.group = a->heads / a->kv_heads;
    if (p.group * a->length > kMaxRows)
        return fail(SLIMKV_ERR_UNSUPPORTED_SHAPE, "at most %d query rows per KV head", kMaxRows);
    p.wl = (std::max(a->rank_k, a->rank_v) + 63) / 64 * 64;
    p.wl = std::max(p.wl, 128);
    if (p.wl > 320) p.wl = 512;                  // one wide instantiation (32-key tiles)
    p.rvp = (a->rank_v + 63) / 64 * 64;
    const int lat_rows = a->heads * a->length;
    p.mtl = lat_rows <= 32 ? 2 : 4;
    p.lat_row_blocks = (lat_rows + 16 * p.mtl - 1) / (16 * p.mtl);
    p.lat_rows = p.lat_row_blocks * 16 * p.mtl;
    p.raw_rows = 16;
    const int lat_len = a->latent_len_max > 0 ? std::min(a->latent_len_max, a->lat_capacity) : a->lat_capacity;
    const int raw_len = a->raw_len_max > 0 ? std::min(a->raw_len_max, a->raw_capacity) : a->raw_capacity;
    const int lt = lat_tile_keys(p.wl);
    const int lat_tiles = std::max(1, (lat_len + lt - 1) / lt);
    const int raw_tiles = std::max(1, (raw_len + kTile - 1) / kTile);
    // Balance bytes: one CTA per SM, each streaming about the same volume.
    const double lat_tile_bytes = double(lt) * (a->rank_k + a->rank_v) * 2;
    const double raw_tile_bytes = double(kTile) * a->head_dim * 2 * 2;
    const double total = a->batch * (p.lat_row_blocks * lat_tiles * lat_tile_bytes +
                                     a->kv_heads * raw_tiles * raw_tile_bytes);
    const double per_cta = total / std::max(device_info().sm_count, 1);
    int ls = a->latent_splits > 0 ? a->latent_splits
                                  : int(std::ceil(lat_tiles * lat_tile_bytes / std::max(per_cta, 1.0)));
    int rs = a->raw_splits > 0 ? a->raw_splits : int(std::ceil(raw_tiles * raw_tile_bytes / std::max(per_cta, 1.0)));
    // The merge kernel combines at most kMergeMaxSplits splits per branch.
    ls = std::max(1, std::min({ls, lat_tiles, kMergeMaxSplits}));
    rs = std::max(1, std::min({rs, raw_tiles, kMergeMaxSplits}));
    p.lat_tps = (lat_tiles + ls - 1) / ls;
    p.lat_splits = (lat_tiles + p.lat_tps - 1) / p.lat_tps;
    p.raw_tps = (raw_tiles + rs - 1) / rs;
    p.raw_splits = (raw_tiles + p.raw_tps - 1) / p.raw_tps;
    p.lat_cover = std::min(a->lat_capacity, p.lat_splits * p.lat_tps * lt);
    p.raw_cover = std::min(a->raw_capacity, p.raw_splits * p.raw_tps * kTile);
    const size_t B = a->batch, L = a->length, H = a->heads;
    // 8: the raw score columns per query.  The 40-head layout cycles V
    // chunk pairs through a ring: an even number of 64-column V chunks.
    p.wide = a->heads == kTcWideHeads && p.wl <= 512 && p.group <= 8 && ((a->rank_v + 63) / 64) % 2 == 0;
    p.tc = (a->heads == kTcHeads && p.wl <= 320 && p.group <= 8) || p.wide;
    if (p.tc) {
        // One persistent launch: CTAs (at most one per SM) split the latent and
        // raw work by volume on the device (latent_tc_plan.cuh).  latent_splits
        // and raw_splits, when given, set the CTA count of the launch and of
        // the raw class.
        const int sms = std::max(device_info().sm_count, 1);
        const int cap = std::min({sms, kMergeMaxSplits - 1, kTcMaxCtas});
        p.ctas = std::max(3, std::min(a->latent_splits > 0 ? a->latent_splits : sms, cap));
        p.raw_ctas = a->raw_splits > 0 ? std::min(a->raw_splits, p.ctas - 2) : 0;
        p.lat_rows = 2 * a->heads;
        p.raw_rows = 2 * p.group;
        p.lat_pieces = tc_max_pieces(p.wide ? 2 * a->batch : a->batch, p.ctas);
        // The device plan tiles every sequence to its own length.
        p.lat_cover = a->lat_capacity;
        p.raw_cover = a->raw_capacity;
    }
    p.q_rot = B * L * H * a->head_dim;
    p.q_lat = p.tc ? B * (p.wide ? kTcWideRows : 128) * p.wl : B * L * H * p.wl;
    if (p.tc) {
        const size_t raw_pieces = tc_max_pieces(a->batch * a->kv_heads, p.ctas);
        p.plan = tc_plan_layout(a->batch, a->kv_heads, p.wide).words;
        p.lat_o = 2 * size_t(p.lat_pieces) * p.lat_rows * p.wl;
        p.lat_lse = 2 * size_t(p.lat_pieces) * p.lat_rows;
        p.raw_o = raw_pieces * p.raw_rows * 128;
        p.raw_lse = raw_pieces * p.raw_rows;
    } else {
        p.lat_o = B * p.lat_splits * p.lat_rows * p.wl;
        p.lat_lse = B * p.lat_splits * p.lat_rows;
        p.raw_o = B * a->kv_heads * p.raw_splits * p.raw_rows * 128;
        p.raw_lse = B * a->kv_heads * p.raw_splits * p.raw_rows;
    }
    return SLIMKV_OK;
}

struct Buffers {
    __nv_bfloat16* q_rot;
    __half* q_lat;
    float *lat_o, *lat_lse, *raw_o, *raw_lse;
    int32_t* plan;          // tensor-memory route: the device plan (latent_tc.h)
};

Buffers carve(Carver& c, const DecodePlan& p) {
    Buffers w;
    w.q_rot = c.take<__nv_bfloat16>(p.q_rot);
    w.q_lat = c.take<__half>(p.q_lat);
    w.lat_o = c.take<float>(p.lat_o);
    w.lat_lse = c.take<float>(p.lat_lse);
    w.raw_o = c.take<float>(p.raw_o);
    w.raw_lse = c.take<float>(p.raw_lse);
    w.plan = c.take<int32_t>(p.plan);
    return w;
}

template <int WL, int MTL>
int launch_decode_attention(const CUtensorMap& lk, const CUtensorMap& lv, const CUtensorMap& rk,
                            const CUtensorMap& rv, const AttnJob& jl, const AttnJob& jr, int row_blocks,
                            int n_latent, int n_raw, cudaStream_t stream) {
    constexpr int smem = std::max(AttnCfg<WL, MTL, kStageBudget, lat_tile_keys(WL)>::SMEM, AttnCfg<128, 1>::SMEM);
    auto kernel = decode_attention_kernel<WL, MTL>;
    static bool configured[64] = {};
    const int dev = device_info().device;
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
            return fail(SLIMKV_ERR_CUDA, "cudaFuncSetAttribute failed");
        configured[dev] = true;
    }
    kernel<<<n_latent + n_raw, kThreads, smem, stream>>>(lk, lv, rk, rv, jl, jr, row_blocks, n_latent);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(SLIMKV_ERR_CUDA, "decode attention launch failed: %s", cudaGetErrorString(e));
    return SLIMKV_OK;
}

template <int WL>
int launch_wl(int mtl, const CUtensorMap& lk, const CUtensorMap& lv, const CUtensorMap& rk, const CUtensorMap& rv,
              const AttnJob& jl, const AttnJob& jr, int rb, int nl, int nr, cudaStream_t s) {
    if (mtl == 2) return launch_decode_attention<WL, 2>(lk, lv, rk, rv, jl, jr, rb, nl, nr, s);
    return launch_decode_attention<WL, 4>(lk, lv, rk, rv, jl, jr, rb, nl, nr, s);
}

}  // namespace
}  // namespace slimkv

using namespace slimkv;

extern "C" size_t slimkv_latent_decode_workspace_size(const slimkv_latent_decode_args* a) {
    DecodePlan p;
    if (plan_decode(a, p) != SLIMKV_OK) return 0;
    Carver c(nullptr, 0);
    carve(c, p);
    return c.used + 256;
}

extern "C" int slimkv_latent_decode(const slimkv_latent_decode_args* a, void* workspace, size_t workspace_bytes,
                                    void* stream_ptr) {
    DecodePlan p;
    int rc = plan_decode(a, p);
    if (rc) return rc;
    const bool paged = a->lat_pages != nullptr;
    if (!a->q || !a->raw_k_rot || !a->raw_v || (!paged && (!a->lat_k || !a->lat_v)) || !a->raw_len ||
        !a->latent_len || !a->qpos || !a->uk || !a->uv || !a->cos || !a->sin || !a->out)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if ((a->new_k == nullptr) != (a->new_v == nullptr) || (a->new_lat_k == nullptr) != (a->new_lat_v == nullptr))
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "new K/V (and new latent K/V) must be given together");
    if (a->latent_shard && a->new_lat_k)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "a latent shard without this step's Beacon takes no new latents");
    if (a->raw_stride_token % 8 || a->raw_stride_batch % 8 || !aligned16(a->raw_k_rot) || !aligned16(a->raw_v) ||
        !aligned16(a->uv) ||
        (!paged && (a->lat_stride_row % 8 || a->lat_stride_batch % 8 || !aligned16(a->lat_k) || !aligned16(a->lat_v))))
        return fail(SLIMKV_ERR_ALIGNMENT, "caches must be 16-byte aligned with strides that are multiples of 8");
    const int64_t raw_sh = a->raw_stride_head > 0 ? a->raw_stride_head : a->head_dim;
    // Token-major [B, cap, Hkv, D] (head stride D) or head-major [B, Hkv, cap, D]
    // (token stride D): either way the rows of different heads and tokens must
    // not overlap.
    const bool token_major = raw_sh == a->head_dim && a->raw_stride_token >= (int64_t)a->kv_heads * a->head_dim;
    const bool head_major = a->raw_stride_token == a->head_dim && raw_sh >= (int64_t)a->raw_capacity * a->head_dim;
    if (raw_sh % 8 || !(token_major || head_major))
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "raw caches must be token-major [B, cap, Hkv, D] or head-major "
                                                 "[B, Hkv, cap, D] (strides multiples of 8)");
    if (!paged && a->lat_stride_row < std::max(a->rank_k, a->rank_v))
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "cache row stride smaller than a row");
    if (paged) {
        if (!p.tc) return fail(SLIMKV_ERR_UNSUPPORTED_SHAPE, "paged latent caches need 32 or 40 query heads");
        if (!a->lat_table || a->lat_slots <= 0 || a->lat_slots % 16 || a->lat_num_pages <= 0 ||
            a->lat_table_stride <= 0 || a->lat_sink_elements < 0 || a->lat_sink_elements % 8 ||
            a->lat_page_stride % 8 || !aligned16(a->lat_pages) ||
            a->lat_page_stride < a->lat_sink_elements + int64_t(a->lat_slots) * (a->rank_k + a->rank_v))
            return fail(SLIMKV_ERR_INVALID_ARGUMENT,
                        "paged latent cache: need a block table, slots a multiple of 16, 16-byte aligned pages");
        if (int64_t(a->lat_capacity) > a->lat_table_stride * a->lat_slots)
            return fail(SLIMKV_ERR_INVALID_ARGUMENT, "lat_capacity exceeds the rows the block table can address");
    }
    Carver c(workspace, workspace_bytes);
    const Buffers w = carve(c, p);
    if (!workspace || !c.fits())
        return fail(SLIMKV_ERR_WORKSPACE, "workspace too small (%zu < %zu)", workspace_bytes, c.used);
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    unsigned int* status = status_word();

    // 1. prologue
    if (!aligned16(a->uk) || !aligned16(a->q) || a->q_stride[0] % 8 || a->q_stride[1] % 8 || a->q_stride[2] % 8)
        return fail(SLIMKV_ERR_ALIGNMENT, "q and U_k must be 16-byte aligned with strides that are multiples of 8");
    if ((a->new_k && (a->new_stride % 8 || !aligned16(a->new_k) || !aligned16(a->new_v))) ||
        (a->new_lat_k && (a->new_lat_stride % 8 || !aligned16(a->new_lat_k) || !aligned16(a->new_lat_v))))
        return fail(SLIMKV_ERR_ALIGNMENT, "new rows must be 16-byte aligned with strides that are multiples of 8");
    const int rps = a->length * p.group;
    PrologueArgs pa{};
    pa.q = static_cast<const __nv_bfloat16*>(a->q);
    pa.q_sb = a->q_stride[0]; pa.q_sl = a->q_stride[1]; pa.q_sh = a->q_stride[2];
    pa.batch = a->batch; pa.length = a->length; pa.heads = a->heads; pa.kv_heads = a->kv_heads;
    pa.dim = a->head_dim; pa.rank_k = a->rank_k; pa.rank_v = a->rank_v; pa.width = p.wl; pa.group = p.group;
    // About 16 query rows per CTA: enough CTAs to spread the staging loads
    // over the machine (the MMA tile still has 64 rows; unused rows are zero).
    pa.seq_per_cta = std::max(1, std::min(kProRows / rps, 16 / rps));
    pa.qpos = a->qpos; pa.qlens = a->query_len; pa.cos = a->cos; pa.sin = a->sin;
    pa.rope_positions = a->rope_positions;
    pa.uk = static_cast<const __nv_bfloat16*>(a->uk);
    pa.q_rot = w.q_rot; pa.q_lat = w.q_lat;
    pa.q_hilo = reinterpret_cast<__nv_bfloat16*>(w.q_lat); pa.hilo = p.tc ? 1 : 0;
    pa.hilo_rows = p.wide ? kTcWideRows : 128; pa.hilo_split = p.wide ? 1 : 0;
    pa.new_k = static_cast<const __nv_bfloat16*>(a->new_k);
    pa.new_v = static_cast<const __nv_bfloat16*>(a->new_v);
    pa.new_stride = a->new_stride > 0 ? a->new_stride : (int64_t)a->kv_heads * a->head_dim;
    pa.raw_k_rot = static_cast<__nv_bfloat16*>(a->raw_k_rot);
    pa.raw_v = static_cast<__nv_bfloat16*>(a->raw_v);
    pa.raw_k_pre = static_cast<__nv_bfloat16*>(a->raw_k_pre);
    pa.raw_sb = a->raw_stride_batch; pa.raw_st = a->raw_stride_token; pa.raw_sh = raw_sh;
    pa.raw_len = a->raw_len; pa.raw_capacity = a->raw_capacity;
    pa.new_lat_k = static_cast<const __nv_bfloat16*>(a->new_lat_k);
    pa.new_lat_v = static_cast<const __nv_bfloat16*>(a->new_lat_v);
    if (a->new_lat_k && a->new_lat_stride <= 0 && a->rank_k != a->rank_v)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "new_lat_stride is required when the ranks differ");
    pa.new_lat_stride = a->new_lat_stride > 0 ? a->new_lat_stride : a->rank_k;
    pa.lat_k = static_cast<__nv_bfloat16*>(a->lat_k);
    pa.lat_v = static_cast<__nv_bfloat16*>(a->lat_v);
    pa.lat_sb = a->lat_stride_batch; pa.lat_sr = a->lat_stride_row;
    pa.latent_len = a->latent_len; pa.lat_capacity = a->lat_capacity;
    pa.lat_cover = p.lat_cover; pa.raw_cover = p.raw_cover;
    pa.lat_pages = static_cast<__nv_bfloat16*>(a->lat_pages);
    pa.lat_page_stride = a->lat_page_stride; pa.lat_table_stride = a->lat_table_stride;
    pa.lat_slots = a->lat_slots; pa.lat_sink = a->lat_sink_elements; pa.lat_num_pages = a->lat_num_pages;
    pa.lat_table = a->lat_table;
    int32_t* plan = a->plan ? const_cast<int32_t*>(a->plan) : w.plan;
    if (p.tc) {
        pa.do_plan = a->plan ? 0 : 1;
        TcPlanArgs& pl = pa.plan;
        pl.batch = a->batch; pl.kv_heads = a->kv_heads; pl.length = a->length;
        pl.latent_len = a->latent_len; pl.raw_len = a->raw_len; pl.query_len = a->query_len;
        pl.lat_chunks = (a->rank_k + 63) / 64 + (a->rank_v + 63) / 64;
        pl.ctas = p.ctas; pl.raw_ctas = p.raw_ctas; pl.with_raw = 1; pl.plan = plan;
        pl.split_queries = p.wide ? 1 : 0;
    }
    pa.status = status;
    const dim3 pgrid(a->kv_heads, p.wl / 64, (a->batch + pa.seq_per_cta - 1) / pa.seq_per_cta + (p.tc ? 1 : 0));
    decode_prologue_kernel<<<pgrid, 256, 0, stream>>>(pa);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(SLIMKV_ERR_CUDA, "prologue launch failed: %s", cudaGetErrorString(e));

    // 2. attention over both branches
    CUtensorMap lk, lv, rk, rv;     // maps of the split-KV route (the tensor-core route builds its own)
    if (!p.tc) {
        int bc = 0;
        const int64_t lat_stride[3] = {a->lat_stride_batch, a->lat_stride_row, a->lat_stride_row};
        const int lt = lat_tile_keys(p.wl);
        if ((rc = make_bshd_map(&lk, a->lat_k, a->batch, a->lat_capacity, 1, a->rank_k, lat_stride, &bc, lt)))
            return rc;
        if ((rc = make_bshd_map(&lv, a->lat_v, a->batch, a->lat_capacity, 1, a->rank_v, lat_stride, &bc, lt)))
            return rc;
        const int64_t raw_stride[3] = {a->raw_stride_batch, a->raw_stride_token, raw_sh};
        if ((rc = make_bshd_map(&rk, a->raw_k_rot, a->batch, a->raw_capacity, a->kv_heads, a->head_dim, raw_stride,
                                &bc, kTile)))
            return rc;
        if ((rc = make_bshd_map(&rv, a->raw_v, a->batch, a->raw_capacity, a->kv_heads, a->head_dim, raw_stride,
                                &bc, kTile)))
            return rc;
    }
    const float scale_log2 = a->scale * 1.4426950408889634f;
    AttnJob jl{};
    jl.q = w.q_lat; jl.q_fp16 = 1; jl.q_sb = (int64_t)a->length * a->heads * p.wl; jl.q_sl = (int64_t)a->heads * p.wl; jl.q_sh = p.wl;
    jl.seqlens = a->latent_len; jl.keys = a->lat_capacity; jl.qlens = a->query_len; jl.queries = a->length;
    jl.group = a->heads; jl.kv_heads = 1; jl.dk = a->rank_k; jl.scale_log2 = scale_log2;
    jl.causal = a->latent_shard ? 0 : 1;
    jl.splits = p.lat_splits; jl.tiles_per_split = p.lat_tps; jl.rows_alloc = p.lat_rows; jl.out_width = p.wl;
    jl.part_o = w.lat_o; jl.part_lse = w.lat_lse; jl.status = status;
    AttnJob jr{};
    jr.q = w.q_rot; jr.q_fp16 = 0; jr.q_sb = (int64_t)a->length * a->heads * a->head_dim; jr.q_sl = (int64_t)a->heads * a->head_dim;
    jr.q_sh = a->head_dim;
    jr.seqlens = a->raw_len; jr.keys = a->raw_capacity; jr.qlens = a->query_len; jr.queries = a->length;
    jr.group = p.group; jr.kv_heads = a->kv_heads; jr.dk = a->head_dim; jr.scale_log2 = scale_log2; jr.causal = 0;
    jr.splits = p.raw_splits; jr.tiles_per_split = p.raw_tps; jr.rows_alloc = p.raw_rows; jr.out_width = 128;
    jr.part_o = w.raw_o; jr.part_lse = w.raw_lse; jr.status = status;
    const int n_raw = a->batch * a->kv_heads * p.raw_splits;
    if (p.tc) {
        // Both branches in one launch of the tensor-core kernel.
        TcLaunch tl{};
        tl.batch = a->batch; tl.length = a->length; tl.scale = a->scale;
        tl.query_len = a->query_len; tl.status = status; tl.with_raw = 1;
        tl.kv_heads = a->kv_heads; tl.ctas = p.ctas; tl.plan = plan; tl.lat_pieces = p.lat_pieces;
        tl.wide = p.wide ? 1 : 0;
        tl.wait_ns = a->wait_limit_ns;
        // With the plan ready the attention may start before the prologue
        // ends — not when its duration is being timed (the begin event would
        // come after its start).
        // Only for a prologue of at most three waves: with more, the early
        // attention CTAs hold whole SMs while the prologue drains (config 3,
        // 4.2 waves: 1132 us against 903 us started after it; config 5, 2.85
        // waves, still gains 2 % from the early start).
        tl.early = a->plan && !a->attn_event_begin && int(pgrid.x * pgrid.y * pgrid.z) <= 3 * prologue_wave() ? 1 : 0;
        TcSide& L = tl.lat;
        L.k = a->lat_k; L.v = a->lat_v; L.dim_k = a->rank_k; L.dim_v = a->rank_v;
        L.kv_heads = 1; L.capacity = a->lat_capacity;
        L.stride_batch = a->lat_stride_batch; L.stride_row = a->lat_stride_row; L.stride_head = 0;
        L.q = w.q_lat; L.q_rows = 0; L.heads = a->heads; L.group = a->heads; L.causal = a->latent_shard ? 0 : 1;
        L.seqlens = a->latent_len; L.rows_alloc = p.lat_rows; L.width = p.wl;
        L.part_o = w.lat_o; L.part_lse = w.lat_lse;
        L.pages = a->lat_pages; L.page_stride = a->lat_page_stride; L.slots = a->lat_slots;
        L.sink_elements = a->lat_sink_elements; L.num_pages = a->lat_num_pages;
        L.table = a->lat_table; L.table_stride = a->lat_table_stride;
        TcSide& R = tl.raw;
        R.k = a->raw_k_rot; R.v = a->raw_v; R.dim_k = a->head_dim; R.dim_v = a->head_dim;
        R.kv_heads = a->kv_heads; R.capacity = a->raw_capacity;
        R.stride_batch = a->raw_stride_batch; R.stride_row = a->raw_stride_token; R.stride_head = raw_sh;
        R.q = w.q_rot; R.q_rows = 1; R.heads = a->heads; R.group = p.group; R.causal = 0;
        R.seqlens = a->raw_len; R.rows_alloc = p.raw_rows; R.width = a->head_dim;
        R.part_o = w.raw_o; R.part_lse = w.raw_lse;
        if (a->attn_event_begin && cudaEventRecord(static_cast<cudaEvent_t>(a->attn_event_begin), stream) != cudaSuccess)
            return fail(SLIMKV_ERR_CUDA, "attn_event_begin record failed");
        if ((rc = launch_decode_tc(tl, stream))) return rc;
        if (a->attn_event_end && cudaEventRecord(static_cast<cudaEvent_t>(a->attn_event_end), stream) != cudaSuccess)
            return fail(SLIMKV_ERR_CUDA, "attn_event_end record failed");
    } else {
    const int n_latent = a->batch * p.lat_row_blocks * p.lat_splits;
    if (a->attn_event_begin && cudaEventRecord(static_cast<cudaEvent_t>(a->attn_event_begin), stream) != cudaSuccess)
        return fail(SLIMKV_ERR_CUDA, "attn_event_begin record failed");
    switch (p.wl) {
        case 128: rc = launch_wl<128>(p.mtl, lk, lv, rk, rv, jl, jr, p.lat_row_blocks, n_latent, n_raw, stream); break;
        case 192: rc = launch_wl<192>(p.mtl, lk, lv, rk, rv, jl, jr, p.lat_row_blocks, n_latent, n_raw, stream); break;
        case 256: rc = launch_wl<256>(p.mtl, lk, lv, rk, rv, jl, jr, p.lat_row_blocks, n_latent, n_raw, stream); break;
        case 320: rc = launch_wl<320>(p.mtl, lk, lv, rk, rv, jl, jr, p.lat_row_blocks, n_latent, n_raw, stream); break;
        default: rc = launch_wl<512>(p.mtl, lk, lv, rk, rv, jl, jr, p.lat_row_blocks, n_latent, n_raw, stream); break;
    }
    if (rc) return rc;
    if (a->attn_event_end && cudaEventRecord(static_cast<cudaEvent_t>(a->attn_event_end), stream) != cudaSuccess)
        return fail(SLIMKV_ERR_CUDA, "attn_event_end record failed");
    }

    // 3. merge
    MergeArgs ma{};
    ma.lat_o = w.lat_o; ma.lat_lse = w.lat_lse; ma.lat_splits = p.lat_splits; ma.lat_rows = p.lat_rows;
    ma.lat_width = p.wl;
    if (p.tc) {
        ma.plan = plan;
        ma.PL = tc_plan_layout(a->batch, a->kv_heads, p.wide);
        ma.lat_pieces = p.lat_pieces;
    }
    ma.raw_o = w.raw_o; ma.raw_lse = w.raw_lse; ma.raw_splits = p.raw_splits; ma.raw_rows = p.raw_rows;
    ma.raw_l_pitch = p.group;
    ma.q_rot = w.q_rot;
    ma.uv = static_cast<const __nv_bfloat16*>(a->uv);
    ma.uk_bias = static_cast<const __nv_bfloat16*>(a->uk_bias);
    ma.uv_bias = static_cast<const __nv_bfloat16*>(a->uv_bias);
    ma.qlens = a->query_len; ma.batch = a->batch; ma.length = a->length; ma.heads = a->heads;
    ma.kv_heads = a->kv_heads; ma.dim = a->head_dim; ma.rank_v = a->rank_v; ma.rank_v_pad = p.rvp;
    ma.group = p.group; ma.scale = a->scale;
    // Merge CTAs: one per (KV head, sequence), its rows split over two CTAs
    // while that still fits one wave (two merge CTAs per SM); for a batch
    // larger than that, as many sequences per CTA as fill its 16 rows.
    {
        const int sms = std::max(device_info().sm_count, 1);
        const int rps_m = a->length * p.group;
        ma.seq_per_cta = a->kv_heads * a->batch <= sms ? 1 : std::max(1, 16 / rps_m);
    }
    ma.out = a->out; ma.out_fp32 = a->out_fp32; ma.o_sb = a->out_stride[0]; ma.o_sl = a->out_stride[1];
    ma.out_lse = a->out_lse;
    const size_t msmem = merge_smem_bytes(p.rvp, a->head_dim);
    {
        static bool configured[64] = {};
        const int dev = device_info().device;
        if (dev >= 0 && dev < 64 && !configured[dev]) {
            if (cudaFuncSetAttribute(decode_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     int(merge_smem_bytes(512, 128))) != cudaSuccess)
                return fail(SLIMKV_ERR_CUDA, "cudaFuncSetAttribute failed");
            configured[dev] = true;
        }
    }
    const int units = a->kv_heads * ((a->batch + ma.seq_per_cta - 1) / ma.seq_per_cta);
    const int row_split = ma.seq_per_cta == 1 && units <= std::max(device_info().sm_count, 1) ? 2 : 1;
    const dim3 mgrid(a->kv_heads, (a->batch + ma.seq_per_cta - 1) / ma.seq_per_cta, row_split);
    // Programmatic dependent launch: the merge's set-up (plan ranges, U_v,
    // LSE shifts) overlaps the attention launch's last CTAs; it reads the
    // partials only after the attention grid has completed.
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = mgrid;
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = msmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, decode_merge_kernel, ma);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return fail(SLIMKV_ERR_CUDA, "merge launch failed: %s", cudaGetErrorString(e));
    return SLIMKV_OK;
}

namespace slimkv {
namespace {

// One block: the step plan of the tensor-core route (plan_tc_work), built in
// this block's shared memory when it fits.
__global__ void __launch_bounds__(256) decode_plan_kernel(TcPlanArgs pl) {
    __shared__ int32_t scratch[8192];
    plan_tc_work(pl, scratch, 8192);
}

}  // namespace
}  // namespace slimkv

extern "C" size_t slimkv_decode_plan_words(const slimkv_latent_decode_args* a) {
    DecodePlan p;
    if (plan_decode(a, p) != SLIMKV_OK) return 0;
    return p.tc ? size_t(tc_plan_layout(a->batch, a->kv_heads, p.wide).words) : 1;
}

extern "C" int slimkv_decode_plan(const slimkv_latent_decode_args* a, int32_t* plan, void* stream_ptr) {
    DecodePlan p;
    if (int rc = plan_decode(a, p)) return rc;
    if (!p.tc) return SLIMKV_OK;                    // the split-KV route plans on the host
    if (!plan || !a->raw_len || !a->latent_len)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "decode plan: null plan or length pointer");
    TcPlanArgs pl{};
    pl.batch = a->batch; pl.kv_heads = a->kv_heads; pl.length = a->length;
    pl.latent_len = a->latent_len; pl.raw_len = a->raw_len; pl.query_len = a->query_len;
    pl.lat_chunks = (a->rank_k + 63) / 64 + (a->rank_v + 63) / 64;
    pl.ctas = p.ctas; pl.raw_ctas = p.raw_ctas; pl.with_raw = 1; pl.plan = plan;
    pl.split_queries = p.wide ? 1 : 0;
    decode_plan_kernel<<<1, 256, 0, static_cast<cudaStream_t>(stream_ptr)>>>(pl);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(SLIMKV_ERR_CUDA, "decode plan launch failed: %s", cudaGetErrorString(e));
    return SLIMKV_OK;
}
