// Drop-in split-KV decode attention: the C ABI behind the Python module that
// replaces the reference's `slimkv_fa2_decode_320.forward`
// (kernels/fa2_decode/binding.cpp:35-121).
#include <algorithm>
#include <mutex>

#include "attn_body.cuh"
#include "host_utils.h"

namespace slimkv {

template <int W, int MT>
__global__ void __launch_bounds__(kThreads, 1)
attention_split_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                       AttnJob job) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    if (threadIdx.x == 0) {
        tma_prefetch_desc(&kmap);
        tma_prefetch_desc(&vmap);
    }
    job.kmap = &kmap;
    job.vmap = &vmap;
    const int bg = blockIdx.y;
    attn_body<W, MT>(job, bg / job.kv_heads, bg % job.kv_heads, blockIdx.x, blockIdx.z, smem);
}

// Merge split partials into the final output and LSE (one warp per row).
// Lane s holds split s's LSE and weight; each split's columns are then read
// with independent loads.
__global__ void __launch_bounds__(256)
attention_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse, int splits,
                         int rows_alloc, int width, int rows_total, int group, int kv_heads, int value_dim,
                         void* __restrict__ out, int out_fp32, int64_t o_sb, int64_t o_sl, int64_t o_sh,
                         float* __restrict__ lse_out, int heads, int queries, float masked_lse) {
    const int bg = blockIdx.x;
    const int b = bg / kv_heads, g = bg % kv_heads;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.y * 8 + warp;
    if (row >= rows_total) return;
    const int64_t base = (int64_t)bg * splits * rows_alloc + row;
    const int l = row / group, h = g * group + (row - l * group);
    const int64_t off = b * o_sb + l * o_sl + h * o_sh;
    auto store = [&](int d, float x) {
        if (out_fp32) static_cast<float*>(out)[off + d] = x;
        else static_cast<__nv_bfloat16*>(out)[off + d] = __float2bfloat16_rn(x);
    };
    // splits <= 128: each lane owns up to four splits
    float my[4], m = -INFINITY;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int s = lane + 32 * j;
        my[j] = s < splits ? part_lse[base + (int64_t)s * rows_alloc] : -INFINITY;
        m = fmaxf(m, my[j]);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (m == -INFINITY) {
        for (int d = lane; d < value_dim; d += 32) store(d, 0.f);
        if (lane == 0) lse_out[((int64_t)b * heads + h) * queries + l] = masked_lse;
        return;
    }
    float w[4], total = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        w[j] = my[j] == -INFINITY ? 0.f : expf(my[j] - m);
        total += w[j];
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
    const float inv = 1.f / total;
    for (int d0 = 0; d0 < value_dim; d0 += 32 * 4) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int s = 0; s < splits; ++s) {
            const float ws = __shfl_sync(0xffffffffu, w[s >> 5], s & 31);
            const float* src = part_o + (base + (int64_t)s * rows_alloc) * width;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int d = d0 + lane + 32 * i;
                if (d < value_dim) acc[i] = fmaf(ws, src[d], acc[i]);
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int d = d0 + lane + 32 * i;
            if (d < value_dim) store(d, acc[i] * inv);
        }
    }
    if (lane == 0) lse_out[((int64_t)b * heads + h) * queries + l] = m + logf(total);
}

namespace {

struct Plan {
    int width = 0, mt = 0, row_blocks = 0, rows_alloc = 0, splits = 0, tiles_per_split = 0;
    size_t part_o = 0, part_lse = 0;
};

int pick_width(int d) {
    int w = (d + 63) / 64 * 64;
    return w;
}

int plan_attention(const slimkv_attention_args* a, Plan& p) {
    if (!a) return fail(SLIMKV_ERR_INVALID_ARGUMENT, "null arguments");
    if (a->batch <= 0 || a->heads <= 0 || a->kv_heads <= 0 || a->heads % a->kv_heads)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "invalid GQA head counts");
    if (a->queries != 1 && a->queries != 2)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "decode supports one or two queries");
    if (a->keys <= 0) return fail(SLIMKV_ERR_INVALID_ARGUMENT, "empty key range");
    if (a->head_dim <= 0 || a->head_dim > 320 || a->head_dim % 8 || a->value_dim <= 0 ||
        a->value_dim > 320 || a->value_dim % 8)
        return fail(SLIMKV_ERR_UNSUPPORTED_SHAPE, "widths must be multiples of 8 in [8, 320]");
    p.width = pick_width(std::max(a->head_dim, a->value_dim));
    const int group = a->heads / a->kv_heads;
    const int rows = group * a->queries;
    p.mt = rows <= 16 ? 1 : rows <= 32 ? 2 : 4;
    p.row_blocks = (rows + 16 * p.mt - 1) / (16 * p.mt);
    p.rows_alloc = p.row_blocks * 16 * p.mt;
    const int n_tiles = (a->keys + kTile - 1) / kTile;
    const int base = a->batch * a->kv_heads * p.row_blocks;
    int splits = a->num_splits;
    if (splits <= 0) {
        // One resident CTA per SM (shared memory bound): fill one wave.
        const int sms = std::max(device_info().sm_count, 1);
        splits = std::max(1, sms / base);
    }
    splits = std::max(1, std::min({splits, n_tiles, 128}));   // the combine handles <= 128 splits
    p.tiles_per_split = (n_tiles + splits - 1) / splits;
    p.splits = (n_tiles + p.tiles_per_split - 1) / p.tiles_per_split;
    p.part_o = (size_t)a->batch * a->kv_heads * p.splits * p.rows_alloc * p.width;
    p.part_lse = (size_t)a->batch * a->kv_heads * p.splits * p.rows_alloc;
    return SLIMKV_OK;
}

template <int W, int MT>
int launch_split(const CUtensorMap& km, const CUtensorMap& vm, const AttnJob& job, dim3 grid,
                 cudaStream_t stream) {
    constexpr int smem = AttnCfg<W, MT>::SMEM;
    auto kernel = attention_split_kernel<W, MT>;
    static bool configured[64] = {};
    const int dev = device_info().device;
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
            return fail(SLIMKV_ERR_CUDA, "cudaFuncSetAttribute failed");
        configured[dev] = true;
    }
    kernel<<<grid, kThreads, smem, stream>>>(km, vm, job);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(SLIMKV_ERR_CUDA, "attention launch failed: %s", cudaGetErrorString(e));
    return SLIMKV_OK;
}

template <int W>
int launch_width(int mt, const CUtensorMap& km, const CUtensorMap& vm, const AttnJob& job, dim3 grid,
                 cudaStream_t stream) {
    switch (mt) {
        case 1: return launch_split<W, 1>(km, vm, job, grid, stream);
        case 2: return launch_split<W, 2>(km, vm, job, grid, stream);
        default: return launch_split<W, 4>(km, vm, job, grid, stream);
    }
}

}  // namespace

int launch_attention_job(int width, int mt, const CUtensorMap& km, const CUtensorMap& vm, const AttnJob& job,
                         dim3 grid, cudaStream_t stream) {
    switch (width) {
        case 64: return launch_width<64>(mt, km, vm, job, grid, stream);
        case 128: return launch_width<128>(mt, km, vm, job, grid, stream);
        case 192: return launch_width<192>(mt, km, vm, job, grid, stream);
        case 256: return launch_width<256>(mt, km, vm, job, grid, stream);
        case 320: return launch_width<320>(mt, km, vm, job, grid, stream);
        default: return fail(SLIMKV_ERR_UNSUPPORTED_SHAPE, "unsupported padded width %d", width);
    }
}

// Tensor map over a BSHD cache view [B, N, Hkv, D] with element strides
// {sb, sn, sh}; a zero batch stride maps one shared batch.
int make_bshd_map(CUtensorMap* map, const void* base, int batch, int keys, int kv_heads, int dim,
                  const int64_t stride[3], int* bcast, int box_rows) {
    if (!aligned16(base)) return fail(SLIMKV_ERR_ALIGNMENT, "K/V base pointer must be 16-byte aligned");
    const int64_t sb = stride[0], sn = stride[1], sh = kv_heads > 1 ? stride[2] : stride[1];
    if (sn % 8 || sh % 8 || sb % 8 || sn <= 0 || sh <= 0 || sb < 0)
        return fail(SLIMKV_ERR_ALIGNMENT, "K/V strides must be positive multiples of 8 elements");
    *bcast = sb == 0 ? 1 : 0;
    const int b_dim = sb == 0 ? 1 : batch;
    const int64_t sb_eff = sb == 0 ? sn * keys : sb;
    return encode_map_4d(map, base, dim, kv_heads, keys, b_dim, sh * 2, sn * 2, sb_eff * 2, box_rows);
}

}  // namespace slimkv

using namespace slimkv;

extern "C" size_t slimkv_attention_workspace_size(const slimkv_attention_args* a) {
    Plan p;
    if (plan_attention(a, p) != SLIMKV_OK) return 0;
    Carver c(nullptr, 0);
    c.take<float>(p.part_o);
    c.take<float>(p.part_lse);
    return c.used + 256;
}

extern "C" int slimkv_attention_forward(const slimkv_attention_args* a, void* workspace, size_t workspace_bytes,
                                        void* stream_ptr) {
    Plan p;
    int rc = plan_attention(a, p);
    if (rc) return rc;
    if (!a->q || !a->k || !a->v || !a->out || !a->lse)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (a->q_stride[0] % 8 || a->q_stride[1] % 8 || a->q_stride[2] % 8 || !aligned16(a->q))
        return fail(SLIMKV_ERR_ALIGNMENT, "q must be 16-byte aligned with strides that are multiples of 8");
    Carver c(workspace, workspace_bytes);
    float* part_o = c.take<float>(p.part_o);
    float* part_lse = c.take<float>(p.part_lse);
    if (!workspace || !c.fits()) return fail(SLIMKV_ERR_WORKSPACE, "workspace too small (%zu < %zu)",
                                             workspace_bytes, c.used);
    CUtensorMap km, vm;
    int kb = 0, vb = 0;
    if ((rc = make_bshd_map(&km, a->k, a->batch, a->keys, a->kv_heads, a->head_dim, a->k_stride, &kb, kTile))) return rc;
    if ((rc = make_bshd_map(&vm, a->v, a->batch, a->keys, a->kv_heads, a->value_dim, a->v_stride, &vb, kTile))) return rc;
    AttnJob job{};
    job.q = a->q;
    job.q_fp16 = 0;
    job.q_sb = a->q_stride[0];
    job.q_sl = a->q_stride[1];
    job.q_sh = a->q_stride[2];
    job.k_bcast = kb;
    job.v_bcast = vb;
    job.seqlens = a->cache_seqlens;
    job.keys = a->keys;
    job.qlens = nullptr;
    job.queries = a->queries;
    job.group = a->heads / a->kv_heads;
    job.kv_heads = a->kv_heads;
    job.dk = a->head_dim;
    job.scale_log2 = a->scale * 1.4426950408889634f;
    job.causal = a->causal && a->queries > 1;
    job.splits = p.splits;
    job.tiles_per_split = p.tiles_per_split;
    job.rows_alloc = p.rows_alloc;
    job.out_width = p.width;
    job.part_o = part_o;
    job.part_lse = part_lse;
    job.status = status_word();
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    dim3 grid(p.splits, a->batch * a->kv_heads, p.row_blocks);
    if ((rc = launch_attention_job(p.width, p.mt, km, vm, job, grid, stream))) return rc;
    const int rows_total = job.group * a->queries;
    dim3 cgrid(a->batch * a->kv_heads, (rows_total + 7) / 8);
    attention_combine_kernel<<<cgrid, 256, 0, stream>>>(
        part_o, part_lse, p.splits, p.rows_alloc, p.width, rows_total, job.group, a->kv_heads, a->value_dim,
        a->out, a->out_fp32, a->out_stride[0], a->out_stride[1], a->out_stride[2], a->lse,
        a->heads, a->queries, a->lse_masked_positive ? INFINITY : -INFINITY);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(SLIMKV_ERR_CUDA, "combine launch failed: %s", cudaGetErrorString(e));
    return SLIMKV_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free variant.  Its split scratch lives in a fixed static device
// array instead of a caller-provided workspace, for callers that cannot
// allocate device memory themselves.
namespace slimkv {

constexpr size_t kStaticScratchBytes = size_t(16) << 20;   // 16 MiB per device
static __device__ __align__(256) unsigned char g_attention_scratch[kStaticScratchBytes];

// Device address of this device's copy of the scratch array.  The array's name
// is only a host-side handle, so the address is looked up once per device with
// that device current and cached.
static int static_scratch(void** out) {
    static std::mutex lock;
    static void* cache[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return fail(SLIMKV_ERR_CUDA, "no current CUDA device");
    std::lock_guard<std::mutex> guard(lock);
    if (!cache[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_attention_scratch);
        if (e != cudaSuccess)
            return fail(SLIMKV_ERR_CUDA, "cudaGetSymbolAddress of the static scratch failed: %s", cudaGetErrorString(e));
        cache[dev] = p;
    }
    *out = cache[dev];
    return SLIMKV_OK;
}

}  // namespace slimkv

extern "C" int slimkv_attention_forward_noalloc(const slimkv_attention_args* a, void* stream) {
    Plan p;
    const int rc = plan_attention(a, p);
    if (rc) return rc;
    const size_t need = slimkv_attention_workspace_size(a);
    if (need > kStaticScratchBytes)
        return fail(SLIMKV_ERR_WORKSPACE,
                    "this call needs %zu bytes of split scratch; the allocation-free entry point has a fixed "
                    "%zu-byte buffer (use slimkv_attention_forward with a workspace, or fewer splits)",
                    need, kStaticScratchBytes);
    void* scratch = nullptr;
    if (const int e = static_scratch(&scratch)) return e;
    // Every element of the partials that the combine reads is written first
    // by the split kernel, so the shared buffer needs no clearing.
    return slimkv_attention_forward(a, scratch, kStaticScratchBytes, stream);
}
