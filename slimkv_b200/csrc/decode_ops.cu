// Standalone decode element-wise ops: BF16-exact RoPE of q and raw K
// (replaces decode_ops.fused_rope, slimkv/llama3/decode_ops.py:14-31) and
// the LSE merge of the raw and latent branches (replaces
// decode_ops.fused_merge, decode_ops.py:34-48).  One thread per output pair
// of elements; both are bandwidth-trivial next to the attention kernels.
#include <algorithm>

#include "common.cuh"
#include "host_utils.h"

namespace slimkv {

__device__ __forceinline__ float rope_value(float x, float partner, int d, int half, float c, float s) {
    const float rot = d < half ? -partner : partner;
    const float first = bf16_round(__fmul_rn(x, bf16_round(c)));
    const float second = bf16_round(__fmul_rn(rot, bf16_round(s)));
    return __fadd_rn(first, second);
}

struct RopeArgs {
    const __nv_bfloat16* q; int64_t qb, qh, qs;
    const __nv_bfloat16* k; int64_t kb, kh, ks;
    const float* cos; const float* sin; int positions;
    const int64_t* qpos; int64_t qpos_stride;
    const int64_t* raw_idx; int sink, history;
    int batch, heads, kv_heads, queries, keys, dim;
    __nv_bfloat16* q_out; __nv_bfloat16* k_out;
    unsigned int* status;
};

__global__ void rope_decode_kernel(RopeArgs a) {
    const int64_t nq = (int64_t)a.batch * a.heads * a.queries * a.dim;
    const int64_t nk = (int64_t)a.batch * a.kv_heads * a.keys * a.dim;
    const int half = a.dim / 2;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nq + nk; i += (int64_t)gridDim.x * blockDim.x) {
        const bool is_q = i < nq;
        const int64_t off = is_q ? i : i - nq;
        const int d = off % a.dim;
        const int s = (off / a.dim) % (is_q ? a.queries : a.keys);
        const int h = (off / ((int64_t)a.dim * (is_q ? a.queries : a.keys))) % (is_q ? a.heads : a.kv_heads);
        const int b = off / ((int64_t)a.dim * (is_q ? a.queries : a.keys) * (is_q ? a.heads : a.kv_heads));
        int64_t pos;
        const __nv_bfloat16* row;
        if (is_q) {
            pos = a.qpos[b * a.qpos_stride + s];
            row = a.q + b * a.qb + h * a.qh + s * a.qs;
        } else {
            if (s < a.sink) pos = s;
            else if (s == a.keys - 1) pos = a.qpos[b * a.qpos_stride];
            else pos = a.raw_idx[s - a.sink] + a.sink + a.history;
            row = a.k + b * a.kb + h * a.kh + s * a.ks;
        }
        if (pos < 0 || pos >= a.positions) {
            report(a.status, SLIMKV_DEVICE_BAD_LENGTH);
            pos = 0;
        }
        const float v = rope_value(__bfloat162float(row[d]), __bfloat162float(row[(d + half) % a.dim]), d, half,
                                   a.cos[pos * a.dim + d], a.sin[pos * a.dim + d]);
        (is_q ? a.q_out : a.k_out)[off] = __float2bfloat16_rn(v);
    }
}

struct RopeRowsArgs {
    const __nv_bfloat16* x; int64_t xb, xt, xh;
    __nv_bfloat16* out; int64_t ob, ot, oh;
    const int32_t* pos; int64_t pos_stride;
    const int32_t* count;
    int batch, tokens, heads, dim;
    const float* cos; const float* sin; int positions;
    unsigned int* status;
};

// out[b, t, h, :] = rope(x[b, t, h, :]) at position pos[b][t], for t < count[b].
__global__ void rope_rows_kernel(RopeRowsArgs a) {
    const int64_t n = (int64_t)a.batch * a.tokens * a.heads * a.dim;
    const int half = a.dim / 2;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int d = i % a.dim;
        const int h = (i / a.dim) % a.heads;
        const int t = (i / ((int64_t)a.dim * a.heads)) % a.tokens;
        const int b = i / ((int64_t)a.dim * a.heads * a.tokens);
        if (t >= (a.count ? a.count[b] : a.tokens)) continue;
        int pos = a.pos[b * a.pos_stride + t];
        if (pos < 0 || pos >= a.positions) {
            report(a.status, SLIMKV_DEVICE_BAD_LENGTH);
            pos = 0;
        }
        const __nv_bfloat16* row = a.x + b * a.xb + t * a.xt + h * a.xh;
        const float v = rope_value(__bfloat162float(row[d]), __bfloat162float(row[(d + half) % a.dim]), d, half,
                                   a.cos[(int64_t)pos * a.dim + d], a.sin[(int64_t)pos * a.dim + d]);
        a.out[b * a.ob + t * a.ot + h * a.oh + d] = __float2bfloat16_rn(v);
    }
}

struct MergeOpArgs {
    const __nv_bfloat16* raw; int64_t rb, rh, rs;
    const float* rl; int64_t rlb, rlh, rls;
    const __nv_bfloat16* lat; int64_t lb, lh, ls;
    const float* ll; int64_t llb, llh, lls;
    int batch, heads, queries, dim;
    __nv_bfloat16* out;
};

__global__ void merge_kernel(MergeOpArgs a) {
    const int64_t n = (int64_t)a.batch * a.heads * a.queries * a.dim;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int d = i % a.dim;
        const int q = (i / a.dim) % a.queries;
        const int h = (i / ((int64_t)a.dim * a.queries)) % a.heads;
        const int b = i / ((int64_t)a.dim * a.queries * a.heads);
        const float r = a.rl[b * a.rlb + h * a.rlh + q * a.rls];
        const float l = a.ll[b * a.llb + h * a.llh + q * a.lls];
        float value = 0.f;
        if (!(r == -INFINITY && l == -INFINITY)) {
            const float total = fmaxf(r, l) + log1pf(expf(-fabsf(r - l)));
            const float rv = __bfloat162float(a.raw[b * a.rb + h * a.rh + q * a.rs + d]);
            const float lv = __bfloat162float(a.lat[b * a.lb + h * a.lh + q * a.ls + d]);
            value = (r == -INFINITY ? 0.f : expf(r - total) * rv) + (l == -INFINITY ? 0.f : expf(l - total) * lv);
        }
        a.out[i] = __float2bfloat16_rn(value);
    }
}

static int grid_for(int64_t n) {
    const int sms = std::max(device_info().sm_count, 1);
    int64_t blocks = (n + 255) / 256;
    return int(std::min<int64_t>(std::max<int64_t>(blocks, 1), int64_t(sms) * 8));
}

}  // namespace slimkv

using namespace slimkv;

extern "C" int slimkv_rope_decode(const void* q, const int64_t q_stride[3], const void* k, const int64_t k_stride[3],
                                  const float* cos, const float* sin, int rope_positions, const int64_t* qpos,
                                  int64_t qpos_stride, const int64_t* raw_idx, int sink, int history, int batch,
                                  int heads, int kv_heads, int queries, int keys, int head_dim, void* q_out,
                                  void* k_out, void* stream) {
    if (!q || !k || !cos || !sin || !qpos || !q_out || !k_out || !q_stride || !k_stride)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "null pointer");
    if (batch <= 0 || heads <= 0 || kv_heads <= 0 || queries <= 0 || keys <= 0 || head_dim <= 0 || head_dim % 2)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "invalid sizes");
    if (keys - 1 > sink && !raw_idx) return fail(SLIMKV_ERR_INVALID_ARGUMENT, "raw indices required");
    if (sink < 0 || history < 0) return fail(SLIMKV_ERR_INVALID_ARGUMENT, "negative sink/history");
    RopeArgs a{};
    a.q = static_cast<const __nv_bfloat16*>(q); a.qb = q_stride[0]; a.qh = q_stride[1]; a.qs = q_stride[2];
    a.k = static_cast<const __nv_bfloat16*>(k); a.kb = k_stride[0]; a.kh = k_stride[1]; a.ks = k_stride[2];
    a.cos = cos; a.sin = sin; a.positions = rope_positions; a.qpos = qpos; a.qpos_stride = qpos_stride;
    a.raw_idx = raw_idx; a.sink = sink; a.history = history; a.batch = batch; a.heads = heads;
    a.kv_heads = kv_heads; a.queries = queries; a.keys = keys; a.dim = head_dim;
    a.q_out = static_cast<__nv_bfloat16*>(q_out); a.k_out = static_cast<__nv_bfloat16*>(k_out);
    a.status = status_word();
    const int64_t n = (int64_t)batch * (heads * queries + kv_heads * keys) * head_dim;
    rope_decode_kernel<<<grid_for(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(a);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? SLIMKV_OK : fail(SLIMKV_ERR_CUDA, "rope launch failed: %s", cudaGetErrorString(e));
}

extern "C" int slimkv_merge(const void* raw, const int64_t raw_stride[3], const float* raw_lse,
                            const int64_t raw_lse_stride[3], const void* latent, const int64_t latent_stride[3],
                            const float* latent_lse, const int64_t latent_lse_stride[3], int batch, int heads,
                            int queries, int head_dim, void* out, void* stream) {
    if (!raw || !raw_lse || !latent || !latent_lse || !out || !raw_stride || !raw_lse_stride || !latent_stride ||
        !latent_lse_stride)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "null pointer");
    if (batch <= 0 || heads <= 0 || queries <= 0 || head_dim <= 0)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "invalid sizes");
    MergeOpArgs a{};
    a.raw = static_cast<const __nv_bfloat16*>(raw); a.rb = raw_stride[0]; a.rh = raw_stride[1]; a.rs = raw_stride[2];
    a.rl = raw_lse; a.rlb = raw_lse_stride[0]; a.rlh = raw_lse_stride[1]; a.rls = raw_lse_stride[2];
    a.lat = static_cast<const __nv_bfloat16*>(latent);
    a.lb = latent_stride[0]; a.lh = latent_stride[1]; a.ls = latent_stride[2];
    a.ll = latent_lse; a.llb = latent_lse_stride[0]; a.llh = latent_lse_stride[1]; a.lls = latent_lse_stride[2];
    a.batch = batch; a.heads = heads; a.queries = queries; a.dim = head_dim;
    a.out = static_cast<__nv_bfloat16*>(out);
    const int64_t n = (int64_t)batch * heads * queries * head_dim;
    merge_kernel<<<grid_for(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(a);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? SLIMKV_OK : fail(SLIMKV_ERR_CUDA, "merge launch failed: %s", cudaGetErrorString(e));
}

extern "C" int slimkv_rope_rows(const void* x, const int64_t x_stride[3], void* out, const int64_t out_stride[3],
                                const int32_t* positions, int64_t positions_stride, const int32_t* counts, int batch,
                                int tokens, int heads, int head_dim, const float* cos, const float* sin,
                                int rope_positions, void* stream) {
    if (!x || !out || !x_stride || !out_stride || !positions || !cos || !sin)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "null pointer");
    if (x == out) return fail(SLIMKV_ERR_INVALID_ARGUMENT, "rope_rows does not rotate in place");
    if (batch <= 0 || tokens <= 0 || heads <= 0 || head_dim <= 0 || head_dim % 2 || rope_positions <= 0)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "invalid sizes");
    RopeRowsArgs a{};
    a.x = static_cast<const __nv_bfloat16*>(x); a.xb = x_stride[0]; a.xt = x_stride[1]; a.xh = x_stride[2];
    a.out = static_cast<__nv_bfloat16*>(out); a.ob = out_stride[0]; a.ot = out_stride[1]; a.oh = out_stride[2];
    a.pos = positions; a.pos_stride = positions_stride; a.count = counts;
    a.batch = batch; a.tokens = tokens; a.heads = heads; a.dim = head_dim;
    a.cos = cos; a.sin = sin; a.positions = rope_positions; a.status = status_word();
    const int64_t n = (int64_t)batch * tokens * heads * head_dim;
    rope_rows_kernel<<<grid_for(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(a);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? SLIMKV_OK : fail(SLIMKV_ERR_CUDA, "rope rows launch failed: %s", cudaGetErrorString(e));
}
