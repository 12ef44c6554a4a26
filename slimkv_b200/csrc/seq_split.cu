// N-part LSE merge of partial attention results: the exchange step of a
// sequence split, where each GPU attends over a contiguous shard of one
// sequence's keys.  merge_attention (slimkv/llama3/fa2_decode.py:57-66)
// merges the raw and latent partitions of a row; the same identity over N
// partitions is T = log sum_i exp(lse_i), out = sum_i exp(lse_i - T) part_i.
// One warp per row: lanes read the N log-sum-exps, then stream the N partial
// rows as float4 (a few KB per layer in total, so launch latency dominates).
#include <cmath>

#include "common.cuh"
#include "host_utils.h"

namespace slimkv {
namespace {

constexpr int kMaxParts = 64;

struct PartsArgs {
    int parts, rows, dim;
    const float* part_out; int64_t part_stride;
    const float* part_lse; int64_t lse_part_stride;
    void* out; int out_fp32; float* out_lse;
};

__global__ void __launch_bounds__(256) merge_partials_kernel(PartsArgs a) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * 8 + warp;
    if (row >= a.rows) return;
    // Lane i holds part i's (and i+32's) lse; the maximum and the sum of
    // exp(lse - max) by warp shuffles.
    float l0 = lane < a.parts ? __ldg(a.part_lse + lane * a.lse_part_stride + row) : -INFINITY;
    float l1 = lane + 32 < a.parts ? __ldg(a.part_lse + (lane + 32) * a.lse_part_stride + row) : -INFINITY;
    float m = fmaxf(l0, l1);
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float total = -INFINITY;
    if (m != -INFINITY) {
        float s = (l0 == -INFINITY ? 0.f : expf(l0 - m)) + (l1 == -INFINITY ? 0.f : expf(l1 - m));
#pragma unroll
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        total = m + logf(s);
    }
    if (a.out_lse && lane == 0) a.out_lse[row] = total;
    const float w0 = l0 == -INFINITY ? 0.f : expf(l0 - total), w1 = l1 == -INFINITY ? 0.f : expf(l1 - total);
    // Every lane runs the same iterations (the shuffles need the whole warp).
    for (int c0 = 0; c0 < a.dim; c0 += 128) {
        const int c = c0 + lane * 4;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        if (total != -INFINITY) {
            for (int i = 0; i < a.parts; ++i) {
                const float w = __shfl_sync(0xffffffffu, i < 32 ? w0 : w1, i & 31);
                if (w == 0.f || c >= a.dim) continue;
                const float4 x =
                    __ldg(reinterpret_cast<const float4*>(a.part_out + i * a.part_stride + (int64_t)row * a.dim + c));
                acc.x = fmaf(w, x.x, acc.x); acc.y = fmaf(w, x.y, acc.y);
                acc.z = fmaf(w, x.z, acc.z); acc.w = fmaf(w, x.w, acc.w);
            }
        }
        if (c >= a.dim) continue;
        const int64_t o = (int64_t)row * a.dim + c;
        if (a.out_fp32) {
            *reinterpret_cast<float4*>(static_cast<float*>(a.out) + o) = acc;
        } else {
            __nv_bfloat162* dst = reinterpret_cast<__nv_bfloat162*>(static_cast<__nv_bfloat16*>(a.out) + o);
            dst[0] = __floats2bfloat162_rn(acc.x, acc.y);
            dst[1] = __floats2bfloat162_rn(acc.z, acc.w);
        }
    }
}

}  // namespace
}  // namespace slimkv

using namespace slimkv;

extern "C" int slimkv_merge_partials(const slimkv_merge_partials_args* a, void* stream) {
    if (!a) return fail(SLIMKV_ERR_INVALID_ARGUMENT, "null arguments");
    if (a->parts < 1 || a->parts > kMaxParts || a->rows < 0 || a->dim <= 0)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "need 1..%d parts, rows >= 0, dim > 0", kMaxParts);
    if (a->rows == 0) return SLIMKV_OK;
    if (!a->part_out || !a->part_lse || !a->out) return fail(SLIMKV_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (a->parts > 1 && (a->part_stride < (int64_t)a->rows * a->dim || a->lse_part_stride < a->rows))
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "part strides smaller than a part");
    if (a->dim % 4 || a->part_stride % 4 || !aligned16(a->part_out) ||
        (a->out_fp32 ? !aligned16(a->out) : reinterpret_cast<uintptr_t>(a->out) % 8))
        return fail(SLIMKV_ERR_ALIGNMENT, "dim and part stride must be multiples of 4 with aligned buffers");
    PartsArgs k{a->parts, a->rows, a->dim, a->part_out, a->part_stride, a->part_lse, a->lse_part_stride,
                a->out, a->out_fp32, a->out_lse};
    merge_partials_kernel<<<(a->rows + 7) / 8, 256, 0, static_cast<cudaStream_t>(stream)>>>(k);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(SLIMKV_ERR_CUDA, "merge launch failed: %s", cudaGetErrorString(e));
    return SLIMKV_OK;
}
