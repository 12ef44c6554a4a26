// The decoder layer's element-wise steps around the decode attention, as the
// batched runtime runs them each step (two RMSNorms and one gated activation
// per layer over 2B rows).  Each is one launch doing what the reference's
// modules do in two to four:
//   slimkv_rms_norm — LlamaRMSNorm.forward (slimkv/llama3/modeling_llama.py:
//     79-95): fp32 mean of squares, x * rsqrt(var + eps) rounded to the input
//     dtype (bf16), then times the bf16 weight (rounded again);
//   slimkv_silu_mul — the product inside LlamaMLP.forward (modeling_llama.py:
//     97-113), act_fn(gate) * up with act_fn = SiLU: silu(g) = g / (1 +
//     e^-g) in fp32 rounded to bf16, times up, rounded to bf16.
// Both are latency-bound at decode sizes (a few hundred KB per launch); the
// residual adds around them go into the GEMMs' accumulate (beta = 1).
#include <algorithm>

#include "common.cuh"
#include "host_utils.h"

namespace slimkv {
namespace {

constexpr int kNormThreads = 256;

__device__ __forceinline__ void unpack8(uint4 v, float (&f)[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        f[2 * i] = __uint_as_float(w[i] << 16);
        f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
    return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                      pack_bf16x2(f[6], f[7]));
}

// One CTA per row; each thread keeps its 8-element groups in registers
// between the reduction and the scaling (hidden <= kNormThreads * 8 * 4).
__global__ void __launch_bounds__(kNormThreads) rms_norm_kernel(const __nv_bfloat16* __restrict__ x, int64_t xs,
                                                                const __nv_bfloat16* __restrict__ w,
                                                                __nv_bfloat16* __restrict__ out, int64_t os,
                                                                int hidden, float eps) {
    constexpr int kMaxGroups = 4;
    __shared__ float s_part[kNormThreads / 32];
    const int row = blockIdx.x, tid = threadIdx.x;
    const int groups = hidden / 8;
    const uint4* src = reinterpret_cast<const uint4*>(x + row * xs);
    float v[kMaxGroups][8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxGroups; ++i) {
        const int g = tid + i * kNormThreads;
        if (g < groups) {
            unpack8(__ldg(src + g), v[i]);
#pragma unroll
            for (int e = 0; e < 8; ++e) ss = fmaf(v[i][e], v[i][e], ss);
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((tid & 31) == 0) s_part[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < kNormThreads / 32; ++i) tot += s_part[i];
    const float r = rsqrtf(tot / float(hidden) + eps);
    const uint4* wv = reinterpret_cast<const uint4*>(w);
    uint4* dst = reinterpret_cast<uint4*>(out + row * os);
#pragma unroll
    for (int i = 0; i < kMaxGroups; ++i) {
        const int g = tid + i * kNormThreads;
        if (g < groups) {
            float wf[8], o[8];
            unpack8(__ldg(wv + g), wf);
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = wf[e] * bf16_round(v[i][e] * r);
            dst[g] = pack8(o);
        }
    }
}

// Eight outputs per thread: gate columns [0, inter), up columns [inter, 2 inter).
__global__ void __launch_bounds__(256) silu_mul_kernel(const __nv_bfloat16* __restrict__ gu, int64_t gs,
                                                       __nv_bfloat16* __restrict__ out, int64_t os, int rows,
                                                       int inter) {
    const int per_row = inter / 8;
    const int64_t n = int64_t(rows) * per_row;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        const int r = int(i / per_row), g = int(i - int64_t(r) * per_row);
        const __nv_bfloat16* row = gu + r * gs;
        float a[8], b[8], o[8];
        unpack8(__ldg(reinterpret_cast<const uint4*>(row) + g), a);
        unpack8(__ldg(reinterpret_cast<const uint4*>(row + inter) + g), b);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = bf16_round(a[e] / (1.f + expf(-a[e]))) * b[e];
        reinterpret_cast<uint4*>(out + r * os)[g] = pack8(o);
    }
}

}  // namespace
}  // namespace slimkv

using namespace slimkv;

extern "C" int slimkv_rms_norm(const void* x, int64_t x_row_stride, const void* weight, void* out,
                               int64_t out_row_stride, int rows, int hidden, float eps, void* stream) {
    if (!x || !weight || !out) return fail(SLIMKV_ERR_INVALID_ARGUMENT, "null pointer");
    if (rows <= 0 || hidden <= 0 || hidden % 8 || hidden > kNormThreads * 8 * 4)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "rms_norm: hidden must be a multiple of 8 up to %d",
                    kNormThreads * 8 * 4);
    if (!aligned16(x) || !aligned16(weight) || !aligned16(out) || x_row_stride % 8 || out_row_stride % 8)
        return fail(SLIMKV_ERR_ALIGNMENT, "rms_norm: 16-byte aligned rows");
    rms_norm_kernel<<<rows, kNormThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __nv_bfloat16*>(x), x_row_stride, static_cast<const __nv_bfloat16*>(weight),
        static_cast<__nv_bfloat16*>(out), out_row_stride, hidden, eps);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? SLIMKV_OK : fail(SLIMKV_ERR_CUDA, "rms_norm launch failed: %s", cudaGetErrorString(e));
}

extern "C" int slimkv_silu_mul(const void* gate_up, int64_t gate_up_row_stride, void* out, int64_t out_row_stride,
                               int rows, int intermediate, void* stream) {
    if (!gate_up || !out) return fail(SLIMKV_ERR_INVALID_ARGUMENT, "null pointer");
    if (rows <= 0 || intermediate <= 0 || intermediate % 8)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "silu_mul: intermediate must be a positive multiple of 8");
    if (!aligned16(gate_up) || !aligned16(out) || gate_up_row_stride % 8 || out_row_stride % 8)
        return fail(SLIMKV_ERR_ALIGNMENT, "silu_mul: 16-byte aligned rows");
    const int64_t n = int64_t(rows) * (intermediate / 8);
    const int blocks = int(std::min<int64_t>((n + 255) / 256, 4 * 148));
    silu_mul_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __nv_bfloat16*>(gate_up), gate_up_row_stride, static_cast<__nv_bfloat16*>(out),
        out_row_stride, rows, intermediate);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? SLIMKV_OK : fail(SLIMKV_ERR_CUDA, "silu_mul launch failed: %s", cudaGetErrorString(e));
}
