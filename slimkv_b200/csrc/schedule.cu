// Device-side decode schedule (C ABI slimkv_decode_schedule): per-sequence
// restatement of the reference fast-decode bookkeeping
// (slimkv/llama3/memory.py:101-162) so a captured decode step needs no host
// work.  Integer-only; bit-exact with the reference schedule.
#include "common.cuh"
#include "host_utils.h"

namespace slimkv {

__global__ void decode_schedule_kernel(int batch, int sink, int window, int ratio, int32_t* history,
                                       int32_t* tail, int32_t* raw_len, int32_t* latent_len,
                                       int32_t* query_len, int32_t* qpos) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= batch) return;
    const int t = tail[b], h = history[b];
    const int insert = (t + 1) % ratio == 0 ? 1 : 0;
    query_len[b] = 1 + insert;
    raw_len[b] = sink + t + 1;
    latent_len[b] = h + t / ratio + insert;
    const int pos = sink + h + t + t / ratio;
    qpos[2 * b] = pos;
    qpos[2 * b + 1] = pos + 1;
    if (t + 1 == window) {
        history[b] = h + window / ratio;
        tail[b] = 0;
    } else {
        tail[b] = t + 1;
    }
}

}  // namespace slimkv

extern "C" int slimkv_decode_schedule(int batch, int sink, int window, int ratio, int32_t* history,
                                      int32_t* tail, int32_t* raw_len, int32_t* latent_len, int32_t* query_len,
                                      int32_t* qpos, void* stream) {
    using namespace slimkv;
    if (batch <= 0 || sink < 0 || window <= 0 || ratio <= 0 || window % ratio)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "invalid schedule geometry");
    if (!history || !tail || !raw_len || !latent_len || !query_len || !qpos)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "null pointer");
    decode_schedule_kernel<<<(batch + 127) / 128, 128, 0, static_cast<cudaStream_t>(stream)>>>(
        batch, sink, window, ratio, history, tail, raw_len, latent_len, query_len, qpos);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? SLIMKV_OK : fail(SLIMKV_ERR_CUDA, "schedule launch failed: %s", cudaGetErrorString(e));
}
