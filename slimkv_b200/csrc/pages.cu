// Paged SlimKV cache IO (C ABI slimkv_beacon_pages_* / slimkv_raw_pages_*).
//
// The vLLM plugin's page layouts (slimkv/vllm_plugin/paged_cache.py:12-127),
// byte for byte:
//   Beacon page p = pages + p * page_stride (bf16 elements):
//       [sink_elements = 2 * raw_width][slots x (rank_k + rank_v)]
//     logical Beacon n of a sequence -> page table[n / slots], element
//     sink_elements + (n % slots) * W (K then V, W = rank_k + rank_v);
//     the sequence's sink token (K then V, raw_width each) at the start of
//     its root page table[0].
//   Raw pages [blocks][block_size][2 (K, V)][kv_heads][head_dim]: absolute
//     raw position t -> block table[t / block_size], row t % block_size.
// Batched over sequences (each with its own block table row and cursor);
// one thread per 16-byte vector.  Every page id and position is checked
// against the allocation: a bad one sets SLIMKV_DEVICE_BAD_LENGTH and the
// vector is skipped (no fault).
#include <algorithm>

#include "common.cuh"
#include "host_utils.h"

namespace slimkv {

namespace {

struct BeaconGeom {
    uint16_t* pages;
    int64_t page_stride;
    int slots, rank_k, rank_v, width, sink;
    const int32_t* table;
    int64_t table_stride;
    int num_pages;
    unsigned* status;
};

__device__ __forceinline__ bool beacon_addr(const BeaconGeom& G, int b, int64_t n, int64_t& off) {
    const int64_t page_index = n / G.slots;
    const int page = (n < 0 || page_index >= G.table_stride) ? -1 : G.table[b * G.table_stride + page_index];
    if (page < 0 || page >= G.num_pages) {
        report(G.status, SLIMKV_DEVICE_BAD_LENGTH);
        return false;
    }
    off = int64_t(page) * G.page_stride + G.sink + (n % G.slots) * G.width;
    return true;
}

// Copy unit: U = uint4 (8 elements) when every size, stride and base is a
// multiple of 8 elements, else uint16_t (one element).
template <typename U>
constexpr int kElems = sizeof(U) / 2;

// grid-stride over batch x count x W / E units
template <typename U>
__global__ void beacon_append_kernel(BeaconGeom G, int batch, const int32_t* start, int count, const uint16_t* key,
                                     int64_t ksb, int64_t ksr, const uint16_t* value, int64_t vsb, int64_t vsr) {
    constexpr int E = kElems<U>;
    const int units = G.width / E, ku = G.rank_k / E;
    const int64_t total = int64_t(batch) * count * units;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int u = int(i % units);
        const int64_t r = (i / units) % count;
        const int b = int(i / units / count);
        int64_t off;
        if (!beacon_addr(G, b, int64_t(start[b]) + r, off)) continue;
        const U v = u < ku ? *reinterpret_cast<const U*>(key + b * ksb + r * ksr + u * E)
                           : *reinterpret_cast<const U*>(value + b * vsb + r * vsr + (u - ku) * E);
        *reinterpret_cast<U*>(G.pages + off + u * E) = v;
    }
}

template <typename U>
__global__ void beacon_gather_kernel(BeaconGeom G, int batch, const int32_t* count, int max_count, uint16_t* key,
                                     int64_t ksb, int64_t ksr, uint16_t* value, int64_t vsb, int64_t vsr) {
    constexpr int E = kElems<U>;
    const int units = G.width / E, ku = G.rank_k / E;
    const int64_t total = int64_t(batch) * max_count * units;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int u = int(i % units);
        const int64_t r = (i / units) % max_count;
        const int b = int(i / units / max_count);
        if (r >= count[b]) continue;
        int64_t off;
        if (!beacon_addr(G, b, r, off)) continue;
        const U v = *reinterpret_cast<const U*>(G.pages + off + u * E);
        if (u < ku) *reinterpret_cast<U*>(key + b * ksb + r * ksr + u * E) = v;
        else *reinterpret_cast<U*>(value + b * vsb + r * vsr + (u - ku) * E) = v;
    }
}

// Sink token of each sequence: raw_width K elements then raw_width V elements
// at the start of the root page.  write = 1: dense -> page, else page -> dense.
template <typename U>
__global__ void beacon_sink_kernel(BeaconGeom G, int batch, uint16_t* key, uint16_t* value, int64_t stride_batch,
                                   int write) {
    constexpr int E = kElems<U>;
    const int half = G.sink / 2, units = G.sink / E;
    const int64_t total = int64_t(batch) * units;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int u = int(i % units), b = int(i / units);
        const int page = G.table_stride > 0 ? G.table[b * G.table_stride] : -1;
        if (page < 0 || page >= G.num_pages) {
            report(G.status, SLIMKV_DEVICE_BAD_LENGTH);
            continue;
        }
        uint16_t* slot = G.pages + int64_t(page) * G.page_stride + u * E;
        const int e = u * E;
        uint16_t* dense = e < half ? key + b * stride_batch + e : value + b * stride_batch + (e - half);
        if (write) *reinterpret_cast<U*>(slot) = *reinterpret_cast<const U*>(dense);
        else *reinterpret_cast<U*>(dense) = *reinterpret_cast<const U*>(slot);
    }
}

struct RawGeom {
    uint16_t* pages;
    int block_size, kv_heads, head_dim;
    const int32_t* table;
    int64_t table_stride;
    int num_blocks;
    unsigned* status;
};

// Vector i -> (b, token r, kind, head, 8-element unit).  write = 1: dense
// rows [B][count][Hkv][D] (key, value) -> pages, else pages -> dense.
template <typename U>
__global__ void raw_pages_kernel(RawGeom G, int batch, const int32_t* start, const int32_t* counts, int count,
                                 uint16_t* key, int64_t ksb, int64_t kst, uint16_t* value, int64_t vsb, int64_t vst,
                                 int write) {
    constexpr int E = kElems<U>;
    const int row = G.kv_heads * G.head_dim, units = 2 * row / E;
    const int64_t total = int64_t(batch) * count * units;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int u = int(i % units);
        const int64_t r = (i / units) % count;
        const int b = int(i / units / count);
        if (counts && r >= counts[b]) continue;
        const int64_t t = int64_t(start[b]) + r;
        const int64_t bi = t / G.block_size;
        const int blk = (t < 0 || bi >= G.table_stride) ? -1 : G.table[b * G.table_stride + bi];
        if (blk < 0 || blk >= G.num_blocks) {
            report(G.status, SLIMKV_DEVICE_BAD_LENGTH);
            continue;
        }
        const int e = u * E, kind = e / row, within = e - kind * row;
        uint16_t* slot = G.pages + ((int64_t(blk) * G.block_size + t % G.block_size) * 2 + kind) * row + within;
        uint16_t* dense = kind == 0 ? key + b * ksb + r * kst + within : value + b * vsb + r * vst + within;
        if (write) *reinterpret_cast<U*>(slot) = *reinterpret_cast<const U*>(dense);
        else *reinterpret_cast<U*>(dense) = *reinterpret_cast<const U*>(slot);
    }
}

int grid_for(int64_t vectors) {
    const int sms = std::max(device_info().sm_count, 1);
    return int(std::max<int64_t>(1, std::min<int64_t>((vectors + 255) / 256, int64_t(sms) * 8)));
}

int beacon_geom(const slimkv_beacon_pages* p, BeaconGeom& G) {
    if (!p || !p->pages || !p->table) return fail(SLIMKV_ERR_INVALID_ARGUMENT, "null page arguments");
    if (p->slots <= 0 || p->rank_k <= 0 || p->rank_v <= 0 || p->sink_elements < 0 || p->sink_elements % 2 ||
        p->table_stride <= 0 || p->num_pages <= 0)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "Cache dimensions must be positive.");
    if (p->page_stride < int64_t(p->sink_elements) + int64_t(p->slots) * (p->rank_k + p->rank_v))
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "Physical page is too small for the declared ranks.");
    G.pages = static_cast<uint16_t*>(p->pages);
    G.page_stride = p->page_stride;
    G.slots = p->slots;
    G.rank_k = p->rank_k;
    G.rank_v = p->rank_v;
    G.width = p->rank_k + p->rank_v;
    G.sink = p->sink_elements;
    G.table = p->table;
    G.table_stride = p->table_stride;
    G.num_pages = p->num_pages;
    G.status = status_word();
    return SLIMKV_OK;
}

int raw_geom(const slimkv_raw_pages* p, RawGeom& G) {
    if (!p || !p->pages || !p->table) return fail(SLIMKV_ERR_INVALID_ARGUMENT, "null page arguments");
    if (p->block_size <= 0 || p->kv_heads <= 0 || p->head_dim <= 0 || p->table_stride <= 0 || p->num_blocks <= 0)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "Cache dimensions must be positive.");
    G.pages = static_cast<uint16_t*>(p->pages);
    G.block_size = p->block_size;
    G.kv_heads = p->kv_heads;
    G.head_dim = p->head_dim;
    G.table = p->table;
    G.table_stride = p->table_stride;
    G.num_blocks = p->num_blocks;
    G.status = status_word();
    return SLIMKV_OK;
}

// 16-byte units apply when every base, stride and size is a multiple of 8
// elements.
bool vec_ok(const void* base, int64_t a, int64_t b) { return aligned16(base) && a % 8 == 0 && b % 8 == 0; }

int launched(const char* what) {
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? SLIMKV_OK : fail(SLIMKV_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(e));
}

}  // namespace
}  // namespace slimkv

using namespace slimkv;

extern "C" int slimkv_beacon_pages_append(const slimkv_beacon_pages* pages, int batch, const int32_t* start, int count,
                                          const void* key, int64_t key_stride_batch, int64_t key_stride_row,
                                          const void* value, int64_t value_stride_batch, int64_t value_stride_row,
                                          void* stream) {
    BeaconGeom G;
    if (int rc = beacon_geom(pages, G)) return rc;
    if (batch < 0 || count < 0 || !start || !key || !value)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "invalid batch, count or rows");
    if (batch == 0 || count == 0) return SLIMKV_OK;
    const bool vec = vec_ok(G.pages, G.page_stride, G.sink) && G.rank_k % 8 == 0 && G.rank_v % 8 == 0 &&
                     vec_ok(key, key_stride_batch, key_stride_row) && vec_ok(value, value_stride_batch, value_stride_row);
    const int64_t units = int64_t(batch) * count * (vec ? G.width / 8 : G.width);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const auto* k = static_cast<const uint16_t*>(key);
    const auto* v = static_cast<const uint16_t*>(value);
    if (vec)
        beacon_append_kernel<uint4><<<grid_for(units), 256, 0, st>>>(G, batch, start, count, k, key_stride_batch,
                                                                     key_stride_row, v, value_stride_batch,
                                                                     value_stride_row);
    else
        beacon_append_kernel<uint16_t><<<grid_for(units), 256, 0, st>>>(G, batch, start, count, k, key_stride_batch,
                                                                        key_stride_row, v, value_stride_batch,
                                                                        value_stride_row);
    return launched("Beacon page append");
}

extern "C" int slimkv_beacon_pages_gather(const slimkv_beacon_pages* pages, int batch, const int32_t* count,
                                          int max_count, void* key, int64_t key_stride_batch, int64_t key_stride_row,
                                          void* value, int64_t value_stride_batch, int64_t value_stride_row,
                                          void* stream) {
    BeaconGeom G;
    if (int rc = beacon_geom(pages, G)) return rc;
    if (batch < 0 || max_count < 0 || !count || !key || !value)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "invalid batch, count or rows");
    if (batch == 0 || max_count == 0) return SLIMKV_OK;
    const bool vec = vec_ok(G.pages, G.page_stride, G.sink) && G.rank_k % 8 == 0 && G.rank_v % 8 == 0 &&
                     vec_ok(key, key_stride_batch, key_stride_row) && vec_ok(value, value_stride_batch, value_stride_row);
    const int64_t units = int64_t(batch) * max_count * (vec ? G.width / 8 : G.width);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    auto* k = static_cast<uint16_t*>(key);
    auto* v = static_cast<uint16_t*>(value);
    if (vec)
        beacon_gather_kernel<uint4><<<grid_for(units), 256, 0, st>>>(G, batch, count, max_count, k, key_stride_batch,
                                                                     key_stride_row, v, value_stride_batch,
                                                                     value_stride_row);
    else
        beacon_gather_kernel<uint16_t><<<grid_for(units), 256, 0, st>>>(G, batch, count, max_count, k,
                                                                        key_stride_batch, key_stride_row, v,
                                                                        value_stride_batch, value_stride_row);
    return launched("Beacon page gather");
}

extern "C" int slimkv_beacon_pages_sink(const slimkv_beacon_pages* pages, int batch, void* key, void* value,
                                        int64_t stride_batch, int write, void* stream) {
    BeaconGeom G;
    if (int rc = beacon_geom(pages, G)) return rc;
    if (batch < 0 || G.sink == 0 || !key || !value)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "no sink area in the page layout, or null rows");
    if (batch == 0) return SLIMKV_OK;
    const bool vec = vec_ok(G.pages, G.page_stride, (G.sink / 2)) && vec_ok(key, stride_batch, 0) &&
                     vec_ok(value, stride_batch, 0);
    const int64_t units = int64_t(batch) * (vec ? G.sink / 8 : G.sink);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    auto* k = static_cast<uint16_t*>(key);
    auto* v = static_cast<uint16_t*>(value);
    if (vec) beacon_sink_kernel<uint4><<<grid_for(units), 256, 0, st>>>(G, batch, k, v, stride_batch, write ? 1 : 0);
    else beacon_sink_kernel<uint16_t><<<grid_for(units), 256, 0, st>>>(G, batch, k, v, stride_batch, write ? 1 : 0);
    return launched("Beacon page sink");
}

namespace {
int raw_io(const slimkv_raw_pages* pages, int batch, const int32_t* start, const int32_t* counts, int count, void* key,
           int64_t ksb, int64_t kst, void* value, int64_t vsb, int64_t vst, int write, cudaStream_t st) {
    RawGeom G;
    if (int rc = raw_geom(pages, G)) return rc;
    if (batch < 0 || count < 0 || !start || !key || !value)
        return fail(SLIMKV_ERR_INVALID_ARGUMENT, "invalid batch, count or rows");
    if (batch == 0 || count == 0) return SLIMKV_OK;
    const int row = G.kv_heads * G.head_dim;
    const bool vec = row % 8 == 0 && aligned16(G.pages) && vec_ok(key, ksb, kst) && vec_ok(value, vsb, vst);
    const int64_t units = int64_t(batch) * count * (vec ? 2 * row / 8 : 2 * row);
    auto* k = static_cast<uint16_t*>(key);
    auto* v = static_cast<uint16_t*>(value);
    if (vec)
        raw_pages_kernel<uint4><<<grid_for(units), 256, 0, st>>>(G, batch, start, counts, count, k, ksb, kst, v, vsb,
                                                                 vst, write);
    else
        raw_pages_kernel<uint16_t><<<grid_for(units), 256, 0, st>>>(G, batch, start, counts, count, k, ksb, kst, v, vsb,
                                                                    vst, write);
    return launched(write ? "raw page write" : "raw page read");
}
}  // namespace

extern "C" int slimkv_raw_pages_write(const slimkv_raw_pages* pages, int batch, const int32_t* start, int count,
                                      const void* key, int64_t key_stride_batch, int64_t key_stride_token,
                                      const void* value, int64_t value_stride_batch, int64_t value_stride_token,
                                      void* stream) {
    return raw_io(pages, batch, start, nullptr, count, const_cast<void*>(key), key_stride_batch, key_stride_token,
                  const_cast<void*>(value), value_stride_batch, value_stride_token, 1,
                  static_cast<cudaStream_t>(stream));
}

extern "C" int slimkv_raw_pages_read(const slimkv_raw_pages* pages, int batch, const int32_t* start,
                                     const int32_t* count, int max_count, void* key, int64_t key_stride_batch,
                                     int64_t key_stride_token, void* value, int64_t value_stride_batch,
                                     int64_t value_stride_token, void* stream) {
    if (!count) return fail(SLIMKV_ERR_INVALID_ARGUMENT, "null count");
    return raw_io(pages, batch, start, count, max_count, key, key_stride_batch, key_stride_token, value,
                  value_stride_batch, value_stride_token, 0, static_cast<cudaStream_t>(stream));
}
