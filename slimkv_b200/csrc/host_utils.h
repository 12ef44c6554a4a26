// Host-side helpers shared by the C-ABI entry points: error text, device
// properties, TMA tensor-map encoding and workspace carving.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "slimkv_b200.h"

namespace slimkv {

void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);

// Multiprocessor count and opt-in shared memory of the current device.
struct DeviceInfo {
    int device = -1;
    int sm_count = 0;
    int smem_optin = 0;
};
const DeviceInfo& device_info();

// Encode a 4-D bf16 tiled tensor map {d0, d1, d2, d3} with byte strides
// {s1, s2, s3} for dims 1..3, box {64, 1, box_rows, 1} and the 128-byte
// swizzle.  Returns SLIMKV_OK or SLIMKV_ERR_TENSOR_MAP (text in last error).
int encode_map_4d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                  uint64_t d3, uint64_t s1, uint64_t s2, uint64_t s3, uint32_t box_rows);
// The same with box {64, box1, box2, 1}: box1 x box2 rows of 128 bytes.
int encode_map_4d_box(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t d3,
                      uint64_t s1, uint64_t s2, uint64_t s3, uint32_t box1, uint32_t box2);
// fp32 3-D map without swizzle (row-major [d2][d1][d0], strides in bytes),
// box {box0, box1, 1}: the target of bulk tensor stores of staged tiles.
int encode_map_f32_3d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1,
                      uint64_t s2, uint32_t box0, uint32_t box1);

// Bump allocator over a caller-provided workspace (256-byte aligned pieces).
struct Carver {
    uint8_t* base;
    size_t size, used = 0;
    Carver(void* b, size_t s) : base(static_cast<uint8_t*>(b)), size(s) {}
    template <typename T>
    T* take(size_t count) {
        used = (used + 255) & ~size_t(255);
        T* p = reinterpret_cast<T*>(base ? base + used : nullptr);
        used += count * sizeof(T);
        return p;
    }
    bool fits() const { return used <= size; }
};

// Device address of this device's status word (resolved once per device).
unsigned int* status_word();

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace slimkv
