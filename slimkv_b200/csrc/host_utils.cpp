#include "host_utils.h"

#include <cudaTypedefs.h>

#include <mutex>

namespace slimkv {

static thread_local std::string g_last_error;

void set_error(const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
}

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

const DeviceInfo& device_info() {
    static thread_local DeviceInfo info;
    int dev = 0;
    cudaGetDevice(&dev);
    if (info.device != dev) {
        info.device = dev;
        cudaDeviceGetAttribute(&info.sm_count, cudaDevAttrMultiProcessorCount, dev);
        cudaDeviceGetAttribute(&info.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    }
    return info;
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        void* p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

int encode_map_4d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                  uint64_t d3, uint64_t s1, uint64_t s2, uint64_t s3, uint32_t box_rows) {
    return encode_map_4d_box(map, base, d0, d1, d2, d3, s1, s2, s3, 1, box_rows);
}

int encode_map_4d_box(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t d3,
                      uint64_t s1, uint64_t s2, uint64_t s3, uint32_t box1, uint32_t box2) {
    auto fn = encode_fn();
    if (!fn) return fail(SLIMKV_ERR_TENSOR_MAP, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[4] = {d0, d1, d2, d3};
    cuuint64_t strides[3] = {s1, s2, s3};
    cuuint32_t box[4] = {64, box1, box2, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box,
                    estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(SLIMKV_ERR_TENSOR_MAP,
                    "cuTensorMapEncodeTiled failed (%d): dims {%llu,%llu,%llu,%llu} strides {%llu,%llu,%llu}",
                    int(r), (unsigned long long)d0, (unsigned long long)d1, (unsigned long long)d2,
                    (unsigned long long)d3, (unsigned long long)s1, (unsigned long long)s2,
                    (unsigned long long)s3);
    return SLIMKV_OK;
}

int encode_map_f32_3d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1,
                      uint64_t s2, uint32_t box0, uint32_t box1) {
    auto fn = encode_fn();
    if (!fn) return fail(SLIMKV_ERR_TENSOR_MAP, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[3] = {d0, d1, d2};
    cuuint64_t strides[2] = {s1, s2};
    cuuint32_t box[3] = {box0, box1, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(SLIMKV_ERR_TENSOR_MAP, "cuTensorMapEncodeTiled (f32) failed (%d): dims {%llu,%llu,%llu}", int(r),
                    (unsigned long long)d0, (unsigned long long)d1, (unsigned long long)d2);
    return SLIMKV_OK;
}

}  // namespace slimkv

extern "C" const char* slimkv_last_error(void) { return slimkv::g_last_error.c_str(); }
extern "C" int slimkv_version(void) { return 100; }
