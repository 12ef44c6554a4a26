// Per-device status word that kernels set instead of trapping or hanging.
#include "host_utils.h"

namespace slimkv {

__device__ unsigned int g_device_status;

unsigned int* status_word() {
    static unsigned int* cache[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return nullptr;
    if (!cache[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_device_status) != cudaSuccess) return nullptr;
        cache[dev] = static_cast<unsigned int*>(p);
    }
    return cache[dev];
}

}  // namespace slimkv

extern "C" int slimkv_device_status(unsigned int* status, int clear) {
    unsigned int value = 0;
    if (cudaDeviceSynchronize() != cudaSuccess ||
        cudaMemcpyFromSymbol(&value, slimkv::g_device_status, sizeof(value)) != cudaSuccess)
        return slimkv::fail(SLIMKV_ERR_CUDA, "reading the device status word failed");
    if (clear) {
        const unsigned int zero = 0;
        if (cudaMemcpyToSymbol(slimkv::g_device_status, &zero, sizeof(zero)) != cudaSuccess)
            return slimkv::fail(SLIMKV_ERR_CUDA, "clearing the device status word failed");
    }
    if (status) *status = value;
    return SLIMKV_OK;
}
