// Error reporting, version and the device error word shared by all kernels.
#include <stdarg.h>
#include <stdio.h>

#include "common.cuh"

namespace dkv {

static thread_local char g_err[1024] = "";

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

// One word per device that kernels OR error bits into instead of trapping:
//   0x10 append rows over the per-call limit   0x20 drafter slot capacity
//   0x40 attention scratch too small           0x80 bounded wait expired
__device__ uint32_t g_device_error;

uint32_t* device_error_word() {
    static thread_local int cached_dev = -1;
    static thread_local uint32_t* cached = nullptr;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev != cached_dev || cached == nullptr) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
        cached = (uint32_t*)p;
        cached_dev = dev;
    }
    return cached;
}

}  // namespace dkv

extern "C" const char* dkv_last_error(void) { return dkv::g_err; }

extern "C" int dkv_version(void) { return 10000; }

extern "C" int dkv_device_error(uint32_t* out_code, void* stream) {
    DKV_REQUIRE(out_code != nullptr, "out_code is NULL");
    uint32_t* w = dkv::device_error_word();
    DKV_REQUIRE(w != nullptr, "device error word unavailable");
    cudaStream_t st = (cudaStream_t)stream;
    DKV_CUDA(cudaMemcpyAsync(out_code, w, sizeof(uint32_t), cudaMemcpyDeviceToHost, st));
    DKV_CUDA(cudaStreamSynchronize(st));
    DKV_CUDA(cudaMemsetAsync(w, 0, sizeof(uint32_t), st));
    DKV_CUDA(cudaStreamSynchronize(st));
    return DKV_OK;
}
