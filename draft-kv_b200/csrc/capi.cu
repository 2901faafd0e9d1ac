// Error reporting, version and the device error word shared by all kernels.
#include <stdarg.h>
#include <stdio.h>

#include <vector>

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

// ------------------------------------------------------------------ profiling
namespace {
struct ProfRec {
    int kind;
    double bytes;
    cudaEvent_t a, b;
};
struct Prof {
    bool on = false;
    int used = 0;
    std::vector<ProfRec> recs;
} g_prof;
}  // namespace

ProfScope::ProfScope(int kind, double bytes, cudaStream_t s) : st(s) {
    if (!g_prof.on || g_prof.used >= (int)g_prof.recs.size()) return;
    slot = g_prof.used++;
    g_prof.recs[slot].kind = kind;
    g_prof.recs[slot].bytes = bytes;
    cudaEventRecord(g_prof.recs[slot].a, st);
}

ProfScope::~ProfScope() {
    if (slot >= 0) cudaEventRecord(g_prof.recs[slot].b, st);
}

}  // namespace dkv

extern "C" int dkv_prof_start(int max_records) {
    using dkv::g_prof;
    DKV_REQUIRE(max_records > 0 && max_records <= (1 << 20), "dkv_prof_start: max_records");
    while ((int)g_prof.recs.size() < max_records) {
        dkv::ProfRec r{};
        DKV_CUDA(cudaEventCreate(&r.a));
        DKV_CUDA(cudaEventCreate(&r.b));
        g_prof.recs.push_back(r);
    }
    g_prof.used = 0;
    g_prof.on = true;
    return DKV_OK;
}

extern "C" int dkv_prof_stop(void) {
    dkv::g_prof.on = false;
    return DKV_OK;
}

extern "C" int dkv_prof_summary(int kind, double* total_ms, int64_t* launches, double* total_bytes) {
    using dkv::g_prof;
    DKV_REQUIRE(total_ms && launches && total_bytes, "dkv_prof_summary: outputs required");
    *total_ms = 0.0;
    *launches = 0;
    *total_bytes = 0.0;
    for (int i = 0; i < g_prof.used; ++i) {
        const dkv::ProfRec& r = g_prof.recs[i];
        if (r.kind != kind) continue;
        DKV_CUDA(cudaEventSynchronize(r.b));
        float ms = 0.f;
        DKV_CUDA(cudaEventElapsedTime(&ms, r.a, r.b));
        *total_ms += ms;
        *launches += 1;
        *total_bytes += r.bytes;
    }
    return DKV_OK;
}

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
