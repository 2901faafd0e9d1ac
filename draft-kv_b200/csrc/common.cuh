// Shared helpers for the draftkv_b200 kernels (sm_100a).
#pragma once

#include <atomic>
#include <utility>

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stddef.h>

#include "../../include/draftkv_b200.h"

#define DKV_DEV __device__ __forceinline__

namespace dkv {

// ------------------------------------------------------------------ errors
void set_error(const char* fmt, ...);

#define DKV_REQUIRE(cond, ...)                                   \
    do {                                                         \
        if (!(cond)) {                                           \
            ::dkv::set_error(__VA_ARGS__);                       \
            return DKV_EINVAL;                                   \
        }                                                        \
    } while (0)

#define DKV_UNSUPPORTED(cond, ...)                               \
    do {                                                         \
        if (!(cond)) {                                           \
            ::dkv::set_error(__VA_ARGS__);                       \
            return DKV_EUNSUPPORTED;                             \
        }                                                        \
    } while (0)

#define DKV_CUDA(expr)                                                         \
    do {                                                                       \
        cudaError_t e_ = (expr);                                               \
        if (e_ != cudaSuccess) {                                               \
            ::dkv::set_error("%s failed: %s (%s:%d)", #expr,                  \
                             cudaGetErrorString(e_), __FILE__, __LINE__);      \
            return DKV_ECUDA;                                                  \
        }                                                                      \
    } while (0)

#define DKV_LAUNCHED() DKV_CUDA(cudaGetLastError())

#define DKV_TRY(expr)                         \
    do {                                      \
        int s_ = (expr);                      \
        if (s_ != DKV_OK) return s_;          \
    } while (0)

// Sets the dynamic shared memory limit of a kernel once per process.
template <typename K>
inline cudaError_t allow_smem(K kernel, size_t bytes) {
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

// Raises a kernel's dynamic shared memory limit to the device's opt-in
// maximum minus the kernel's static shared memory.
template <typename K>
inline cudaError_t allow_smem_max(K kernel) {
    int dev = 0, optin = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaFuncAttributes fa;
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, kernel);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)fa.sharedSizeBytes);
}

// Once-per-device set-up (kernel attributes such as the shared-memory limit
// apply to the current device only, so every device needs its own call).
// run(fn) calls fn() the first time it is reached with a given current device
// and remembers a success; two threads racing on the first call may both run
// fn, which must therefore be idempotent.  Devices beyond 63 run fn on every
// call.  A cudaDeviceReset() discards the attributes but not these flags:
// calls must not cross a reset of a device they have already used.
struct DeviceOnce {
    std::atomic<uint64_t> done{0};
    template <typename F>
    cudaError_t run(F&& fn) {
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        const uint64_t bit = dev >= 0 && dev < 64 ? (1ull << dev) : 0ull;
        if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
        e = fn();
        if (e == cudaSuccess && bit) done.fetch_or(bit, std::memory_order_acq_rel);
        return e;
    }
};

// allow_smem_max(Kern) once per device (one flag set per kernel: the kernel
// is a template argument, not a runtime value).
template <auto Kern>
inline cudaError_t allow_smem_max_once() {
    static DeviceOnce once;
    return once.run([] { return allow_smem_max(Kern); });
}

// Bytes of one drafter-cache vector of d elements at `bits` per element
// (16: raw entries of raw_dtype).  A layer's vectors are stored densely at
// this stride inside each (sequence, layer, head) region of cap x cb_max
// bytes, so a narrow configuration streams contiguous bytes.
__host__ __device__ inline int code_row_bytes(int d, int bits, int raw_dtype) {
    return bits >= 16 ? d * (raw_dtype == DKV_F32 ? 4 : 2) : d * bits / 8;
}

// ---- mbarrier / bulk-copy helpers (TMA without multicast: each copy lands
// in the issuing CTA's own shared memory)
DKV_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
DKV_DEV void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count));
}
DKV_DEV void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }
DKV_DEV void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
DKV_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
DKV_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: gives up after ~2^22 polls (each poll may suspend briefly),
// records 0x80 in the device error word and returns false.
DKV_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err) {
    for (uint32_t i = 0; i < (1u << 22); ++i)
        if (mbar_try_wait(bar, parity)) return true;
    if (err) atomicOr(err, 0x80u);
    return false;
}

// Programmatic dependent launch.  A kernel launched with launch_pdl() may
// start while the previous kernel on the stream is still running: it must
// execute pdl_wait() before it reads anything an earlier kernel wrote or
// writes anything an earlier kernel reads.  pdl_trigger() lets the next
// kernel start early (it still waits for this one to complete in its own
// pdl_wait()).  Both are no-ops for kernels launched the ordinary way.
DKV_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
DKV_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" :::); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Bump allocator over a caller-provided scratch buffer.
struct Arena {
    char* base;
    size_t cap, used;
    Arena(void* p, size_t n) : base((char*)p), cap(n), used(0) {}
    template <typename T>
    T* take(size_t count) {
        size_t off = align_up(used, 256);
        size_t need = off + count * sizeof(T);
        if (need > cap || base == nullptr) return nullptr;
        used = need;
        return reinterpret_cast<T*>(base + off);
    }
};

// ------------------------------------------------------------------ profiling
// Optional CUDA-event timing of each launch by kernel class (dkv_prof_*).
// When profiling is off a ProfScope costs one branch.
struct ProfScope {
    int slot = -1;
    cudaStream_t st;
    ProfScope(int kind, double bytes, cudaStream_t s);
    ~ProfScope();
};

// ------------------------------------------------------------------ types
DKV_DEV float to_f32(float v) { return v; }
DKV_DEV float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
DKV_DEV float bf16_bits_to_f32(uint16_t b) { return __uint_as_float(((uint32_t)b) << 16); }
DKV_DEV uint16_t f32_to_bf16_bits(float f) {
    __nv_bfloat16 h = __float2bfloat16_rn(f);
    return *reinterpret_cast<uint16_t*>(&h);
}
DKV_DEV float half_bits_to_f32(uint16_t b) {
    __half h = *reinterpret_cast<__half*>(&b);
    return __half2float(h);
}
DKV_DEV uint16_t f32_to_half_bits(float f) {
    __half h = __float2half_rn(f);
    return *reinterpret_cast<uint16_t*>(&h);
}

// Loads element i of a buffer of dtype DKV_F32 / DKV_BF16 as f32.
DKV_DEV float load_as_f32(const void* p, int dtype, size_t i) {
    return dtype == DKV_F32 ? reinterpret_cast<const float*>(p)[i]
                            : bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(p)[i]);
}
DKV_DEV void store_from_f32(void* p, int dtype, size_t i, float v) {
    if (dtype == DKV_F32)
        reinterpret_cast<float*>(p)[i] = v;
    else
        reinterpret_cast<uint16_t*>(p)[i] = f32_to_bf16_bits(v);
}

// ------------------------------------------------------------------ reductions
// Butterfly reductions followed by a broadcast of lane 0, so every lane holds
// the bit-identical value whatever the lane.
DKV_DEV float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return __shfl_sync(0xffffffffu, v, 0);
}
DKV_DEV float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
DKV_DEV float warp_min(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
DKV_DEV double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return __shfl_sync(0xffffffffu, v, 0);
}
DKV_DEV unsigned long long warp_min_u64(unsigned long long v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
        v = w < v ? w : v;
    }
    return v;
}
DKV_DEV int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
DKV_DEV int warp_max_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide sum in a fixed order (warp partials summed by warp 0 in order).
// `red` must hold 32 floats; all threads must call; result in every thread.
DKV_DEV float block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    if (wid == 0) {
        float t = lane < nw ? red[lane] : 0.f;
        t = warp_sum(t);
        if (lane == 0) red[0] = t;
    }
    __syncthreads();
    return red[0];
}
DKV_DEV float block_max(float v, float* red) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    if (wid == 0) {
        float t = lane < nw ? red[lane] : -INFINITY;
        t = warp_max(t);
        if (lane == 0) red[0] = t;
    }
    __syncthreads();
    return red[0];
}

// ------------------------------------------------------------------ Philox
// Philox4x32-10 counter-based generator (Salmon, Moraes, Dror, Shaw,
// "Parallel random numbers: as easy as 1, 2, 3", SC'11): ten rounds of two
// 32x32->64 multiplies with the published multipliers and Weyl key bumps.
struct U4 { uint32_t x, y, z, w; };

DKV_DEV U4 philox4x32_10(U4 ctr, uint32_t k0, uint32_t k1) {
    const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
    const uint32_t W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        uint32_t hi0 = __umulhi(M0, ctr.x), lo0 = M0 * ctr.x;
        uint32_t hi1 = __umulhi(M1, ctr.z), lo1 = M1 * ctr.z;
        U4 n;
        n.x = hi1 ^ ctr.y ^ k0;
        n.y = lo1;
        n.z = hi0 ^ ctr.w ^ k1;
        n.w = lo0;
        ctr = n;
        k0 += W0;
        k1 += W1;
    }
    return ctr;
}

// Uniform double in [0, 1) from 53 random bits.
DKV_DEV double philox_uniform(uint64_t seed, uint64_t counter, uint32_t stream, uint32_t sub) {
    U4 c{(uint32_t)counter, (uint32_t)(counter >> 32), stream, sub};
    U4 r = philox4x32_10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
    uint64_t bits = ((uint64_t)r.x << 21) ^ ((uint64_t)r.y >> 11);
    bits &= ((1ull << 53) - 1);
    return (double)bits * (1.0 / 9007199254740992.0);
}

}  // namespace dkv
