// Shared device helpers and host-side error plumbing of the Pop-KV B200 library.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>

#include "popkv_b200.h"

namespace popkv {

// ---------------------------------------------------------------- host side
void set_error(const char* fmt, ...);
int fail(int status, const char* fmt, ...);
int check_launch(const char* what);

inline cudaStream_t as_stream(popkv_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

inline size_t dtype_size(int dtype) {
    switch (dtype) {
        case POPKV_F32: return 4;
        case POPKV_F16: return 2;
        case POPKV_BF16: return 2;
        default: return 0;
    }
}

// Programmatic dependent launch: every kernel of the library is launched with
// programmatic stream serialization, lets its dependents launch at once
// (pdl_trigger) and waits for its predecessor's results (pdl_wait) before reading
// them, so a kernel's launch and set-up overlap the tail of the one before it.
// Without a predecessor launched this way both are no-ops.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// SM count of the current device (queried once per device).
inline int num_sms() {
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 148;
    if (dev < 64 && cached[dev] > 0) return cached[dev];
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    if (dev < 64) cached[dev] = n;
    return n;
}

// launch_pdl for a kernel launched in clusters of `cluster_x` CTAs along x.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                               cudaStream_t st, unsigned cluster_x, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cluster_x;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// --------------------------------------------------------------- device side
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::); }

template <typename T> __device__ __forceinline__ float to_float(T v);
template <> __device__ __forceinline__ float to_float<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_float<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_float<__nv_bfloat16>(__nv_bfloat16 v) {
    return __bfloat162float(v);
}

template <typename T> __device__ __forceinline__ T from_float(float v);
template <> __device__ __forceinline__ float from_float<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_float<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float v) {
    return __float2bfloat16_rn(v);
}

// Representative division.  Default: IEEE round-to-nearest.  With reference
// division the PTX full-range approximate divide is issued instead, which is what
// a --use_fast_math build (the reference's JIT flags) uses for float '/'.
__device__ __forceinline__ float rep_div(float a, float b, bool reference_division) {
    if (reference_division) {
        float r;
        asm("div.full.ftz.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
        return r;
    }
    return __fdiv_rn(a, b);
}

// Mean of the low / high lanes with the reference's fallbacks
// (csrc/popkv_ext.cu:77-83 and 139-145).
__device__ __forceinline__ void representatives(float low_sum, int low_count, float high_sum,
                                                int high_count, bool ref_div, float& low,
                                                float& high) {
    if (low_count == 0) {
        low = high_count ? rep_div(high_sum, static_cast<float>(high_count), ref_div) : 0.0f;
        high = low;
    } else {
        low = rep_div(low_sum, static_cast<float>(low_count), ref_div);
        high = high_count ? rep_div(high_sum, static_cast<float>(high_count), ref_div) : low;
    }
}

// ------------------------------------------- mbarriers and bulk (TMA) copies
// Plain global -> shared bulk copies completed on an mbarrier's transaction count;
// no multicast anywhere.
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_addr(bar)) : "memory");
}
// Bulk prefetch of [p, p + bytes) into L2 (p 16-byte aligned, bytes a multiple of 16).
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    if ((reinterpret_cast<uintptr_t>(p) & 15u) != 0u || bytes == 0u) return;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(p), "r"(bytes) : "memory");
}
// bytes: a multiple of 16; both addresses 16-byte aligned.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n"
                 ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
                 " selp.u32 %0, 1, 0, p;\n}\n"
                 : "=r"(done) : "r"(smem_addr(bar)), "r"(parity) : "memory");
    return done != 0;
}
__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// try_wait that lets the hardware suspend the thread until the phase completes or
// about `hint_ns` pass, instead of returning at once (no busy polling).
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t done;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
                 " selp.u32 %0, 1, 0, p;\n}\n"
                 : "=r"(done) : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns) : "memory");
    return done != 0;
}
// Waits for phase `parity` of the barrier for at most ~limit_ns; false if it ran out.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  unsigned long long limit_ns = 2000000000ull) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer_ns();
    while (!mbar_try_wait_suspend(bar, parity, 1000000u))
        if (globaltimer_ns() - t0 > limit_ns) return false;
    return true;
}

__host__ __device__ __forceinline__ int64_t imin64(int64_t a, int64_t b) { return a < b ? a : b; }

// Order-preserving map of fp32 to uint32 (larger float -> larger key); -0.0 maps
// like +0.0 so that the two compare equal, as float comparison does.
__device__ __forceinline__ uint32_t order_key(float x) {
    uint32_t u = __float_as_uint(x);
    if (u == 0x80000000u) u = 0u;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

}  // namespace popkv
