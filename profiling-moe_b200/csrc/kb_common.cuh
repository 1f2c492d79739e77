// Shared device/host helpers for libkolibri_b200 (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/kolibri_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libkolibri_b200 is built for sm_100a only"
#endif

namespace kb {

constexpr unsigned FULL_MASK = 0xffffffffu;
constexpr int WARP = 32;
constexpr int E_MAX = 512;   // largest expert count any kernel accepts

// ------------------------------------------------------------------------------------
// Programmatic dependent launch.  Every kernel calls pdl_wait() before its first global
// memory access and pdl_launch() right after it, so a dependent kernel launched with the
// programmatic-serialization attribute overlaps only its launch and block scheduling
// with this kernel's tail.  Both are no-ops for a kernel launched without the attribute.
// ------------------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// Host: launch with optional PDL attribute.  Returns a cudaError_t (0 = success).
bool pdl_enabled();

// Host: multiprocessor count of the current device (cached per device; 148 on B200).
int device_sm_count();

// Host: the poll limit of the kernels' bounded waits (kb_set_wait_limit), or dflt when none
// was set.
long long wait_limit(long long dflt);

// Host: byte offsets of the error words in the workspaces, and the device address of the
// static scratch of kb_expert_maps_noalloc on the current device (resolved on first use).
size_t maps_err_offset();
size_t chain_err_offset();
size_t ep_err_offset();
int noalloc_scratch_address(void** out);

template <typename... KArgs, typename... Args>
inline int launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                  cudaStream_t stream, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    if (pdl_enabled()) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
    return static_cast<int>(err);
}

// Set the dynamic shared memory limit of a kernel once per process (per kernel).
template <typename... KArgs>
inline int allow_smem(void (*kernel)(KArgs...), size_t bytes) {
    if (bytes <= 48 * 1024) return 0;
    return static_cast<int>(cudaFuncSetAttribute(
        kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)));
}

// ------------------------------------------------------------------------------------
// Element conversion for the activation dtypes.
// ------------------------------------------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<__nv_bfloat16> {
    static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
    static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};
template <> struct Elem<__half> {
    static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
    static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};
template <> struct Elem<float> {
    static __device__ __forceinline__ float to_f(float v) { return v; }
    static __device__ __forceinline__ float from_f(float v) { return v; }
};

// 16-byte vector of activation elements.
template <typename T> struct Vec16 {
    static constexpr int N = 16 / sizeof(T);
    union { uint4 u; T e[N]; };
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL_MASK, v, o);
    return v;
}

__device__ __forceinline__ int warp_incl_scan(int v, int lane) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int n = __shfl_up_sync(FULL_MASK, v, o);
        if (lane >= o) v += n;
    }
    return v;
}

// Streaming 16-byte load that does not allocate in L1 (data read once).
__device__ __forceinline__ uint4 ld_stream(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}
__device__ __forceinline__ float4 ld_stream_f4(const float* p) {
    float4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w) : "l"(p));
    return r;
}
// 16-byte store with evict-first policy (written once, not re-read by this kernel).
__device__ __forceinline__ void st_stream(void* p, uint4 v) {
    asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};"
                 :: "l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace kb
