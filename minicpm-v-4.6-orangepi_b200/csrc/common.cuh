// Shared helpers of libmcv_b200: status plumbing, launch helper with
// programmatic dependent launch, and the small inline-PTX primitives the
// GEMV kernels share.  sm_100a only.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <string>

#include "mcv_matmul.h"

namespace mcv {

// ---- status ---------------------------------------------------------------

void set_error(const std::string& msg);
int fail(int status, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);
bool pdl_enabled();
int tuning(int key);

#define MCV_CHECK_CUDA(expr)                                   \
    do {                                                       \
        cudaError_t _e = (expr);                               \
        if (_e != cudaSuccess) return ::mcv::cuda_fail(_e, #expr); \
    } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Launches `kernel` with the PDL attribute when enabled, so its prologue (the
// weight prefetch) overlaps the tail of the previous kernel on the stream.
template <typename... KArgs, typename... Args>
int launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
           Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
    if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx");
    return MCV_OK;
}

int sm_count();

// ---- device primitives ---------------------------------------------------

// Programmatic dependent launch controls (no-ops when launched without PDL).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// 16-byte streaming load of data read exactly once (weights): non-coherent
// path, no L1 allocation.
__device__ __forceinline__ uint4 ld_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    // (a & b) | c
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// acc_lo += lo(a)*lo(b); acc_hi += hi(a)*hi(b): fp16 operands, fp32
// accumulation in one rounding (sm_100 mixed-precision FMA).
__device__ __forceinline__ void fma2_f16_f32(float& acc_lo, float& acc_hi, uint32_t a,
                                             uint32_t b) {
    asm("{\n\t.reg .f16 al, ah, bl, bh;\n\t"
        "mov.b32 {al, ah}, %2;\n\t"
        "mov.b32 {bl, bh}, %3;\n\t"
        "fma.rn.f32.f16 %0, al, bl, %0;\n\t"
        "fma.rn.f32.f16 %1, ah, bh, %1;\n\t}"
        : "+f"(acc_lo), "+f"(acc_hi)
        : "r"(a), "r"(b));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ uint64_t warp_max_u64(uint64_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const uint64_t u = __shfl_xor_sync(0xffffffffu, v, o);
        v = u > v ? u : v;
    }
    return v;
}

// Order-preserving argmax key: larger logit -> larger key; equal logits ->
// smaller index wins.  -0 is folded into +0 so it ties with +0 like a float
// comparison does.
__device__ __forceinline__ uint64_t argmax_key(float logit, uint32_t index) {
    uint32_t u = __float_as_uint(logit + 0.0f);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return (static_cast<uint64_t>(u) << 32) | static_cast<uint64_t>(0xffffffffu - index);
}

__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u32_as_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

}  // namespace mcv
