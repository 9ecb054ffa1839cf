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

// Same, as thread-block clusters of the given shape (1x1x1: none).
template <typename... KArgs, typename... Args>
int launch_clustered(void (*kernel)(KArgs...), dim3 grid, dim3 block, dim3 cluster, size_t smem,
                     cudaStream_t stream, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    unsigned n = 0;
    if (cluster.x * cluster.y * cluster.z > 1) {
        attr[n].id = cudaLaunchAttributeClusterDimension;
        attr[n].val.clusterDim.x = cluster.x;
        attr[n].val.clusterDim.y = cluster.y;
        attr[n].val.clusterDim.z = cluster.z;
        ++n;
    }
    if (pdl_enabled()) {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
    if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx");
    return MCV_OK;
}

int sm_count();

// Cross-GPU exchange of the argmax keys through peer mailboxes (see
// p2p.cu).  nranks <= 1 disables it.  Mailbox of rank r, in 64-bit words:
// [parity 2][source rank 8][row 8], one word each (key and call tag);
// written by every rank over NVLink with plain stores, read only by its owner.
struct P2PArgs {
    uint64_t* mbox[8];   // mailbox of each rank, as addressable from this GPU
    uint64_t* seq_dev;   // this rank's call counter (device memory)
    unsigned* err;       // this rank's error word
    int rank, nranks;
};

// rms_norm applied to the activation rows in a kernel's prologue (see
// neighbours.cuh for the arithmetic).
struct NormArgs {
    const __half* gamma;  // null: no normalisation
    float eps;
    int variant;          // 0: the engine's fp16 chain with (1 + gamma); 1: the fp32 kernel with gamma
};

// The fused lm_head GEMV + argmax (dense.cu), shared by every lm_head entry
// point.  p2p (may be null): cross-GPU exchange in the last block.  x_param
// (host memory, may be null): when set and M * K <= 2048, x rides in the
// launch parameters and `x` is not read.  norm (may be null): rms_norm of x
// first.
int lm_head_argmax_impl_p2p(const void* x, const void* w, void* out_key, void* out_index, int64_t M, int64_t K,
                            int64_t N, int64_t n_offset, int fp16_logits, void* ws, size_t ws_bytes,
                            cudaStream_t s, const P2PArgs* p2p, const void* x_param, const NormArgs* norm);
int lm_head_argmax_impl(const void* x, const void* w, void* out_key, void* out_index, int64_t M, int64_t K,
                        int64_t N, int64_t n_offset, int fp16_logits, void* ws, size_t ws_bytes, cudaStream_t s);
const P2PArgs* p2p_args_checked(void* ctx, int64_t n_offset, int64_t N, int* status);

// Device-side error bits: kernels OR one in when a bounded wait gives up.
enum : unsigned { kDevErrTimeout = 1u };

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
// comparison does.  A NaN logit gets the lowest ordered value (below -inf),
// so it never beats a number: the reference's scan `v > best` is false for
// every NaN (src/csrc/lib/language_model.cpp:474-477).
__device__ __forceinline__ uint64_t argmax_key(float logit, uint32_t index) {
    uint32_t u = __float_as_uint(logit + 0.0f);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    if (logit != logit) u = 0u;
    return (static_cast<uint64_t>(u) << 32) | static_cast<uint64_t>(0xffffffffu - index);
}

// ---- mbarrier + bulk-copy (TMA) primitives, single-CTA scope ------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait on an mbarrier phase: gives up after ~2 s of wall time and
// returns false so the kernel can record an error and exit instead of hanging.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 0 && globaltimer_ns() - t0 > 2000000000ull) return false;
    }
}

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`
// (no multicast).  dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

// The barrier's pending count drops once this thread's earlier cp.async
// copies have landed (counted in the barrier's initial arrival count).
__device__ __forceinline__ void cp_async_mbar_arrive(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Orders this thread's generic-proxy shared-memory accesses before later
// async-proxy (bulk copy) writes to the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u32_as_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

}  // namespace mcv
