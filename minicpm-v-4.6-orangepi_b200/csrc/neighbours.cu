// Stand-alone rms_norm and silu_mul: the element-wise neighbours of the
// decode GEMVs, for callers that do not use the fused forms
// (mcv_lm_head_argmax with a norm, mcv_w4a16_gemv_silu_mul).
//
// Reference behaviour replaced: rms_norm (src/csrc/lib/ops.cpp:564-737),
// rms_norm1024 (ops.cpp:536-562, kernel op_kernel/rms_norm1024_custom.cpp)
// and silu_mul (ops.cpp:437-456, kernel op_kernel/silu_mul_custom.cpp).  The
// arithmetic is in neighbours.cuh.  Both are HBM-bound and tiny at decode
// (one 1024- or 3584-wide row): one block per row for the norm, a grid-stride
// loop over 16-byte vectors for silu_mul.
#include "neighbours.cuh"

namespace mcv {
namespace {

constexpr int kNormThreads = 256;

__global__ void __launch_bounds__(kNormThreads)
rms_norm_kernel(const __half* __restrict__ x, __half* __restrict__ out, int H, NormArgs na) {
    pdl_trigger();
    pdl_wait();
    const int64_t row = blockIdx.x;
    rms_norm_rows_block<1>(x + row * H, out + row * H, H, na);
}

constexpr int kSiluThreads = 256;

__global__ void __launch_bounds__(kSiluThreads)
silu_mul_kernel(const __half* __restrict__ g, const __half* __restrict__ u, __half* __restrict__ out, int64_t n) {
    pdl_trigger();
    pdl_wait();
    const int64_t stride = static_cast<int64_t>(gridDim.x) * kSiluThreads;
    const int64_t nv = n / 8;
    const uint4* g4 = reinterpret_cast<const uint4*>(g);
    const uint4* u4 = reinterpret_cast<const uint4*>(u);
    uint4* o4 = reinterpret_cast<uint4*>(out);
    for (int64_t i = blockIdx.x * static_cast<int64_t>(kSiluThreads) + threadIdx.x; i < nv; i += stride)
        o4[i] = silu_mul8(g4[i], u4[i]);
    for (int64_t i = nv * 8 + blockIdx.x * static_cast<int64_t>(kSiluThreads) + threadIdx.x; i < n; i += stride)
        out[i] = silu_mul1(g[i], u[i]);
}

}  // namespace

int check_norm(const void* gamma, int variant, int64_t H) {
    if (!gamma) return fail(MCV_ERR_NULL, "rms_norm: null gamma");
    if (variant != 0 && variant != 1) return fail(MCV_ERR_VALUE, "rms_norm: variant must be 0 (engine chain) or 1 (fp32)");
    if (H < 1 || H > (1 << 20)) return fail(MCV_ERR_SHAPE, "rms_norm: bad hidden size");
    return MCV_OK;
}

}  // namespace mcv

using namespace mcv;

extern "C" {

int mcv_rms_norm(const void* x, const void* gamma, void* out, int64_t rows, int64_t H, float eps, int variant,
                 mcv_stream_t stream) {
    if (!x || !out) return fail(MCV_ERR_NULL, "rms_norm: null x or out");
    int st = check_norm(gamma, variant, H);
    if (st) return st;
    if (rows < 1 || rows > 0x7fffffffLL) return fail(MCV_ERR_SHAPE, "rms_norm: rows must be positive");
    NormArgs na{static_cast<const __half*>(gamma), eps, variant};
    return launch(rms_norm_kernel, dim3(static_cast<unsigned>(rows)), dim3(kNormThreads), 0,
                  static_cast<cudaStream_t>(stream), static_cast<const __half*>(x), static_cast<__half*>(out),
                  static_cast<int>(H), na);
}

int mcv_silu_mul(const void* gate, const void* up, void* out, int64_t n, mcv_stream_t stream) {
    if (!gate || !up || !out) return fail(MCV_ERR_NULL, "silu_mul: null pointer");
    if (n < 1) return fail(MCV_ERR_SHAPE, "silu_mul: n must be positive");
    if (!aligned16(gate) || !aligned16(up) || !aligned16(out))
        return fail(MCV_ERR_ALIGN, "silu_mul: pointers must be 16-byte aligned");
    const int64_t want = (n / 8 + kSiluThreads - 1) / kSiluThreads;
    const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
    const int grid = static_cast<int>(want < 1 ? 1 : (want < cap ? want : cap));
    return launch(silu_mul_kernel, dim3(grid), dim3(kSiluThreads), 0, static_cast<cudaStream_t>(stream),
                  static_cast<const __half*>(gate), static_cast<const __half*>(up), static_cast<__half*>(out), n);
}

}  // extern "C"
