// Fused lm_head GEMV + greedy argmax for callers that cannot allocate device
// memory.
//
// mcv_lm_head_argmax needs a caller-provided workspace (one 64-bit key per
// block and row, plus a block counter).  Some callers have no way to provide
// one: code that runs where cudaMalloc is not allowed or not wanted (inside a
// host callback, under an allocator that must not grow, in a plugin whose host
// owns every device allocation).  This file gives them one entry point whose
// workspace is a fixed array in the library's own device memory, reserved
// when the library is loaded on a GPU and held until the process exits.
#include <mutex>

#include "common.cuh"

namespace mcv {

namespace {

// Large enough for mcv_lm_head_workspace_size(M) for every supported M: an
// arrival counter and one 64-bit running key per row.
constexpr size_t kNoAllocBytes = 256;

static __device__ __align__(256) unsigned char g_lm_head_scratch[kNoAllocBytes];

std::mutex g_mu;
void* g_scratch_ptr[64] = {};

// Device address of g_lm_head_scratch on the current device.  In host code
// the symbol's name only stands in for the array; the address a kernel may
// use comes from cudaGetSymbolAddress, looked up once per device.
int scratch_for_current_device(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev < 0 || dev >= 64) return fail(MCV_ERR_VALUE, "lm_head_argmax_noalloc: device index above 63");
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_lm_head_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_lm_head_scratch)");
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return MCV_OK;
}

}  // namespace
}  // namespace mcv

using namespace mcv;

extern "C" {

size_t mcv_lm_head_noalloc_max_bytes(void) { return kNoAllocBytes; }

int mcv_lm_head_argmax_noalloc(const void* x, const void* w, void* out_key, void* out_index, int64_t M,
                               int64_t K, int64_t N_shard, int64_t n_offset, int fp16_logits,
                               mcv_stream_t stream) {
    if (!out_key && !out_index) return fail(MCV_ERR_NULL, "lm_head_argmax_noalloc: out_key and out_index both null");
    if (M < 1 || M > 8) return fail(MCV_ERR_SHAPE, "lm_head_argmax_noalloc: M must be 1..8");
    const size_t need = mcv_lm_head_workspace_size(M);
    if (need > kNoAllocBytes)
        return fail(MCV_ERR_WORKSPACE, "lm_head_argmax_noalloc: request needs more than the fixed scratch array");
    void* ws = nullptr;
    int st = scratch_for_current_device(&ws);
    if (st) return st;
    auto s = static_cast<cudaStream_t>(stream);
    // The array keeps whatever the previous call left; its counter and
    // running keys must be zero when a call begins.
    cudaError_t e = cudaMemsetAsync(ws, 0, kNoAllocBytes, s);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(lm_head scratch)");
    return lm_head_argmax_impl(x, w, out_key, out_index, M, K, N_shard, n_offset, fp16_logits, ws, kNoAllocBytes, s);
}

}  // extern "C"
