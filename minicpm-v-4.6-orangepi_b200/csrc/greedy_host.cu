// One greedy decoding step of the lm_head from host memory to a host token
// id in one native call: the reference's lm_head_greedy
// (src/csrc/lib/language_model.cpp:412-482) - final rms_norm, vocabulary
// GEMV, first-max argmax - which hands the token back to the host.  x rides in the launch parameters when small (else one copy-in),
// the fused GEMV + argmax stores the index straight into page-locked host
// memory (else one 8-byte copy-out), then the stream is synchronised: one
// library call and, for a 1024-wide row, one queued GPU operation per token.
#include <chrono>
#include <cstdint>

#include "common.cuh"

namespace mcv {
}  // namespace mcv

using namespace mcv;

extern "C" {

int mcv_lm_head_greedy_host(void* p2p_ctx, const void* x_host, void* x_dev, const void* norm_gamma, float norm_eps,
                            const void* w, void* index_dev, int64_t* index_host, int64_t M, int64_t K,
                            int64_t N_shard, int64_t n_offset, int fp16_logits, void* workspace,
                            size_t workspace_bytes, mcv_stream_t stream) {
    if (!x_host || !x_dev || !index_dev || !index_host) return fail(MCV_ERR_NULL, "lm_head_greedy_host: null pointer");
    if (M < 1 || M > 8 || K < 1) return fail(MCV_ERR_SHAPE, "lm_head_greedy_host: M must be 1..8");
    // x_host is read on the host when it travels in the launch: refuse
    // device memory rather than fault the process
    cudaPointerAttributes pa_in{};
    if (cudaPointerGetAttributes(&pa_in, x_host) == cudaSuccess) {
        if (pa_in.type == cudaMemoryTypeDevice)
            return fail(MCV_ERR_VALUE, "lm_head_greedy_host: x_host must be host memory");
    } else {
        (void)cudaGetLastError();  // unregistered host memory
    }
    auto s = static_cast<cudaStream_t>(stream);
    // lm_head_greedy's final rms_norm (language_model.cpp:423), fused into
    // the kernel's prologue when a gamma is given
    const NormArgs norm{static_cast<const __half*>(norm_gamma), norm_eps, 0};
    const P2PArgs* pa = nullptr;
    if (p2p_ctx) {
        int st = MCV_OK;
        pa = p2p_args_checked(p2p_ctx, n_offset, N_shard, &st);
        if (st) return st;
    }
    // Small activations (M * K <= 2048, e.g. one 1024-wide row) travel in
    // the launch parameters: no copy-in is queued before the kernel.
    const bool by_param = M * K <= 2048;
    if (!by_param) {
        cudaError_t e = cudaMemcpyAsync(x_dev, x_host, static_cast<size_t>(M * K) * 2, cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(x in)");
    }
    // Page-locked index_host is device-addressable: the kernel's last block
    // then stores the indices straight into it and no copy-out is queued.
    void* out = index_dev;
    cudaPointerAttributes pa_out{};
    if (cudaPointerGetAttributes(&pa_out, index_host) == cudaSuccess && pa_out.type == cudaMemoryTypeHost &&
        pa_out.devicePointer != nullptr)
        out = pa_out.devicePointer;
    else
        (void)cudaGetLastError();  // pageable memory: not an error, copy out below
    // With the index stored straight into page-locked memory, the host
    // watches that memory instead of waiting for the stream: the answer is
    // there as soon as the kernel's last block has stored it, ahead of the
    // grid's retirement and the stream's completion signal.
    constexpr int64_t kSentinel = INT64_MIN;
    volatile int64_t* watch = nullptr;
    if (out != index_dev) {
        watch = index_host;
        for (int64_t m = 0; m < M; ++m) watch[m] = kSentinel;
    }
    const int st = lm_head_argmax_impl_p2p(by_param ? nullptr : x_dev, w, nullptr, out, M, K, N_shard, n_offset,
                                           fp16_logits, workspace, workspace_bytes, s, pa,
                                           by_param ? x_host : nullptr, norm_gamma ? &norm : nullptr);
    if (st) return st;
    cudaError_t e = cudaSuccess;
    if (out == index_dev) {
        e = cudaMemcpyAsync(index_host, index_dev, static_cast<size_t>(M) * sizeof(int64_t), cudaMemcpyDeviceToHost,
                            s);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(index out)");
    }
    if (watch) {
        // bounded: after 10 s fall through to the stream wait, which reports
        // whatever stopped the kernel
        const auto t0 = std::chrono::steady_clock::now();
        for (uint32_t i = 1;; ++i) {
            bool all = true;
            for (int64_t m = 0; m < M; ++m) all = all && watch[m] != kSentinel;
            if (all) return MCV_OK;
            if ((i & 1023u) == 0 && std::chrono::steady_clock::now() - t0 > std::chrono::seconds(10)) break;
        }
    }
    e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
    return MCV_OK;
}

}  // extern "C"
