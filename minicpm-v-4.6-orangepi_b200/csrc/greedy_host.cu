// One greedy decoding step of the lm_head from host memory to a host token
// id in one native call: the device half of the reference's lm_head_greedy
// (src/csrc/lib/language_model.cpp:412-482), which hands the token back to
// the host.  Doing the copy in, the fused GEMV + argmax, the 8-byte copy out
// and the stream synchronisation in C keeps a decode loop's per-token host
// overhead to one library call.
#include "common.cuh"

using namespace mcv;

extern "C" {

int mcv_lm_head_greedy_host(void* p2p_ctx, const void* x_host, void* x_dev, const void* w, void* index_dev,
                            int64_t* index_host, int64_t M, int64_t K, int64_t N_shard, int64_t n_offset,
                            int fp16_logits, void* workspace, size_t workspace_bytes, mcv_stream_t stream) {
    if (!x_host || !x_dev || !index_dev || !index_host) return fail(MCV_ERR_NULL, "lm_head_greedy_host: null pointer");
    if (M < 1 || M > 8 || K < 1) return fail(MCV_ERR_SHAPE, "lm_head_greedy_host: M must be 1..8");
    auto s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(x_dev, x_host, static_cast<size_t>(M * K) * 2, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(x in)");
    // Page-locked index_host is device-addressable: the kernel's last block
    // then stores the indices straight into it and no copy-out is queued.
    void* out = index_dev;
    cudaPointerAttributes pa{};
    if (cudaPointerGetAttributes(&pa, index_host) == cudaSuccess && pa.type == cudaMemoryTypeHost &&
        pa.devicePointer != nullptr)
        out = pa.devicePointer;
    else
        (void)cudaGetLastError();  // pageable memory: not an error, copy out below
    const int st = p2p_ctx ? mcv_lm_head_argmax_p2p(p2p_ctx, x_dev, w, nullptr, out, M, K, N_shard, n_offset,
                                                    fp16_logits, workspace, workspace_bytes, stream)
                           : mcv_lm_head_argmax(x_dev, w, nullptr, out, M, K, N_shard, n_offset, fp16_logits,
                                                workspace, workspace_bytes, stream);
    if (st) return st;
    if (out == index_dev) {
        e = cudaMemcpyAsync(index_host, index_dev, static_cast<size_t>(M) * sizeof(int64_t), cudaMemcpyDeviceToHost,
                            s);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(index out)");
    }
    e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
    return MCV_OK;
}

}  // extern "C"
