// Vocab-sharded lm_head with the cross-GPU (max, index) reduction fused into
// the kernel over NVLink peer memory, in place of a separate NCCL all-reduce.
//
// Every rank owns a small mailbox (128 64-bit slots, 1 KB, plus a call
// counter and an error word) in its own HBM and maps every peer's mailbox
// through CUDA IPC.  The last block of each rank's fused lm_head + argmax
// kernel writes the rank's keys into all mailboxes, one relaxed system-scope
// 64-bit store per key and peer (the word carries the key and an 8-bit call
// tag together, so no fence is needed), waits (bounded, 1 s) for all peers'
// keys in its own mailbox, and writes the global winner - one kernel, no
// collective launch.  The call counter lives in device memory, so captured
// CUDA graphs replay correctly; slots alternate by counter parity.
//
// The reference has no multi-device code (it runs its 16 lm_head chunks one
// after another on one NPU, src/csrc/lib/language_model.cpp:464-480).
#include "common.cuh"

namespace mcv {

namespace {

constexpr size_t kMboxWords = 2 * 8 * 8;                   // [parity][rank][row]: key + call tag
constexpr int64_t kP2PMaxIndex = 0xffffff;                 // indices travel in 24 bits of a mailbox word
constexpr size_t kMboxBytes = (kMboxWords + 2) * sizeof(uint64_t);  // + call counter + error word

struct P2PCtx {
    int nranks = 0, rank = 0, device = 0;
    uint64_t* local = nullptr;  // own mailbox, counter at [kMboxWords], error word at [kMboxWords + 1]
    void* peers[8] = {};        // opened IPC mappings (nullptr for self)
    P2PArgs args{};
};

}  // namespace
// Connected context's kernel arguments for a call on rows
// [n_offset, n_offset + N); null with *status set when the call is invalid.
const P2PArgs* p2p_args_checked(void* ctx, int64_t n_offset, int64_t N, int* status) {
    auto* c = static_cast<P2PCtx*>(ctx);
    *status = MCV_OK;
    if (!c || !c->args.seq_dev) {
        *status = fail(MCV_ERR_NULL, "lm_head p2p: context not connected");
        return nullptr;
    }
    if (n_offset < 0 || N < 0 || n_offset + N > kP2PMaxIndex) {
        *status = fail(MCV_ERR_SHAPE, "lm_head p2p: vocabulary indices must stay below 2^24 - 1");
        return nullptr;
    }
    return &c->args;
}

}  // namespace mcv

using namespace mcv;

extern "C" {

size_t mcv_p2p_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int mcv_p2p_create(void** ctx_out, int nranks, int rank, void* handle_out) {
    if (!ctx_out || !handle_out) return fail(MCV_ERR_NULL, "p2p_create: null pointer");
    if (nranks < 1 || nranks > 8 || rank < 0 || rank >= nranks)
        return fail(MCV_ERR_VALUE, "p2p_create: nranks must be 1..8 and 0 <= rank < nranks");
    auto* c = new P2PCtx;
    c->nranks = nranks;
    c->rank = rank;
    cudaError_t e = cudaGetDevice(&c->device);
    if (e == cudaSuccess) e = cudaMalloc(&c->local, kMboxBytes);  // set-up time only
    if (e == cudaSuccess) e = cudaMemset(c->local, 0, kMboxBytes);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, c->local);
    if (e != cudaSuccess) {
        if (c->local) cudaFree(c->local);
        delete c;
        return cuda_fail(e, "p2p_create");
    }
    memcpy(handle_out, &h, sizeof(h));
    *ctx_out = c;
    return MCV_OK;
}

int mcv_p2p_connect(void* ctx, const void* all_handles) {
    auto* c = static_cast<P2PCtx*>(ctx);
    if (!c || !all_handles) return fail(MCV_ERR_NULL, "p2p_connect: null pointer");
    const auto* hs = static_cast<const cudaIpcMemHandle_t*>(all_handles);
    for (int r = 0; r < c->nranks; ++r) {
        if (r == c->rank) {
            c->args.mbox[r] = c->local;
            continue;
        }
        void* p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, hs[r], cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
        c->peers[r] = p;
        c->args.mbox[r] = static_cast<uint64_t*>(p);
    }
    c->args.seq_dev = c->local + kMboxWords;
    c->args.err = reinterpret_cast<unsigned*>(c->local + kMboxWords + 1);
    c->args.rank = c->rank;
    c->args.nranks = c->nranks;
    return MCV_OK;
}

int mcv_p2p_destroy(void* ctx) {
    auto* c = static_cast<P2PCtx*>(ctx);
    if (!c) return MCV_OK;
    for (int r = 0; r < 8; ++r)
        if (c->peers[r]) cudaIpcCloseMemHandle(c->peers[r]);
    if (c->local) cudaFree(c->local);
    delete c;
    return MCV_OK;
}

unsigned mcv_p2p_errors(void* ctx) {
    auto* c = static_cast<P2PCtx*>(ctx);
    if (!c || !c->args.err) return 0;
    unsigned v = 0;
    if (cudaMemcpy(&v, c->args.err, sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess) return ~0u;
    if (v) cudaMemset(c->args.err, 0, sizeof(v));
    return v;
}

int mcv_lm_head_argmax_p2p(void* ctx, const void* x, const void* w, void* out_key, void* out_index, int64_t M,
                           int64_t K, int64_t N_shard, int64_t n_offset, int fp16_logits, void* workspace,
                           size_t workspace_bytes, mcv_stream_t stream) {
    auto* c = static_cast<P2PCtx*>(ctx);
    if (!c || !c->args.seq_dev) return fail(MCV_ERR_NULL, "lm_head_argmax_p2p: context not connected");
    if (!out_key && !out_index) return fail(MCV_ERR_NULL, "lm_head_argmax_p2p: out_key and out_index both null");
    if (n_offset < 0 || N_shard < 0 || n_offset + N_shard > kP2PMaxIndex)
        return fail(MCV_ERR_SHAPE, "lm_head_argmax_p2p: vocabulary indices must stay below 2^24 - 1");
    return lm_head_argmax_impl_p2p(x, w, out_key, out_index, M, K, N_shard, n_offset, fp16_logits, workspace,
                                   workspace_bytes, static_cast<cudaStream_t>(stream), &c->args, nullptr,
                                   nullptr);
}

}  // extern "C"
