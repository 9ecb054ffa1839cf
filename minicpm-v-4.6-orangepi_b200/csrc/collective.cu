// Vocab-sharded lm_head across the GPUs of one node: each rank runs the fused
// GEMV + argmax over its contiguous slice of the tied embedding, then one
// NCCL all-reduce (max) of the 64-bit argmax keys over NVLink/NVSwitch gives
// every rank the global first-max index.
//
// The reference runs its 16 lm_head chunks one after another on a single NPU
// (src/csrc/lib/language_model.cpp:464-480) and has no collective; the chunk
// loop is the seam where vocab rows are split over ranks here.  Because the
// key packs (ordered logit bits, 0xFFFFFFFF - index), max over keys equals the
// reference's strict '>' scan over the whole vocabulary.
#include <nccl.h>

#include "common.cuh"

namespace mcv {
int key_to_index_impl(const void* key, void* out_index, int64_t M, cudaStream_t s);

namespace {
int nccl_fail(ncclResult_t r, const char* what) {
    return fail(MCV_ERR_NCCL, std::string(what) + ": " + ncclGetErrorString(r));
}
}  // namespace
}  // namespace mcv

using namespace mcv;

extern "C" {

size_t mcv_nccl_unique_id_bytes(void) { return sizeof(ncclUniqueId); }

int mcv_nccl_get_unique_id(void* id_out) {
    if (!id_out) return fail(MCV_ERR_NULL, "nccl_get_unique_id: null pointer");
    ncclUniqueId id;
    ncclResult_t r = ncclGetUniqueId(&id);
    if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
    memcpy(id_out, &id, sizeof(id));
    return MCV_OK;
}

int mcv_nccl_comm_init(void** comm_out, int nranks, const void* id, int rank) {
    if (!comm_out || !id) return fail(MCV_ERR_NULL, "nccl_comm_init: null pointer");
    if (nranks < 1 || rank < 0 || rank >= nranks) return fail(MCV_ERR_VALUE, "nccl_comm_init: bad rank or size");
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof(uid));
    ncclComm_t comm = nullptr;
    ncclResult_t r = ncclCommInitRank(&comm, nranks, uid, rank);
    if (r != ncclSuccess) return nccl_fail(r, "ncclCommInitRank");
    *comm_out = comm;
    return MCV_OK;
}

int mcv_nccl_comm_destroy(void* comm) {
    if (!comm) return MCV_OK;
    ncclResult_t r = ncclCommDestroy(static_cast<ncclComm_t>(comm));
    if (r != ncclSuccess) return nccl_fail(r, "ncclCommDestroy");
    return MCV_OK;
}

int mcv_lm_head_argmax_allreduce(void* comm, const void* x, const void* w, void* out_key, void* out_index,
                                 int64_t M, int64_t K, int64_t N_shard, int64_t n_offset, int fp16_logits,
                                 void* workspace, size_t workspace_bytes, mcv_stream_t stream) {
    if (!comm || !out_key || !out_index) return fail(MCV_ERR_NULL, "lm_head_argmax_allreduce: null comm, out_key or out_index");
    auto s = static_cast<cudaStream_t>(stream);
    int st = lm_head_argmax_impl(x, w, out_key, nullptr, M, K, N_shard, n_offset, fp16_logits, workspace,
                                 workspace_bytes, s);
    if (st) return st;
    ncclResult_t r = ncclAllReduce(out_key, out_key, static_cast<size_t>(M), ncclUint64, ncclMax,
                                   static_cast<ncclComm_t>(comm), s);
    if (r != ncclSuccess) return nccl_fail(r, "ncclAllReduce");
    return key_to_index_impl(out_key, out_index, M, s);
}

}  // extern "C"
