/*
 * mcv_matmul.h -- C ABI of the B200 (sm_100a) decode-matmul library
 * (libmcv_b200.so).
 *
 * This is the drop-in boundary for the decode matmul hot path of the
 * MiniCPM-V 4.6 engine (lvyufeng/minicpm-v-4.6-orangepi).  Each entry point
 * names the reference interface it replaces (file:line in that project).
 *
 * Conventions
 *  - All tensor arguments are raw DEVICE pointers unless the name ends in
 *    `_host`.  fp16 data is IEEE binary16 passed as `void*`/`uint16_t*`.
 *  - Nothing here allocates device memory.  Buffers, including workspaces
 *    sized by the `*_workspace_size` queries, belong to the caller.
 *  - Calls are asynchronous and stream-ordered on `stream` (a cudaStream_t;
 *    NULL = legacy default stream).  Unlike the reference, which synchronises
 *    its stream after every op (src/csrc/lib/ops.cpp:359-377), no call here
 *    synchronises; the C++ wrappers in mcv_ops.hpp offer that as an option.
 *  - Every function returns an mcv_status; 0 is success.  Errors are reported,
 *    never thrown and never trapped on the device; mcv_last_error() gives a
 *    message for the calling thread.
 *  - Kernels are launched with programmatic dependent launch: a GEMV issues
 *    its weight loads before waiting for the previous kernel on the stream,
 *    and reads activations only after that wait.  Weights must therefore not
 *    be written by the kernel immediately preceding the call on the same
 *    stream while that kernel is still running; use mcv_set_pdl(0) to turn
 *    the early start off.
 */
#ifndef MCV_MATMUL_H
#define MCV_MATMUL_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* mcv_stream_t; /* cudaStream_t */

enum mcv_status {
    MCV_OK = 0,
    MCV_ERR_NULL = 1,        /* a required pointer is NULL */
    MCV_ERR_SHAPE = 2,       /* unsupported or inconsistent dimensions */
    MCV_ERR_ALIGN = 3,       /* a pointer is not 16-byte aligned */
    MCV_ERR_CUDA = 4,        /* a CUDA runtime call failed */
    MCV_ERR_NCCL = 5,        /* an NCCL call failed */
    MCV_ERR_WORKSPACE = 6,   /* workspace missing or too small */
    MCV_ERR_VALUE = 7,       /* bad argument value (layout code, g_idx, zero range) */
    MCV_ERR_TIMEOUT = 8,     /* a bounded device-side wait gave up */
    MCV_ERR_FORMAT = 9       /* a file cannot be read or is not a valid safetensors file */
};

const char* mcv_status_string(int status);
/* Message describing the last failure on the calling thread ("" if none). */
const char* mcv_last_error(void);
/* Library ABI version, (major << 16) | minor. */
int mcv_version(void);
/* 1 (default): launch kernels with programmatic dependent launch; 0: plain launches. */
void mcv_set_pdl(int enabled);

/* Kernel-choice overrides for performance tuning; 0 restores the default.
 *   MCV_TUNE_W4A16_MODE: 1 = register-buffered streaming kernel (each warp
 *   owns whole 16-column strips), 2 = one block per strip with K split over
 *   its warps (K <= 8192), 3 = streaming kernel fed by warp-private
 *   bulk-copy rings; default: K-split below 4 strips per SM, else 3.
 *   MCV_TUNE_ROWS_BLOCKS_PER_SM: blocks per SM of the persistent lm_head /
 *   [N][K] GEMV grid (1..4; default 4 up to 600 rows per SM, else 2).
 *   MCV_TUNE_ROWS_PREFETCH: how many row steps ahead of its loads each warp
 *   of that grid warms L2 (1..16; -1 = no warm-up; default: 1 up to 600
 *   rows per SM, else none).
 *   MCV_TUNE_ROWS_WALK: 1 = that grid's warps take rows strided by the grid
 *   (default), 2 = each warp a contiguous range.
 *   MCV_TUNE_GEMM_SPLIT_K: k slices (1..8, thread-block cluster along z) of
 *   mcv_w4a16_gemm; default: doubled while the output tiles times the
 *   slices fit the SMs and every slice keeps >= 4 stages of 64 k.
 *   MCV_TUNE_W8A8_KERNEL: the [N][K] W8A8 kernel - 1 = DP4A dot products,
 *   2 = integer tensor-core MMAs (mma.sync m16n8k32 s8); default: DP4A for
 *   M = 1, MMAs from M = 2.  Both give the same bits.
 *   MCV_TUNE_W4A16_GRID: blocks of the bulk-copy streaming W4A16 kernel
 *   (capped at 3 per SM); default: 3 per SM, or one warp per strip when
 *   there are fewer strips.
 *   MCV_TUNE_W4A16_MATH: the W4A16 GEMV's per-group arithmetic - 1 = exact
 *   (q - zero) per weight on four MMA chains, 2 = the same on two chains with
 *   integer-built zero constants, 3 = zero point folded out (raw
 *   exponent-bias weights, sum(x) from an all-ones MMA); default: 1 for the
 *   K-split schedule, 2 for the bulk-copy ring.
 *   MCV_TUNE_W4A16_KSPLIT_WARPS: warps per strip of the K-split W4A16 kernel
 *   (8, 16 or 32; arithmetic 1 only); default 8 up to K = 1024, else 16. */
enum mcv_tuning_key {
    MCV_TUNE_W4A16_MODE = 2,
    MCV_TUNE_ROWS_BLOCKS_PER_SM = 3,
    MCV_TUNE_ROWS_PREFETCH = 4,
    MCV_TUNE_GEMM_SPLIT_K = 5,
    MCV_TUNE_W8A8_KERNEL = 6,
    MCV_TUNE_W4A16_GRID = 7,
    MCV_TUNE_W4A16_MATH = 8,
    MCV_TUNE_ROWS_WALK = 9,
    MCV_TUNE_W4A16_KSPLIT_WARPS = 10,
    MCV_TUNE_COUNT = 11
};
int mcv_set_tuning(int key, int value);
/* Device-side error bits recorded since the last call (and cleared by it):
 * bit 0 = a bounded wait inside a kernel gave up (that kernel returned early
 * and its outputs are incomplete).  Synchronises the current device. */
unsigned mcv_device_errors(void);
int mcv_get_tuning(int key);

/* ======================================================================== */
/* W4A16: int4 weights, fp16 group scales and 4-bit zeros, fp16 activations */
/* ======================================================================== */
/*
 * Device weight layout "mcv-int4" (prepared once at load time; group = 128,
 * the only quantization group the reference supports, ops.h:95-103):
 *   qweight  uint32 [Npad/16][K/64][32][4]   Npad = N rounded up to 16.
 *            Output columns form strips of 16; per strip, 64-k quads follow
 *            each other; entry [s][q][l][j] is lane l's word for the j-th
 *            MMA of quad q: the eight 4-bit values it feeds to one m16n8k16
 *            tensor-core MMA as its A fragment (rows = the strip's columns).
 *            With kb = 64q + 16(l%4) + 4j, they are (col, k) = (l/4, kb),
 *            (l/4, kb+1), (l/4+8, kb), (l/4+8, kb+1), (l/4, kb+2),
 *            (l/4, kb+3), (l/4+8, kb+2), (l/4+8, kb+3), in nibble slots
 *            0,4,1,5,2,6,3,7 (k is permuted inside each quad identically for
 *            weights and activations, which leaves every dot product intact).
 *   scales   fp16   [Npad][Gpad]   G = K/128, Gpad = G rounded up to 8
 *   zeros    uint32 [Npad][ceil(G/8)]  4-bit zero of (g, n) at nibble g%8 of
 *            word g/8; effective zero = nibble + zero_bias
 *   zero_bias 0 for AWQ and synthetic weights, 1 for GPTQ (whose stored zero
 *            is one less than the true zero, src/csrc/lib/quantized_weight.cpp:112)
 * Padding columns and groups have q = zero = 0 and scale 0.  Dequantised
 * weight w[k][n] = (q - zero) * scale.  K must be a multiple of 128.
 */

/* Bytes of each array of the mcv-int4 layout. */
int mcv_w4a16_layout_bytes(int64_t K, int64_t N, int64_t group, size_t* qweight_bytes,
                           size_t* scales_bytes, size_t* zeros_bytes);

/* Host repack from logical arrays: q uint8 [K][N] (0..15), z uint8 [G][N]
 * (0..15), scales fp16 [G][N].  Writes the three mcv-int4 arrays (host memory). */
int mcv_w4a16_pack_host(const uint8_t* q_kn, const uint8_t* z_gn, const uint16_t* scales_gn,
                        int64_t K, int64_t N, int64_t group, uint32_t* qweight_out,
                        uint16_t* scales_out, uint32_t* zeros_out);

/* The inverse of the packers: the mcv-int4 arrays back to the logical
 * (q - zero) int8 [K][N] and scales fp16 [K/group][N] - the form the
 * reference's unpackers produce (HostW4A16Weight, quantized_weight.cpp:19-25).
 * For checking a loaded checkpoint against another loader. */
int mcv_w4a16_unpack_host(const uint32_t* qweight, const uint16_t* scales, const uint32_t* zeros, int zero_bias,
                          int64_t K, int64_t N, int64_t group, int8_t* w_kn, uint16_t* scales_gn);

/* Host repack of a GPTQ checkpoint tensor set (qweight int32 [K/8][N],
 * qzeros int32 [G][N/8], g_idx int32 [K] or NULL, scales fp16 [G][N]).
 * Replaces unpack_gptq_weight + pack_w4a16_weight of
 * src/csrc/lib/quantized_weight.cpp:75-120, 48-73 (load_w4a16_quantized_weight,
 * :212-229).  Like the reference kernel, scales are indexed by k/group, so a
 * g_idx other than k/group is rejected (MCV_ERR_VALUE).  *zero_bias_out = 1. */
int mcv_w4a16_pack_gptq_host(const int32_t* qweight, const int32_t* qzeros,
                             const int32_t* g_idx, const uint16_t* scales, int64_t K,
                             int64_t N, int64_t group, uint32_t* qweight_out,
                             uint16_t* scales_out, uint32_t* zeros_out, int* zero_bias_out);

/* Host repack of an AWQ tensor set (qweight int32 [K][N/8], qzeros int32
 * [G][N/8], slot order {0,2,4,6,1,3,5,7}; scales fp16 [G][N]).
 * Replaces unpack_awq_weight, src/csrc/lib/quantized_weight.cpp:122-160. */
int mcv_w4a16_pack_awq_host(const int32_t* qweight, const int32_t* qzeros,
                            const uint16_t* scales, int64_t K, int64_t N, int64_t group,
                            uint32_t* qweight_out, uint16_t* scales_out, uint32_t* zeros_out,
                            int* zero_bias_out);

/* Host repack of the reference's own tile-packed int8 (q - zero) layout
 * (src/csrc/lib/quantized_weight.cpp:41-73, the `w_int8` argument of
 * matmul_w4a16, src/csrc/include/minicpmv/ops.h:95-108) with its scales fp16
 * [G][N].  A zero is chosen per (group, column) so every value fits 4 bits;
 * MCV_ERR_VALUE if a group/column spans more than 16 levels. */
int mcv_w4a16_pack_from_tiles_host(const int8_t* packed, int64_t tile_len,
                                   const uint16_t* scales_gn, int64_t K, int64_t N,
                                   uint32_t* qweight_out, uint16_t* scales_out,
                                   uint32_t* zeros_out, int* zero_bias_out);

/* out[m][n] = sum_k x[m][k] * w[k][n], M = 1..64, fp32 accumulation, fp16 out.
 * x fp16 [M][K], out fp16 [M][N]; group must be 128; x, qweight and scales
 * 16-byte aligned.  M = 9..64 (batched decode) shares each dequantised weight
 * fragment across up to eight MMAs and needs K <= 8192.
 * Replaces matmul_w4a16 (src/csrc/lib/ops.cpp:1030-1095, ops.h:95-108; M=1
 * there) and its kernel op_kernel/matmul_w4a16_custom.cpp. */
int mcv_w4a16_gemv(const void* x, const void* qweight, const void* scales, const void* zeros,
                   int zero_bias, void* out, int64_t M, int64_t K, int64_t N, int64_t group,
                   mcv_stream_t stream);

/* out[m][n] = sum_k x[m][k] * w[k][n] for larger M (batched decode, prefill;
 * intended for M >= 16), on the tcgen05 tensor cores: x and the packed int4
 * tiles by TMA into shared memory, weights dequantised to fp16
 * (q - zero) * scale into tensor memory as the MMA's A operand, fp32
 * accumulation in tensor memory, fp16 out; small grids split k over a
 * thread-block cluster (MCV_TUNE_GEMM_SPLIT_K).  Same mcv-int4 weights as
 * mcv_w4a16_gemv; group 128; x, qweight and scales 16-byte aligned, zeros
 * 4-byte; K a multiple of 128.  The reference has no quantized GEMM for M > 1: it runs prefill through
 * matmul_b_transposed's dense path (src/csrc/lib/ops.cpp:215-322). */
int mcv_w4a16_gemm(const void* x, const void* qweight, const void* scales, const void* zeros,
                   int zero_bias, void* out, int64_t M, int64_t K, int64_t N, int64_t group,
                   mcv_stream_t stream);

/* Several independent W4A16 GEMVs (same M) in one launch: problems is a HOST
 * array; each entry's x/out/weights are device pointers.  No problem may read
 * another problem's output.  For projections that share an input (q/k/v,
 * gate/up, the linear-attention qkv/z/a/b of src/csrc/lib/decoder_layer.cpp:
 * 1110-1114, :970-972, :1200-1201) and for batches of unrelated GEMVs.
 * Launches ceil(count/48) kernels. */
typedef struct mcv_w4a16_problem {
    const void* x;
    const void* qweight;
    const void* scales;
    const void* zeros;
    void* out;
    int32_t K;
    int32_t N;
    int32_t group;
    int32_t zero_bias;
} mcv_w4a16_problem;
int mcv_w4a16_gemv_grouped(const mcv_w4a16_problem* problems, int count, int64_t M,
                           mcv_stream_t stream);

/* The MLP's gate and up projections with SwiGLU in the epilogue:
 * act fp16 [M][N] = silu_mul(x . Wg, x . Wu) for x fp16 [M][K] and two mcv-int4
 * weights of equal K and N (the problems' x and out fields are ignored).  The
 * gate and up sums are rounded to fp16 - the projections' output type - and
 * combined exactly as mcv_silu_mul does (fp32 g / (1 + exp(-g)) * u,
 * op_kernel/silu_mul_custom.cpp:63-72), in one launch and with no gate / up
 * round trip through memory.  Replaces the gate and up matmul_decode_dispatch
 * calls and the silu_mul of decoder_layer.cpp:1186-1203.  M = 1..8,
 * K <= 4096 (multiple of 128), group 128. */
int mcv_w4a16_gemv_gate_up_silu(const void* x, const mcv_w4a16_problem* gate, const mcv_w4a16_problem* up, void* act,
                                int64_t M, mcv_stream_t stream);

/* ======================================================================== */
/* dense fp16 GEMV and the lm_head                                          */
/* ======================================================================== */

/* out fp16 [M][N] = x fp16 [M][K] . W, M = 1..8, fp32 accumulation.
 * w_layout 0: W stored [N][K] (the checkpoint / tied-embedding layout);
 * w_layout 1: W stored [K][N] (the reference's pre-transposed "natural" B).
 * Replaces matmul_b_transposed at M=1 (src/csrc/lib/ops.cpp:159-209,
 * ops.h:19) and the cube kernel op_kernel/matmul_cube_custom.cpp. */
int mcv_gemv_f16(const void* x, const void* w, void* out, int64_t M, int64_t K, int64_t N,
                 int w_layout, mcv_stream_t stream);

/* out fp16 [M][N] = x fp16 [M][K] . W^T, W fp16 [N][K], fp32 accumulation, on
 * the tcgen05 tensor cores (TMA-fed shared-memory operands, accumulator in
 * tensor memory; k split over a thread-block cluster when the output tiles
 * leave SMs idle).  Any M >= 1 (meant for M > 8, where the GEMV stops);
 * K a multiple of 64, N a multiple of 8.  Replaces matmul_b_transposed's
 * aclnnMm / K-tiled path for M > 1 (src/csrc/lib/ops.cpp:215-322). */
int mcv_gemm_f16(const void* x, const void* w, void* out, int64_t M, int64_t K, int64_t N, mcv_stream_t stream);
/* dst fp16 [cols][rows] = src fp16 [rows][cols]^T: the load-time transpose that
 * turns the reference's pre-transposed [K][N] weights (load_matmul_weight_transposed,
 * src/csrc/lib/language_model.cpp:84-105) back into [N][K] for mcv_gemm_f16. */
int mcv_transpose_f16(const void* src, void* dst, int64_t rows, int64_t cols, mcv_stream_t stream);

/* Workspace bytes for mcv_lm_head_argmax with M rows; must be zero-filled
 * once before first use (each call leaves it zeroed again). */
size_t mcv_lm_head_workspace_size(int64_t M);

/* Fused lm_head GEMV + greedy argmax over one contiguous vocab shard.
 *   x       fp16 [M][K] (M = 1..8)
 *   w       fp16 [N_shard][K] rows of the tied embedding, global rows
 *           n_offset .. n_offset+N_shard-1
 *   out_key uint64 [M] (may be NULL): order-preserving argmax key,
 *           (ordered fp32 bits of the winning logit << 32) | (0xFFFFFFFF - index)
 *   out_index int64 [M] (may be NULL): winning global vocab index
 * Logits are fp32 dots; ties go to the smallest index (the first maximum,
 * language_model.cpp:475 and tests/test_lm_head_pipeline.cpp:104).
 * fp16_logits = 1 compares logits rounded to fp16, as the production
 * lm_head_greedy does on its D2H-copied fp16 chunk (language_model.cpp:471-479);
 * unlike that host scan it keeps fp16 subnormals instead of reading them as
 * zero, which can only matter when the largest logit is below 6.1e-5 in
 * magnitude.  (mcv_lm_head_argmax_w8a8 reads them as zero, as the scan does.)
 * Replaces the per-chunk matmul + D2H + host argmax loop of lm_head_greedy,
 * src/csrc/lib/language_model.cpp:464-480. */
int mcv_lm_head_argmax(const void* x, const void* w, void* out_key, void* out_index, int64_t M,
                       int64_t K, int64_t N_shard, int64_t n_offset, int fp16_logits,
                       void* workspace, size_t workspace_bytes, mcv_stream_t stream);

/* lm_head_greedy's device half including its final rms_norm
 * (src/csrc/lib/language_model.cpp:422-423): x is the raw last hidden state
 * [M][K]; every block normalises it in its prologue (gamma fp16 [K],
 * norm_variant 0 = the engine's rms_norm, ops.cpp:564-737: fp16 chain with
 * (1 + gamma); 1 = the rms_norm1024 kernel's fp32 arithmetic with gamma), then
 * the same GEMV + argmax as mcv_lm_head_argmax.  p2p_ctx NULL: this GPU's
 * shard alone; else the peer exchange of mcv_lm_head_argmax_p2p.  Saves the
 * separate normalisation launch and its 2 KB round trip per token. */
int mcv_lm_head_argmax_rmsnorm(void* p2p_ctx, const void* x, const void* norm_gamma, float norm_eps,
                               int norm_variant, const void* w, void* out_key, void* out_index, int64_t M,
                               int64_t K, int64_t N_shard, int64_t n_offset, int fp16_logits, void* workspace,
                               size_t workspace_bytes, mcv_stream_t stream);

/* Greedy argmax of fp16 logits [M][V] -> int64 [M], first maximum wins.
 * Replaces argmax_last_dim (src/csrc/lib/ops.cpp:324-357, ops.h:21). */
int mcv_argmax_last_dim_f16(const void* logits, void* out_index, int64_t M, int64_t V,
                            mcv_stream_t stream);

/* mcv_lm_head_argmax without a caller workspace.  No counterpart in the
 * reference: it exists for callers that cannot allocate device memory (code
 * running where cudaMalloc is forbidden or unwanted, e.g. a host callback or a
 * plugin whose host owns every allocation).  Its workspace is a fixed array of
 * mcv_lm_head_noalloc_max_bytes() bytes in the library's device memory,
 * reserved on every GPU that loads the library until the process exits; it is
 * large enough for every supported M (1..8), and larger requests are rejected
 * with MCV_ERR_WORKSPACE.  The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress), so make that first call before any
 * stream capture.  Each call clears the array with cudaMemsetAsync on `stream` and
 * allocates nothing.  All calls share the one array: calls that
 * may overlap on the GPU (other streams, other threads) race and must be
 * serialised by the caller.  The looked-up address is kept for the life of the
 * process: a cudaDeviceReset of a device this entry point has run on is not
 * supported (the next call would use the old address). */
size_t mcv_lm_head_noalloc_max_bytes(void);
int mcv_lm_head_argmax_noalloc(const void* x, const void* w, void* out_key, void* out_index,
                               int64_t M, int64_t K, int64_t N_shard, int64_t n_offset,
                               int fp16_logits, mcv_stream_t stream);

/* int64 index[m] = 0xFFFFFFFF - (uint32)key[m]: decode argmax keys on the device
 * (key 0, "no row", decodes to -1). */
int mcv_argmax_key_to_index(const void* key, void* out_index, int64_t M, mcv_stream_t stream);

/* ---- sharded lm_head across GPUs (one process per GPU, NCCL over NVLink) -- */
/* Size of an NCCL unique id (bytes). */
size_t mcv_nccl_unique_id_bytes(void);
/* Rank 0 creates the id; the caller distributes it to every rank. */
int mcv_nccl_get_unique_id(void* id_out);
/* Creates this rank's communicator on the current CUDA device. */
int mcv_nccl_comm_init(void** comm_out, int nranks, const void* id, int rank);
int mcv_nccl_comm_destroy(void* comm);
/* mcv_lm_head_argmax on this rank's shard, then one ncclAllReduce(max) of the
 * M uint64 keys, then the index decode: every rank ends with the global
 * argmax in out_index (int64 [M]) and out_key (uint64 [M], required). */
int mcv_lm_head_argmax_allreduce(void* comm, const void* x, const void* w, void* out_key,
                                 void* out_index, int64_t M, int64_t K, int64_t N_shard,
                                 int64_t n_offset, int fp16_logits, void* workspace,
                                 size_t workspace_bytes, mcv_stream_t stream);

/* ---- sharded lm_head with the reduction fused into the kernel (NVLink) ---- */
/* Each rank owns a 1 KB mailbox in its HBM and maps every peer's through
 * CUDA IPC; the last block of each rank's lm_head kernel stores the rank's
 * argmax keys into all mailboxes (one relaxed 64-bit store per key and peer
 * over NVLink: key and call tag share the word, so no fence is needed),
 * waits at most 1 s for the peers' keys and writes the global first-max
 * index - one kernel per rank per token, no collective launch.  All ranks
 * must make the same sequence of calls.  Vocabulary indices must stay below
 * 2^24 - 1 (n_offset + N_shard <= 16777215; MCV_ERR_SHAPE otherwise).
 * Set-up allocates the mailbox (cudaMalloc); calls do not allocate.
 * Replaces the same seam as mcv_lm_head_argmax_allreduce. */
size_t mcv_p2p_handle_bytes(void);
/* Creates this rank's context on the current device; writes its IPC handle
 * (mcv_p2p_handle_bytes() bytes) for the caller to all-gather. */
int mcv_p2p_create(void** ctx_out, int nranks, int rank, void* handle_out);
/* Maps the peers' mailboxes; all_handles = nranks handles in rank order. */
int mcv_p2p_connect(void* ctx, const void* all_handles);
int mcv_p2p_destroy(void* ctx);
/* Error bits of this rank since the last call, cleared by it (bit 0: a peer's
 * key did not arrive within 1 s; that call's out_index is -1).  Synchronous. */
unsigned mcv_p2p_errors(void* ctx);
int mcv_lm_head_argmax_p2p(void* ctx, const void* x, const void* w, void* out_key, void* out_index,
                           int64_t M, int64_t K, int64_t N_shard, int64_t n_offset, int fp16_logits,
                           void* workspace, size_t workspace_bytes, mcv_stream_t stream);

/* One greedy step from host memory to a host token id, as the reference's
 * lm_head_greedy hands the token back (src/csrc/lib/language_model.cpp:412-482).
 * norm_gamma (fp16 [K] on the device, may be NULL): the final rms_norm of
 * language_model.cpp:423 (the engine's variant, eps norm_eps) runs in the
 * kernel's prologue on the raw hidden state; NULL: x is already normalised.
 * Runs mcv_lm_head_argmax (p2p_ctx
 * NULL) or mcv_lm_head_argmax_p2p (p2p_ctx from mcv_p2p_create/connect) on
 * this rank's rows for x (M rows, fp16, in host memory), hands the M int64
 * global indices to index_host and synchronises the stream.  x travels in
 * the kernel's launch parameters when M * K <= 2048 (read during this call);
 * larger x is copied to x_dev first (pin x_host for an asynchronous copy).
 * When index_host is page-locked the kernel stores the indices into it
 * directly and the call returns as soon as they are there (the host watches
 * that memory; the kernel may still be retiring, and later work on `stream`
 * stays ordered after it); otherwise they go through index_dev (M int64 on
 * the device), a copy and a stream synchronisation.  x_dev and index_dev are
 * required either way.  The indices are final when the call returns; same
 * workspace rules as mcv_lm_head_argmax. */
int mcv_lm_head_greedy_host(void* p2p_ctx, const void* x_host, void* x_dev, const void* norm_gamma, float norm_eps,
                            const void* w, void* index_dev, int64_t* index_host, int64_t M, int64_t K,
                            int64_t N_shard, int64_t n_offset, int fp16_logits, void* workspace,
                            size_t workspace_bytes, mcv_stream_t stream);

/* ======================================================================== */
/* W8A8: int8 activations (per-token absmax) x int8 weights (per channel)   */
/* ======================================================================== */

/* Per-row symmetric absmax quantization of x fp16 [M][K] to int8 [M][K] and
 * fp16 scales [M]: scale = max|x|/127 (>= 1e-8), q = trunc(clamp(x/scale) +/- 0.5).
 * Replaces w8a8_quantize (src/csrc/lib/ops.cpp:1135-1171, kernel
 * op_kernel/w8a8_quantize_custom.cpp:25-41; M=1 there). */
int mcv_w8a8_quantize(const void* x, void* x_int8, void* x_scale, int64_t M, int64_t K,
                      mcv_stream_t stream);

/* int32 acc [M][N] = x_int8 [M][K] . w_int8, bit-exact.  w_layout 0: w [N][K]
 * (this library's fast layout), 1: w [K][N] (the reference's layout).
 * Replaces matmul_w8a8_i32 (src/csrc/lib/ops.cpp:1097-1133,
 * op_kernel/matmul_w8a8_i32_custom.cpp). */
int mcv_w8a8_gemm_i32(const void* x_int8, const void* w_int8, void* acc, int64_t M, int64_t K,
                      int64_t N, int w_layout, mcv_stream_t stream);

/* out fp16 [M][N] = fp16_rn((float(acc) * float(w_scale[n])) * float(x_scale[m])).
 * Replaces w8a8_dequant (src/csrc/lib/ops.cpp:1173-1210,
 * op_kernel/w8a8_dequant_custom.cpp:52-59). */
int mcv_w8a8_dequant(const void* acc, const void* x_scale, const void* w_scale, void* out,
                     int64_t M, int64_t N, mcv_stream_t stream);

/* matmul_decode_w8a8_prequant (src/csrc/lib/decoder_layer.cpp:216-224): the
 * int32 GEMV of an already-quantized x (x_int8 [M][K], fp16 scales x_scale
 * [M], from mcv_w8a8_quantize) with int8 [N][K] weights, then the dequant
 * RN((acc * w_scale) * x_scale), in one kernel - so one quantization of the
 * MLP input serves both the gate and the up projection, as in
 * decoder_layer.cpp:1186-1197.  acc_out (int32 [M][N]) is optional. */
int mcv_w8a8_gemv_prequant(const void* x_int8, const void* x_scale, const void* w_int8, const void* w_scale, void* out,
                           void* acc_out, int64_t M, int64_t K, int64_t N, mcv_stream_t stream);

/* Independent fused W8A8 GEMVs in one launch, e.g. the gate and up
 * projections on the same input (decoder_layer.cpp:1186-1197) or a batch of
 * unrelated ones: each problem is mcv_w8a8_fused with w_layout 0 (int8
 * [N][K] weights); all share M (1..8) and K; at most 16 problems. */
typedef struct mcv_w8a8_problem {
    const void* x;       /* fp16 [M][K] */
    const void* w_int8;  /* int8 [N][K] */
    const void* w_scale; /* fp16 [N] */
    void* out;           /* fp16 [M][N] */
    int64_t N;
} mcv_w8a8_problem;
int mcv_w8a8_fused_grouped(const mcv_w8a8_problem* problems, int count, int64_t M, int64_t K, mcv_stream_t stream);

/* Quantize + int8 GEMM + dequant in one kernel (w_layout 0) or three
 * (w_layout 1).  acc_out (int32 [M][N]), x_int8_out and x_scale_out are
 * optional copies of the intermediates (may be NULL).
 * Replaces the W8A8 branch of matmul_decode_dispatch
 * (src/csrc/lib/decoder_layer.cpp:216-232). */
int mcv_w8a8_fused(const void* x, const void* w_int8, const void* w_scale, void* out,
                   void* acc_out, void* x_int8_out, void* x_scale_out, int64_t M, int64_t K,
                   int64_t N, int w_layout, mcv_stream_t stream);

/* Fused W8A8 lm_head + greedy argmax: the W8A8 branch of lm_head_greedy
 * (src/csrc/lib/language_model.cpp:430-479, taken when MINICPM_W8A8_DECODE
 * allows "lm_head").  x fp16 [M][K] is quantized per row in the kernel (as
 * mcv_w8a8_quantize); w_int8 holds int8 weight rows [N_shard][K] with fp16
 * per-row scales w_scale (mcv_w8a8_quantize_weight with w_layout 2 from the
 * fp16 embedding); each logit is RN((acc * w_scale) * x_scale) to fp16, read
 * with subnormals as zero like the reference's host argmax, and the first
 * maximum's global index (n_offset + row) is returned.  K a multiple of 16,
 * at most 4096; M = 1..8; workspace as mcv_lm_head_argmax; out_key uses the
 * same order-preserving format (shards combine by max, e.g. through
 * mcv_argmax_key_to_index after an all-reduce). */
int mcv_lm_head_argmax_w8a8(const void* x, const void* w_int8, const void* w_scale, void* out_key,
                            void* out_index, int64_t M, int64_t K, int64_t N_shard, int64_t n_offset,
                            void* workspace, size_t workspace_bytes, mcv_stream_t stream);

/* Per-output-channel int8 quantization of an fp16 weight: w_scale fp16 [N]
 * (truncating fp16 conversion, as the reference).  w_layout 0: input [K][N],
 * wq [N][K]; 1: input [K][N], wq [K][N]; 2: input [N][K] (e.g. the tied
 * embedding for mcv_lm_head_argmax_w8a8), wq [N][K].
 * Replaces quantize_dense_weight_w8a8 (src/csrc/lib/quantized_weight.cpp:231-268). */
int mcv_w8a8_quantize_weight(const void* w_kn, void* wq, void* w_scale, int64_t K, int64_t N,
                             int w_layout, mcv_stream_t stream);

/* ======================================================================== */
/* Checkpoints: safetensors reader and the GPTQ / AWQ loader                  */
/* ======================================================================== */

/* Element types of safetensors tensors. */
enum mcv_dtype {
    MCV_DT_F16 = 1, MCV_DT_BF16 = 2, MCV_DT_F32 = 3, MCV_DT_F64 = 4, MCV_DT_I8 = 5,
    MCV_DT_U8 = 6, MCV_DT_I16 = 7, MCV_DT_I32 = 8, MCV_DT_I64 = 9, MCV_DT_BOOL = 10
};
/* Opens and memory-maps a .safetensors file and parses its header (replaces
 * WeightsIndex, src/csrc/lib/weights.cpp:197-333): every tensor's byte range is
 * checked against its dtype, shape and the file size (MCV_ERR_FORMAT
 * otherwise).  Close with mcv_safetensors_close. */
int mcv_safetensors_open(const char* path, void** st_out);
int mcv_safetensors_close(void* st);
/* Number of tensors and their names in sorted order (WeightsIndex::names). */
int64_t mcv_safetensors_count(const void* st);
const char* mcv_safetensors_name(const void* st, int64_t i);
/* dtype (mcv_dtype), rank (<= 8), shape, host address of the data inside the
 * mapping (valid until close) and byte size; any output may be NULL. */
int mcv_safetensors_info(const void* st, const char* name, int* dtype, int* rank, int64_t* shape,
                         const void** data, uint64_t* nbytes);
/* Copies an F16 tensor, or a BF16 one converted to F16 by the reference's
 * truncating rule (load_to_device_as, weights.cpp:25-33, 239-262), to device
 * memory (dst_bytes >= the tensor's 2-byte-per-element size). */
int mcv_safetensors_copy_f16(const void* st, const char* name, void* dst_dev, uint64_t dst_bytes,
                             mcv_stream_t stream);
/* Dimensions of the quantized projection `base` (base.qweight / .qzeros /
 * .scales, plus .g_idx for GPTQ; without .g_idx it is AWQ), with the dtype and
 * shape checks of quantized_weight.cpp:75-160.  Use K and N with
 * mcv_w4a16_layout_bytes to size the device buffers. */
int mcv_w4a16_safetensors_dims(const void* st, const char* base, int64_t* K, int64_t* N, int* is_gptq);
/* load_w4a16_quantized_weight (src/csrc/lib/quantized_weight.cpp:212-229):
 * the checkpoint's GPTQ or AWQ tensors repacked into the mcv-int4 arrays in
 * the caller's device buffers (scales may be F16 or BF16); *zero_bias_out as
 * the pack_*_host functions set it.  Synchronous (the host staging is
 * released on return).  The _host form writes host arrays instead. */
int mcv_w4a16_load_safetensors(const void* st, const char* base, void* qweight_dev, void* scales_dev,
                               void* zeros_dev, int* zero_bias_out, mcv_stream_t stream);
int mcv_w4a16_load_safetensors_host(const void* st, const char* base, uint32_t* qweight, uint16_t* scales,
                                    uint32_t* zeros, int* zero_bias_out);

/* ======================================================================== */
/* The GEMVs' element-wise neighbours                                        */
/* ======================================================================== */

/* out fp16 [rows][H] = rms_norm(x fp16 [rows][H]) with gamma fp16 [H].
 * variant 0: the engine's rms_norm (src/csrc/lib/ops.cpp:564-737): a chain
 * of fp16 ops - x*x, mean, + eps, rsqrt, x * rstd, each rounded to fp16 -
 * then times (1 + gamma); the mean's sum is exact.  variant 1: rms_norm1024
 * (ops.cpp:536-562, op_kernel/rms_norm1024_custom.cpp:57-70): fp32
 * x / sqrt(mean(x^2) + eps) * gamma, rounded once.  Any H (the custom
 * kernel's fixed 1024 is not required). */
int mcv_rms_norm(const void* x, const void* gamma, void* out, int64_t rows, int64_t H, float eps, int variant,
                 mcv_stream_t stream);
/* out = silu(gate) * up element-wise over n fp16 values (16-byte aligned):
 * fp32 g / (1 + exp(-g)) * u rounded to fp16.  Replaces silu_mul
 * (src/csrc/lib/ops.cpp:437-456, op_kernel/silu_mul_custom.cpp:63-72). */
int mcv_silu_mul(const void* gate, const void* up, void* out, int64_t n, mcv_stream_t stream);

/* ======================================================================== */
/* Decode dispatch: which weight format a projection's matmul runs on        */
/* ======================================================================== */

/* The MINICPM_W8A8_DECODE policy (src/csrc/lib/language_model.cpp:19-41,
 * decoder_layer.cpp:19-25).  The mode string comes from the environment,
 * read once per process on first use; mcv_set_w8a8_decode_mode replaces it
 * (NULL: read the environment again on the next query).
 *   enabled: the mode is non-empty and neither "0" nor "false";
 *   allows(token): "all" -> every token; "1" / "selective" -> "lm_head"
 *   only; any other mode -> the token occurs in the mode string (tokens:
 *   mlp, linear_qkv, linear_z, linear_out, full_q, full_k, full_v, full_o,
 *   lm_head). */
int mcv_set_w8a8_decode_mode(const char* mode);
int mcv_w8a8_decode_enabled(void);
/* The per-layer decode gate that mcv_matmul_decode_dispatch applies
 * (decoder_layer.cpp:19-25): the variable is set (an empty value counts)
 * and is neither "0" nor "false".  It differs from mcv_w8a8_decode_enabled
 * only for a set-but-empty variable, exactly as the reference's two rules do. */
int mcv_w8a8_decode_gate_enabled(void);
int mcv_w8a8_policy_allows(const char* token);
/* The same rule for an explicit mode string (no process state). */
int mcv_w8a8_policy_allows_mode(const char* mode, const char* token);

/* The formats one projection has on the device; absent ones are NULL.
 * dense: fp16, dense_layout 0 = [N][K], 1 = [K][N].  w4_*: mcv-int4
 * (mcv_w4a16_pack_*).  w8_*: int8 [N][K] + fp16 per-channel scales
 * (mcv_w8a8_quantize_weight with w_layout 0). */
typedef struct mcv_decode_weights {
    const void* dense;
    int dense_layout;
    const void* w4_qweight;
    const void* w4_scales;
    const void* w4_zeros;
    int w4_zero_bias;
    const void* w8_weight;
    const void* w8_scale;
} mcv_decode_weights;

/* out fp16 [M][N] = x fp16 [M][K] . W, choosing the format like
 * matmul_decode_dispatch (src/csrc/lib/decoder_layer.cpp:226-244): W8A8
 * (fused quantize + int8 GEMV + dequant) when the policy is enabled, the
 * W8A8 weight is present and M == 1; else W4A16 when present and M == 1;
 * else the dense weight (GEMV up to M = 8, the tcgen05 GEMM above, which
 * needs dense_layout 0).  Beyond the reference: with no dense weight, M > 1
 * stays on the int4 weights (GEMV up to M = 32, the tcgen05 GEMM above)
 * instead of failing.  MCV_ERR_NULL when no format fits. */
int mcv_matmul_decode_dispatch(const void* x, const mcv_decode_weights* w, void* out, int64_t M,
                               int64_t K, int64_t N, mcv_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif
