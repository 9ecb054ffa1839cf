// Dense fp16 GEMM for prefill / batched decode (M > 8) on the 5th-generation
// tensor cores: tcgen05.mma with both operands staged in shared memory by TMA
// and the fp32 accumulator in tensor memory.
//
// Reference behaviour replaced: matmul_b_transposed's path for M > 1
// (src/csrc/lib/ops.cpp:159-322): aclnnMm, with the K-tiled loop of
// :215-280 for M >= 64 and K > 4096, on weights stored [N][K].  Here out =
// x . W^T with W [N][K] (the checkpoint layout; the reference's [K][N]
// "natural" copies are a load-time transpose away) and fp32 accumulation.
//
// As in the W4A16 GEMM, the product is computed transposed, out^T = W x^T:
// 128 weight rows of a block are the MMA's M, up to 256 rows of x its N.  A
// stage is 64 k: the weight tile [128][64] and the x tile [rows][64] land by
// TMA with the 128-byte swizzle into a 4-deep ring.  Roles, meeting only on
// mbarriers: a producer thread (TMA, weights of the first stages requested
// before the PDL wait), an MMA-issuing thread (4 MMAs of K = 16 per stage,
// one commit), and four epilogue warps that read the accumulator (TMEM lane =
// weight row, column = row of x) and write fp16.  When the output tiles leave
// SMs idle, k is split over the CTAs of a thread-block cluster and the slices'
// fp32 partials are summed in rank order through distributed shared memory.
// Every wait is bounded (2 s); on a timeout the block records an error bit,
// drains its own copies and MMAs, frees its tensor memory and returns.
// Single-GPU code: no multicast, no peer memory.
#include "common.cuh"
#include "tcgen05.cuh"

namespace mcv {
unsigned take_dense_gemm_device_error();

namespace {

constexpr int kDW = 128;                   // weight rows per block (MMA M)
constexpr int kDX = 256;                   // rows of x per block (MMA N, at most)
constexpr int kDK = 64;                    // k per stage (one 128-byte swizzle row)
constexpr int kDWBytes = kDW * kDK * 2;    // 16 KB
constexpr int kDXBytes = kDX * kDK * 2;    // 32 KB (at most)
constexpr int kDStageBytes = kDWBytes + kDXBytes;
constexpr int kDStages = 4;
constexpr int kDEpiWarps = 4;              // 128 TMEM lanes
constexpr int kDThreads = (kDEpiWarps + 2) * 32;
constexpr int kDTmemCols = 256;
constexpr int kDSmemBytes = kDStages * kDStageBytes + 1024 + 256;
static_assert(kDSmemBytes <= 227 * 1024, "shared memory budget");
static_assert(kDX * kDW * 4 <= kDStages * kDStageBytes, "split-k partials must fit the ring");

static __device__ unsigned g_dense_gemm_dev_error;

struct DenseGemmArgs {
    __half* out;
    int M, K, N;
    int x_box_rows;  // rows one x tile copy lands
    int splits;      // k slices = CTAs of a cluster along z
};

__global__ void __launch_bounds__(kDThreads, 1)
dense_gemm_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                  const DenseGemmArgs a) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    auto wt = [&](int b) { return smem + b * kDStageBytes; };
    auto xt = [&](int b) { return smem + b * kDStageBytes + kDWBytes; };
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kDStages * kDStageBytes);  // [stages] tiles landed
    uint64_t* done = full + kDStages;                                                // [stages] MMAs complete
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + kDStages);
    volatile int* failed = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * kDW, m0 = blockIdx.y * kDX;
    const int split = blockIdx.z;
    const int nk = a.K / kDK;
    const int i0 = static_cast<int>(static_cast<int64_t>(nk) * split / a.splits);
    const int nst = static_cast<int>(static_cast<int64_t>(nk) * (split + 1) / a.splits) - i0;
    const int rows = a.M - m0 < kDX ? a.M - m0 : kDX;
    const int mma_n = (rows + 15) & ~15;
    const uint32_t x_bytes = static_cast<uint32_t>(a.x_box_rows) * kDK * 2;
    constexpr int kIssuerWarp = kDEpiWarps, kProducerWarp = kDEpiWarps + 1;

    if (warp == kIssuerWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kDTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        for (int i = 0; i < kDStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&done[i], 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        *failed = 0;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_acc = *tmem_slot;
    pdl_trigger();

    if (warp == kProducerWarp) {
        if (lane == 0) {
            // Stage j goes to slot j % stages once the MMAs of stage
            // j - stages have released it.  The weight tiles of the first
            // slots do not depend on the previous kernel.
            const int pre = nst < kDStages ? nst : kDStages;
            for (int j = 0; j < pre; ++j) {
                mbar_expect_tx(&full[j], kDWBytes + x_bytes);
                tma_load_2d(wt(j), &wmap, (i0 + j) * kDK, n0, &full[j]);
            }
            pdl_wait();  // x may be the previous kernel's output
            int j = 0;
            for (; j < nst; ++j) {
                const int sj = j % kDStages;
                if (j >= kDStages) {
                    if (*failed || !mbar_wait(&done[sj], static_cast<uint32_t>((j - kDStages) / kDStages) & 1u)) {
                        *failed = 1;
                        break;
                    }
                    mbar_expect_tx(&full[sj], kDWBytes + x_bytes);
                    tma_load_2d(wt(sj), &wmap, (i0 + j) * kDK, n0, &full[sj]);
                }
                tma_load_2d(xt(sj), &xmap, (i0 + j) * kDK, m0, &full[sj]);
            }
            // drain (bounded): every slot whose copies were requested lands
            // before the block frees its shared memory
            for (int q = (j > kDStages ? j - kDStages : 0); q < j; ++q)
                if (!mbar_wait(&full[q % kDStages], static_cast<uint32_t>(q / kDStages) & 1u)) *failed = 1;
        }
        __syncwarp();
    } else if (warp == kIssuerWarp) {
        if (lane == 0) {
            const uint32_t idesc = instr_desc_f16(kDW, mma_n);
            const uint64_t wdesc0 = smem_desc_sw128(smem_u32(wt(0)));
            const uint64_t xdesc0 = smem_desc_sw128(smem_u32(xt(0)));
            int issued = 0;
            for (int i = 0; i < nst; ++i) {
                const int b = i % kDStages;
                if (*failed || !mbar_wait(&full[b], static_cast<uint32_t>(i / kDStages) & 1u)) {
                    *failed = 1;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < kDK / 16; ++kk) {
                    const uint64_t off = static_cast<uint64_t>((b * kDStageBytes + kk * 32) >> 4);
                    mma_f16_ss(tmem_acc, wdesc0 + off, xdesc0 + off, idesc, (i > 0 || kk > 0) ? 1u : 0u);
                }
                mma_commit(&done[b]);
                issued = i + 1;
            }
            // the last commit covers every MMA issued before it
            if (issued > 0 &&
                !mbar_wait(&done[(issued - 1) % kDStages], static_cast<uint32_t>((issued - 1) / kDStages) & 1u))
                *failed = 1;
            if (issued < nst) *failed = 1;
        }
        __syncwarp();
    }
    if (warp != kProducerWarp) pdl_wait();  // every thread passes the wait before exit
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const bool acc_ready = !*failed;
    if (!acc_ready && tid == 0) atomicOr(&g_dense_gemm_dev_error, kDevErrTimeout);
    const uint32_t acc_lanes = tmem_acc + (static_cast<uint32_t>(warp * 32) << 16);
    if (a.splits == 1) {
        // fp16 outputs through a shared-memory tile (the ring is idle: every
        // copy landed, every MMA completed), then 16-byte stores of 8
        // columns instead of one 2-byte store per column and row
        __half* tile = reinterpret_cast<__half*>(smem);  // [rows][kDW]
        if (warp < kDEpiWarps) {
            if (acc_ready) {
#pragma unroll 1
                for (int j = 0; j * 16 < mma_n; ++j) {
                    float v[16];
                    tmem_ld16(acc_lanes + j * 16, v);
#pragma unroll
                    for (int e = 0; e < 16; ++e) tile[(j * 16 + e) * kDW + warp * 32 + lane] = __float2half_rn(v[e]);
                }
            }
            asm volatile("bar.sync 1, %0;" ::"r"(kDEpiWarps * 32) : "memory");  // the epilogue warps only
            if (acc_ready) {
                const bool vec_ok = (a.N & 7) == 0 && (reinterpret_cast<uintptr_t>(a.out) & 15u) == 0;
                for (int idx = tid; idx < rows * (kDW / 8); idx += kDEpiWarps * 32) {
                    const int r = idx / (kDW / 8), c8 = (idx % (kDW / 8)) * 8, col = n0 + c8;
                    const __half* src = tile + r * kDW + c8;
                    __half* o = a.out + static_cast<size_t>(m0 + r) * a.N + col;
                    if (vec_ok && col + 8 <= a.N) {
                        *reinterpret_cast<uint4*>(o) = *reinterpret_cast<const uint4*>(src);
                    } else {
                        for (int e = 0; e < 8; ++e)
                            if (col + e < a.N) o[e] = src[e];
                    }
                }
            }
        }
    } else {
        // Split k: each CTA parks its fp32 partials in its (idle) ring as
        // red[m][n]; after a cluster barrier CTA `split` sums rows m = split,
        // split + S, ... over all slices in rank order and writes fp16; a
        // second barrier keeps every CTA's memory alive until all are done.
        float* red = reinterpret_cast<float*>(smem);
        int* red_failed = reinterpret_cast<int*>(smem + kDStages * kDStageBytes - 16);
        if (warp < kDEpiWarps) {
#pragma unroll 1
            for (int j = 0; j * 16 < mma_n; ++j) {
                float v[16];
                tmem_ld16(acc_lanes + j * 16, v);
#pragma unroll
                for (int e = 0; e < 16; ++e) red[(j * 16 + e) * kDW + warp * 32 + lane] = v[e];
            }
        }
        if (tid == 0) *red_failed = acc_ready ? 0 : 1;
        cluster_sync();
        int any_failed = 0;
        for (int r = 0; r < a.splits; ++r) any_failed |= ld_cluster_s32(cluster_smem_addr(red_failed, r));
        if (!any_failed && warp < kDEpiWarps) {
            const int n = 4 * lane, col = n0 + n;
            const bool vec_ok = (a.N & 3) == 0 && (reinterpret_cast<uintptr_t>(a.out) & 7u) == 0;
#pragma unroll 1
            for (int m = split + a.splits * warp; m < rows; m += a.splits * kDEpiWarps) {
                float4 part[8];
#pragma unroll
                for (int r = 0; r < 8; ++r)
                    if (r < a.splits) part[r] = ld_cluster_f32x4(cluster_smem_addr(red + m * kDW + n, r));
                float4 acc = part[0];
#pragma unroll
                for (int r = 1; r < 8; ++r)
                    if (r < a.splits) acc.x += part[r].x, acc.y += part[r].y, acc.z += part[r].z, acc.w += part[r].w;
                __half* o = a.out + static_cast<size_t>(m0 + m) * a.N + col;
                if (vec_ok && col + 4 <= a.N) {
                    *reinterpret_cast<uint2*>(o) = make_uint2(h2_as_u32(__floats2half2_rn(acc.x, acc.y)),
                                                              h2_as_u32(__floats2half2_rn(acc.z, acc.w)));
                } else {
                    const float e4[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        if (col + e < a.N) o[e] = __float2half_rn(e4[e]);
                }
            }
        }
        cluster_sync();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kIssuerWarp)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_acc), "r"(kDTmemCols)
                     : "memory");
}

// [R][C] fp16 -> [C][R] through 32x32 shared-memory tiles (load-time
// preparation of [K][N] weights for the GEMM).
__global__ void __launch_bounds__(256) transpose_f16_kernel(const __half* __restrict__ src, __half* __restrict__ dst,
                                                            int64_t R, int64_t C) {
    __shared__ __half tile[32][33];
    pdl_trigger();
    pdl_wait();
    const int64_t r0 = static_cast<int64_t>(blockIdx.y) * 32, c0 = static_cast<int64_t>(blockIdx.x) * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    for (int i = ty; i < 32; i += 8)
        if (r0 + i < R && c0 + tx < C) tile[i][tx] = src[(r0 + i) * C + c0 + tx];
    __syncthreads();
    for (int i = ty; i < 32; i += 8)
        if (c0 + i < C && r0 + tx < R) dst[(c0 + i) * R + r0 + tx] = tile[tx][i];
}

}  // namespace

unsigned take_dense_gemm_device_error() {
    unsigned v = 0;
    if (cudaMemcpyFromSymbol(&v, g_dense_gemm_dev_error, sizeof(v)) != cudaSuccess) return ~0u;
    if (v) {
        const unsigned zero = 0;
        cudaMemcpyToSymbol(g_dense_gemm_dev_error, &zero, sizeof(zero));
    }
    return v;
}

}  // namespace mcv

using namespace mcv;

extern "C" {

int mcv_gemm_f16(const void* x, const void* w, void* out, int64_t M, int64_t K, int64_t N, mcv_stream_t stream) {
    if (!x || !w || !out) return fail(MCV_ERR_NULL, "gemm_f16: null pointer");
    if (M < 1 || K < kDK || N < 1 || K % kDK != 0 || M > (1 << 24) || K > (1 << 20) || N > (1 << 24))
        return fail(MCV_ERR_SHAPE, "gemm_f16: need M >= 1, K a multiple of 64, N >= 1");
    if (N % 8 != 0) return fail(MCV_ERR_SHAPE, "gemm_f16: N must be a multiple of 8 (16-byte weight rows)");
    if (!aligned16(x) || !aligned16(w)) return fail(MCV_ERR_ALIGN, "gemm_f16: x and w must be 16-byte aligned");
    if (reinterpret_cast<uintptr_t>(out) & 1u) return fail(MCV_ERR_ALIGN, "gemm_f16: out must be 2-byte aligned");
    auto enc = encode_fn();
    if (!enc) return fail(MCV_ERR_CUDA, "gemm_f16: cuTensorMapEncodeTiled unavailable");
    const int64_t tiles_n = (N + kDW - 1) / kDW, tiles_m = (M + kDX - 1) / kDX;
    if (tiles_m > 65535) return fail(MCV_ERR_SHAPE, "gemm_f16: M too large");
    const int nk = static_cast<int>(K / kDK);
    int split_k = 1;
    const int forced = tuning(MCV_TUNE_GEMM_SPLIT_K);
    if (forced >= 1 && forced <= 8) {
        split_k = forced < nk ? forced : nk;
    } else {
        while (split_k < 8 && tiles_n * tiles_m * split_k * 2 <= sm_count() && nk / (split_k * 2) >= 4) split_k *= 2;
    }
    const int box_rows = M >= kDX ? kDX : static_cast<int>((M + 15) & ~int64_t(15));
    CUtensorMap xmap, wmap;
    {
        const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(M)};
        const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
        const cuuint32_t box[2] = {kDK, static_cast<cuuint32_t>(box_rows)};
        const cuuint32_t estr[2] = {1, 1};
        CUresult r = enc(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(x), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return fail(MCV_ERR_CUDA, "gemm_f16: cuTensorMapEncodeTiled(x) failed");
    }
    {
        const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(N)};
        const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
        const cuuint32_t box[2] = {kDK, kDW};
        const cuuint32_t estr[2] = {1, 1};
        CUresult r = enc(&wmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(w), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return fail(MCV_ERR_CUDA, "gemm_f16: cuTensorMapEncodeTiled(w) failed");
    }
    cudaError_t e = cudaFuncSetAttribute(dense_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kDSmemBytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(dense_gemm)");
    DenseGemmArgs ga{static_cast<__half*>(out), static_cast<int>(M), static_cast<int>(K), static_cast<int>(N), box_rows,
                     split_k};
    return launch_clustered(dense_gemm_kernel, dim3(static_cast<unsigned>(tiles_n), static_cast<unsigned>(tiles_m), split_k),
                            dim3(kDThreads), dim3(1, 1, split_k), kDSmemBytes, static_cast<cudaStream_t>(stream), xmap,
                            wmap, ga);
}

int mcv_transpose_f16(const void* src, void* dst, int64_t rows, int64_t cols, mcv_stream_t stream) {
    if (!src || !dst) return fail(MCV_ERR_NULL, "transpose_f16: null pointer");
    if (rows < 1 || cols < 1 || (rows + 31) / 32 > 65535 || (cols + 31) / 32 > 0x7fffffffLL)
        return fail(MCV_ERR_SHAPE, "transpose_f16: bad shape");
    return launch(transpose_f16_kernel, dim3(static_cast<unsigned>((cols + 31) / 32), static_cast<unsigned>((rows + 31) / 32)),
                  dim3(256), 0, static_cast<cudaStream_t>(stream), static_cast<const __half*>(src),
                  static_cast<__half*>(dst), rows, cols);
}

}  // extern "C"
