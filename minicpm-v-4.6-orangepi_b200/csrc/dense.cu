// Dense fp16 decode GEMV (M = 1..8) in both weight layouts, the fused
// lm_head GEMV + greedy argmax, and argmax over fp16 logits.
//
// Reference behaviour replaced:
//  * matmul_b_transposed at M=1 (src/csrc/lib/ops.cpp:159-209) and its cube
//    kernel (op_kernel/matmul_cube_custom.cpp:19-55);
//  * lm_head_greedy's 16 sequential [1024,16384] chunk matmuls, each followed
//    by a D2H copy of fp16 logits and a host argmax with strict '>'
//    (src/csrc/lib/language_model.cpp:412-482);
//  * argmax_last_dim (src/csrc/lib/ops.cpp:324-357).
//
// Row kernel ([N][K] weights, K contiguous): one warp per weight row, lane l
// reads 16-byte chunks l, l+32, ... of the row (512 contiguous bytes per
// warp-wide load), fp16 x fp16 products accumulate in fp32 with the sm_100
// mixed-precision FMA, and a 5-step xor-shuffle finishes the dot.  The grid
// is persistent (a multiple of the SM count) and walks rows with a stride, two
// rows per warp per step.  In argmax mode each logit becomes a 64-bit
// order-preserving key (larger logit wins, then smaller index) so the whole
// reduction is an integer max: per warp in registers, per block in shared
// memory, and across blocks through a 64-bit atomicMax per row and an
// arrival counter in the caller's workspace; the last block to arrive reads
// the result and zeroes both, so the next call needs no memset.  Each warp
// warms L2 a tunable number of row steps ahead of its loads
// (cp.async.bulk.prefetch.L2), and the first rows are loaded before
// griddepcontrol.wait.  A second launch form carries the activation rows in
// the kernel parameters (rows_kernel_xp) for callers whose x is in host
// memory; with a peer-exchange context the last block also runs the
// cross-GPU exchange (see finish_argmax).
#include <cstring>
#include <type_traits>

#include "common.cuh"
#include "neighbours.cuh"
#include "w8a8_quant.cuh"

namespace mcv {
namespace {

constexpr int kRowThreads = 256;
constexpr int kRowWarps = kRowThreads / 32;
constexpr int kRowsPerStep = 2;

static __device__ unsigned g_dense_dev_error;

// L2 prefetch of a contiguous range of this GPU's memory (16-byte aligned,
// size a multiple of 16; no multicast).
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

struct RowArgs {
    const __half* x;
    const __half* w;
    __half* out;            // GEMV mode
    unsigned* counter;      // argmax: blocks arrived (zero between calls)
    uint64_t* keys;         // argmax: [M] running maxima (zero between calls)
    uint64_t* out_key;      // argmax: [M] (may be null)
    int64_t* out_index;     // argmax: [M] (may be null)
    int64_t N;
    int K;
    int prefetch;           // L2 warm-up distance in row steps (0: none)
    int64_t n_offset;
    P2PArgs p2p;
    const __half* w_scale;  // int8 lm_head: per-row weight scales [N] (w then holds int8 rows)
    NormArgs norm;          // argmax: rms_norm of x in the prologue (norm.gamma null: x as given)
    int contiguous;         // 1: each warp walks its own contiguous row range; 0: rows strided by the grid
};

// A warp's rows: [begin, end) in steps of `step`, either strided by the grid
// (rows r, r + 2W, ...) or one contiguous range per warp.
struct RowWalk {
    int64_t begin, end, step;
};
__device__ __forceinline__ RowWalk row_walk(const RowArgs& a, int64_t gwarp, int64_t nwarps) {
    if (a.contiguous)
        return RowWalk{(gwarp * a.N) / nwarps, ((gwarp + 1) * a.N) / nwarps, kRowsPerStep};
    return RowWalk{gwarp * kRowsPerStep, a.N, nwarps * kRowsPerStep};
}

__device__ __forceinline__ void st_relaxed_sys(uint64_t* p, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// Mailbox word: bits 63..32 the key's ordered logit, bits 31..24 the call
// tag, bits 23..0 the key's low 24 bits (0xFFFFFF - index; the host limits
// indices below 2^24 - 1, so the key's bits 31..24 are all ones and need no
// room).  Key 0 ("no row") is sent as logit 0 and low bits 0.
__device__ __forceinline__ uint64_t p2p_pack(uint64_t key, uint32_t tag) {
    const uint64_t low = key == 0 ? 0 : (key & 0xffffffull);
    return (key & 0xffffffff00000000ull) | (static_cast<uint64_t>(tag) << 24) | low;
}
__device__ __forceinline__ uint64_t p2p_unpack(uint64_t word) {
    const uint64_t hi = word & 0xffffffff00000000ull, low = word & 0xffffffull;
    return (hi == 0 && low == 0) ? 0 : (hi | 0xff000000ull | low);
}
__device__ __forceinline__ uint64_t ld_relaxed_sys(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Block / grid / (optional) cross-GPU reduction of the argmax keys.  Kept
// out of line so the streaming loop above is scheduled on its own.
template <int M>
__device__ __noinline__ void finish_argmax(const RowArgs& a, const uint64_t (&best)[M], int lane, int warp) {
    __shared__ uint64_t red[kRowWarps][M];
        // keys are already warp-uniform (butterfly reduction).  Blocks fold
        // their key into one global key per row with a 64-bit atomicMax and
        // arrive on a counter with acquire-release order; the last block to
        // arrive reads the final keys and resets both for the next call.
        if (lane == 0) {
#pragma unroll
            for (int m = 0; m < M; ++m) red[warp][m] = best[m];
        }
        __syncthreads();
        __shared__ int is_last;
        if (threadIdx.x == 0) {
#pragma unroll
            for (int m = 0; m < M; ++m) {
                uint64_t b = 0;
                for (int wi = 0; wi < kRowWarps; ++wi) b = red[wi][m] > b ? red[wi][m] : b;
                atomicMax(reinterpret_cast<unsigned long long*>(a.keys + m), static_cast<unsigned long long>(b));
            }
            unsigned prev;
            asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(a.counter) : "memory");
            is_last = (prev == gridDim.x - 1);
        }
        __syncthreads();
        if (is_last) {
            __shared__ uint64_t loc[M];
            if (threadIdx.x == 0) {
#pragma unroll
                for (int m = 0; m < M; ++m) {
                    loc[m] = __ldcg(a.keys + m);
                    a.keys[m] = 0;  // leave the workspace ready for the next call
                }
                *a.counter = 0u;
            }
            __syncthreads();
            if (a.p2p.nranks > 1) {
                // Exchange: thread j = (r, m) stores this rank's key of row m
                // into rank r's mailbox, then waits (bounded) for rank j/M's
                // key of row m in its own mailbox.  A slot is one 64-bit word
                // holding the key and an 8-bit call tag (p2p_pack), so one
                // relaxed system-scope store publishes both and no fence is
                // needed on either side.  Slots alternate by call parity, so
                // a fast rank's next call never overwrites a slot a slow rank
                // has yet to read.
                __shared__ uint64_t got[8][M];
                __shared__ int failed;
                if (threadIdx.x == 0) failed = 0;
                __syncthreads();
                const int R = a.p2p.nranks;
                const uint64_t seq = *a.p2p.seq_dev + 1;
                const int par = static_cast<int>(seq & 1);
                const uint32_t tag = static_cast<uint32_t>(seq & 0xffu);
                const int j = threadIdx.x;
                if (j < R * M) {
                    const int r = j / M, m = j % M;
                    st_relaxed_sys(a.p2p.mbox[r] + (par * 8 + a.p2p.rank) * 8 + m, p2p_pack(loc[m], tag));
                }
                if (j < R * M) {
                    const int r = j / M, m = j % M;
                    const uint64_t* slot = a.p2p.mbox[a.p2p.rank] + (par * 8 + r) * 8 + m;
                    uint64_t key = 0;
                    const uint64_t t0 = globaltimer_ns();
                    for (uint32_t spin = 0;; ++spin) {
                        const uint64_t word = ld_relaxed_sys(slot);
                        if (((word >> 24) & 0xffu) == tag) {
                            key = p2p_unpack(word);
                            break;
                        }
                        if ((spin & 63u) == 63u && globaltimer_ns() - t0 > 1000000000ull) {
                            atomicOr(a.p2p.err, kDevErrTimeout);  // a peer never arrived
                            failed = 1;
                            break;
                        }
                    }
                    got[r][m] = key;
                }
                __syncthreads();
                if (threadIdx.x < M) {
                    const int m = threadIdx.x;
                    uint64_t b = 0;
                    for (int r = 0; r < R; ++r) b = got[r][m] > b ? got[r][m] : b;
                    loc[m] = failed ? 0 : b;  // no answer rather than a partial one
                }
                __syncthreads();
                if (threadIdx.x == 0) *a.p2p.seq_dev = seq;
            }
            if (threadIdx.x < M) {
                const int m = threadIdx.x;
                const uint64_t b = loc[m];
                if (a.out_key) a.out_key[m] = b;
                if (a.out_index)
                    a.out_index[m] = b == 0 ? -1 : static_cast<int64_t>(0xffffffffu - static_cast<uint32_t>(b & 0xffffffffu));
            }
        }
}

// The activation rows normally come from global memory (a.x).  A launch can
// instead carry them in its parameters (RowArgsXP, up to kXParamChunks
// 16-byte chunks): a host-memory x then needs no copy-in before the kernel.
constexpr int kXParamChunks = 256;  // 4 KB: M * K <= 2048
struct RowArgsXP {
    RowArgs a;
    uint4 x[kXParamChunks];
};
__host__ __device__ __forceinline__ const RowArgs& row_args(const RowArgs& a) { return a; }
__host__ __device__ __forceinline__ const RowArgs& row_args(const RowArgsXP& ax) { return ax.a; }

template <int M, int KCH, bool ARGMAX, bool FP16_LOGITS>
__device__ __forceinline__ void rows_body(const RowArgs& a, const uint4* xsrc) {
    extern __shared__ uint4 xs[];  // x as [M][K/8] 16-byte chunks
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int chunks = a.K >> 3;
    const int64_t gwarp = static_cast<int64_t>(blockIdx.x) * kRowWarps + warp;
    const int64_t nwarps = static_cast<int64_t>(gridDim.x) * kRowWarps;
    const uint4* w4 = reinterpret_cast<const uint4*>(a.w);

    // Prefetch this warp's first rows before waiting on the previous kernel.
    uint4 wv[kRowsPerStep][KCH];
    const RowWalk walk = row_walk(a, gwarp, nwarps);
    int64_t r = walk.begin;
    const int64_t step = walk.step, rend = walk.end;
#pragma unroll
    for (int t = 0; t < kRowsPerStep; ++t)
#pragma unroll
        for (int i = 0; i < KCH; ++i) {
            const int c = lane + 32 * i;
            if (r + t < rend && c < chunks) wv[t][i] = ld_stream(w4 + (r + t) * chunks + c);
        }
    // Warm L2 with this warp's next few row pairs too (bulk prefetch, no
    // registers): the weights never depend on the previous kernel, so their
    // stream can start before griddepcontrol.wait releases.
    // Later steps keep the warm-up a.prefetch steps ahead of the loads.
    if (lane < kRowsPerStep * a.prefetch) {
        const int64_t pr = r + step * (1 + lane / kRowsPerStep) + (lane % kRowsPerStep);
        if (pr < rend) prefetch_l2(w4 + pr * chunks, static_cast<uint32_t>(a.K) * 2u);
    }
    pdl_trigger();
    pdl_wait();
    if (a.norm.gamma != nullptr) {
        // lm_head_greedy's rms_norm (language_model.cpp:423), recomputed by
        // every block from the raw hidden rows: x is 2 KB per row, and the
        // first weight rows are already in flight
        rms_norm_rows_block<M>(reinterpret_cast<const __half*>(xsrc), reinterpret_cast<__half*>(xs), a.K, a.norm);
    } else {
        for (int idx = threadIdx.x; idx < M * chunks; idx += kRowThreads)
            xs[idx] = xsrc[idx];
        __syncthreads();
    }

    uint64_t best[M];
#pragma unroll
    for (int m = 0; m < M; ++m) best[m] = 0;

    while (r < rend) {
        float acc0[kRowsPerStep][M], acc1[kRowsPerStep][M];
#pragma unroll
        for (int t = 0; t < kRowsPerStep; ++t)
#pragma unroll
            for (int m = 0; m < M; ++m) acc0[t][m] = acc1[t][m] = 0.0f;
#pragma unroll
        for (int i = 0; i < KCH; ++i) {
            const int c = lane + 32 * i;
            if (c < chunks) {
#pragma unroll
                for (int m = 0; m < M; ++m) {
                    const uint4 xv = xs[m * chunks + c];
#pragma unroll
                    for (int t = 0; t < kRowsPerStep; ++t) {
                        fma2_f16_f32(acc0[t][m], acc1[t][m], wv[t][i].x, xv.x);
                        fma2_f16_f32(acc0[t][m], acc1[t][m], wv[t][i].y, xv.y);
                        fma2_f16_f32(acc0[t][m], acc1[t][m], wv[t][i].z, xv.z);
                        fma2_f16_f32(acc0[t][m], acc1[t][m], wv[t][i].w, xv.w);
                    }
                }
            }
        }
        // issue the next step's loads before reducing this one
        const int64_t rn = r + step;
        if (lane < kRowsPerStep && a.prefetch > 0) {
            const int64_t pr = rn + step * a.prefetch + lane;
            if (pr < rend) prefetch_l2(w4 + pr * chunks, static_cast<uint32_t>(a.K) * 2u);
        }
#pragma unroll
        for (int t = 0; t < kRowsPerStep; ++t)
#pragma unroll
            for (int i = 0; i < KCH; ++i) {
                const int c = lane + 32 * i;
                if (rn + t < rend && c < chunks) wv[t][i] = ld_stream(w4 + (rn + t) * chunks + c);
            }
#pragma unroll
        for (int t = 0; t < kRowsPerStep; ++t) {
            const int64_t row = r + t;
#pragma unroll
            for (int m = 0; m < M; ++m) {
                float v = warp_sum(acc0[t][m] + acc1[t][m]);
                if (row < rend) {
                    if constexpr (ARGMAX) {
                        if constexpr (FP16_LOGITS) v = __half2float(__float2half_rn(v));
                        const uint64_t key = argmax_key(v, static_cast<uint32_t>(a.n_offset + row));
                        best[m] = key > best[m] ? key : best[m];
                    } else {
                        if (lane == m) a.out[static_cast<int64_t>(m) * a.N + row] = __float2half_rn(v);
                    }
                }
            }
        }
        r = rn;
    }

    if constexpr (ARGMAX) finish_argmax<M>(a, best, lane, warp);
}

template <int M, int KCH, bool ARGMAX, bool FP16_LOGITS>
__global__ void __launch_bounds__(kRowThreads)
rows_kernel(RowArgs a) {
    rows_body<M, KCH, ARGMAX, FP16_LOGITS>(a, reinterpret_cast<const uint4*>(a.x));
}

// the same, with the activation rows carried in the launch parameters
template <int M, int KCH, bool ARGMAX, bool FP16_LOGITS>
__global__ void __launch_bounds__(kRowThreads)
rows_kernel_xp(const __grid_constant__ RowArgsXP ax) {
    const RowArgs a = ax.a;
    rows_body<M, KCH, ARGMAX, FP16_LOGITS>(a, ax.x);
}

// [K][N] natural layout: each thread owns 8 consecutive columns (one 16-byte
// load per k row); 4 threads span 32 columns, 64 threads split K; partial
// sums meet in shared memory.
constexpr int kKnTx = 4;
constexpr int kKnTy = 64;

template <int M>
__global__ void __launch_bounds__(kKnTx * kKnTy)
gemv_kn_kernel(const __half* __restrict__ x, const __half* __restrict__ w, __half* __restrict__ out,
               int K, int N) {
    extern __shared__ float red_kn[];  // [kKnTy][M][kKnTx*8]
    const int tx = threadIdx.x % kKnTx;
    const int ty = threadIdx.x / kKnTx;
    const int n0 = blockIdx.x * (kKnTx * 8) + tx * 8;
    pdl_trigger();
    pdl_wait();
    float acc[M][8];
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[m][e] = 0.0f;
    if (n0 < N) {
        for (int k = ty; k < K; k += kKnTy) {
            const uint4 wv = ld_stream(w + static_cast<int64_t>(k) * N + n0);
#pragma unroll
            for (int m = 0; m < M; ++m) {
                const __half xh = x[static_cast<int64_t>(m) * K + k];
                const uint32_t xx = h2_as_u32(__halves2half2(xh, xh));
                fma2_f16_f32(acc[m][0], acc[m][1], wv.x, xx);
                fma2_f16_f32(acc[m][2], acc[m][3], wv.y, xx);
                fma2_f16_f32(acc[m][4], acc[m][5], wv.z, xx);
                fma2_f16_f32(acc[m][6], acc[m][7], wv.w, xx);
            }
        }
    }
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
        for (int e = 0; e < 8; ++e) red_kn[(ty * M + m) * (kKnTx * 8) + tx * 8 + e] = acc[m][e];
    __syncthreads();
    for (int o = threadIdx.x; o < M * kKnTx * 8; o += kKnTx * kKnTy) {
        const int m = o / (kKnTx * 8);
        const int col = o % (kKnTx * 8);
        float s = 0.0f;
        for (int t = 0; t < kKnTy; ++t) s += red_kn[(t * M + m) * (kKnTx * 8) + col];
        const int n = blockIdx.x * (kKnTx * 8) + col;
        if (n < N) out[static_cast<int64_t>(m) * N + n] = __float2half_rn(s);
    }
}

constexpr int kArgThreads = 512;

__global__ void __launch_bounds__(kArgThreads)
argmax_rows_kernel(const __half* __restrict__ logits, int64_t* __restrict__ out, int64_t V) {
    __shared__ uint64_t red[kArgThreads / 32];
    pdl_trigger();
    pdl_wait();
    const __half* row = logits + static_cast<int64_t>(blockIdx.x) * V;
    uint64_t best = 0;
    for (int64_t v = threadIdx.x; v < V; v += kArgThreads) {
        const uint64_t k = argmax_key(__half2float(row[v]), static_cast<uint32_t>(v));
        best = k > best ? k : best;
    }
    best = warp_max_u64(best);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint64_t b = 0;
        for (int i = 0; i < kArgThreads / 32; ++i) b = red[i] > b ? red[i] : b;
        out[blockIdx.x] = static_cast<int64_t>(0xffffffffu - static_cast<uint32_t>(b & 0xffffffffu));
    }
}

__global__ void key_to_index_kernel(const uint64_t* __restrict__ key, int64_t* __restrict__ out, int M) {
    pdl_trigger();
    pdl_wait();
    const int m = threadIdx.x;
    // key 0 means "no row" (every shard empty): -1, as finish_argmax reports it
    if (m < M) out[m] = key[m] == 0 ? -1 : static_cast<int64_t>(0xffffffffu - static_cast<uint32_t>(key[m] & 0xffffffffu));
}

// Rows per SM below which the short-walk settings apply (4 blocks per SM,
// one-step L2 warm-up): a vocabulary shard on 4 or 8 GPUs.
constexpr int64_t kShortWalkRowsPerSm = 600;

int row_grid(int64_t N) {
    // persistent grid: up to 4 blocks of 256 threads per SM, never more
    // blocks than there are row pairs to hand out.  Default: 4 blocks per SM
    // on short walks, 2 on long ones (measured on B200, K = 1024, strided
    // walk: 31,012 rows 13.1 vs 13.8 us, 62,024 rows 22.8 vs 23.4 us, but
    // 124,047 rows 45.3 vs 41.2 us and 248,094 rows 84.6 vs 76.7 us).
    const int64_t warps_needed = (N + kRowsPerStep - 1) / kRowsPerStep;
    const int64_t blocks_needed = (warps_needed + kRowWarps - 1) / kRowWarps;
    const int t = tuning(MCV_TUNE_ROWS_BLOCKS_PER_SM);
    const bool short_walk = N <= kShortWalkRowsPerSm * sm_count();
    const int bps = (t >= 1 && t <= 4) ? t : (short_walk ? 4 : 2);  // <= 4: the workspace is sized for 4
    const int64_t cap = static_cast<int64_t>(sm_count()) * bps;
    return static_cast<int>(blocks_needed < cap ? blocks_needed : cap);
}

// L2 warm-up distance in row steps: MCV_TUNE_ROWS_PREFETCH 1..16, -1 none.
// Default: one step ahead on short walks (see row_grid), none on long ones,
// where the warm-up only competes with the demand loads.  Measured on B200,
// K = 1024, 4 blocks per SM: 31,012 rows 13.1 us with one step against 14.7
// with none and 15.0 with two; 248,094 rows on 2 blocks per SM 76.7 us with
// none against 82.9 with one.
int row_prefetch(int64_t N, int grid) {
    (void)grid;
    const int t = tuning(MCV_TUNE_ROWS_PREFETCH);
    if (t < 0) return 0;
    if (t >= 1 && t <= 16) return t;
    return N <= kShortWalkRowsPerSm * sm_count() ? 1 : 0;
}

// Row walk: MCV_TUNE_ROWS_WALK 1 = rows strided by the grid (default), 2 =
// a contiguous range per warp (every warp within one row of the same count,
// but measured 3-6 % slower at every size from 31k to 248k rows).
int row_contiguous() { return tuning(MCV_TUNE_ROWS_WALK) == 2 ? 1 : 0; }

template <int M, bool ARGMAX, bool FP16, class Args>
int launch_rows_m(int kch, const Args& args, cudaStream_t s, int grid) {
    const size_t smem = static_cast<size_t>(M) * row_args(args).K * 2;
    auto pick = [&](auto kern) -> int {
        if (smem > 48 * 1024) {
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(smem));
            if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(rows_kernel)");
        }
        // a persistent grid: never more blocks than are resident at once
        // (the wider-M variants use more than 64 registers, so fewer than 4
        // of their blocks fit on an SM)
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kRowThreads, smem) == cudaSuccess &&
            per_sm > 0 && grid > per_sm * sm_count())
            grid = per_sm * sm_count();
        return launch(kern, dim3(grid), dim3(kRowThreads), smem, s, args);
    };
    switch (kch) {
        case 1:
            if constexpr (std::is_same_v<Args, RowArgsXP>) return pick(rows_kernel_xp<M, 1, ARGMAX, FP16>);
            else return pick(rows_kernel<M, 1, ARGMAX, FP16>);
        case 2:
            if constexpr (std::is_same_v<Args, RowArgsXP>) return pick(rows_kernel_xp<M, 2, ARGMAX, FP16>);
            else return pick(rows_kernel<M, 2, ARGMAX, FP16>);
        case 4:
            if constexpr (std::is_same_v<Args, RowArgsXP>) return pick(rows_kernel_xp<M, 4, ARGMAX, FP16>);
            else return pick(rows_kernel<M, 4, ARGMAX, FP16>);
        case 8:
            if constexpr (std::is_same_v<Args, RowArgsXP>) return pick(rows_kernel_xp<M, 8, ARGMAX, FP16>);
            else return pick(rows_kernel<M, 8, ARGMAX, FP16>);
        default: return fail(MCV_ERR_SHAPE, "row kernel: K above 16384 unsupported");
    }
}

template <bool ARGMAX, bool FP16, class Args>
int launch_rows(int64_t M, const Args& a, cudaStream_t s, int grid) {
    const int chunks_per_lane = (row_args(a).K / 8 + 31) / 32;
    int kch = 1;
    while (kch < chunks_per_lane) kch *= 2;
    switch (M) {
        case 1: return launch_rows_m<1, ARGMAX, FP16>(kch, a, s, grid);
        case 2: return launch_rows_m<2, ARGMAX, FP16>(kch, a, s, grid);
        case 3: return launch_rows_m<3, ARGMAX, FP16>(kch, a, s, grid);
        case 4: return launch_rows_m<4, ARGMAX, FP16>(kch, a, s, grid);
        case 5: return launch_rows_m<5, ARGMAX, FP16>(kch, a, s, grid);
        case 6: return launch_rows_m<6, ARGMAX, FP16>(kch, a, s, grid);
        case 7: return launch_rows_m<7, ARGMAX, FP16>(kch, a, s, grid);
        default: return launch_rows_m<8, ARGMAX, FP16>(kch, a, s, grid);
    }
}

// ---- int8 (W8A8) lm_head + greedy argmax ------------------------------------
// The W8A8 branch of lm_head_greedy (src/csrc/lib/language_model.cpp:430-479):
// x is quantized per row as w8a8_quantize does, each logit is the int32 dot
// with a weight row dequantized as w8a8_dequant does, RN((acc * ws) * xs) to
// fp16, and the host reads those fp16 logits with subnormals flushed to zero
// (its h2f, :444-458) before the strict '>' first-max scan.  Same walk as
// rows_body over int8 rows of K bytes (half the fp16 traffic), same keys and
// last-block finish (peer exchange included).

// fp16 -> float the way the reference's host argmax reads logits
__device__ __forceinline__ float h2f_flush_subnormal(__half h) {
    const unsigned short b = __half_as_ushort(h);
    if (((b >> 10) & 0x1fu) == 0u) return (b & 0x8000u) ? -0.0f : 0.0f;
    return __half2float(h);
}

template <int M, int KCH>
__global__ void __launch_bounds__(kRowThreads)
rows_w8_kernel(RowArgs a) {
    extern __shared__ uint4 xs[];  // int8 x as [M][K/16] 16-byte chunks
    __shared__ float xscale_s[M];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int chunks = a.K >> 4;
    const int64_t gwarp = static_cast<int64_t>(blockIdx.x) * kRowWarps + warp;
    const int64_t nwarps = static_cast<int64_t>(gridDim.x) * kRowWarps;
    const uint4* w4 = reinterpret_cast<const uint4*>(a.w);

    uint4 wv[kRowsPerStep][KCH];
    float wsc[kRowsPerStep];
    const RowWalk walk = row_walk(a, gwarp, nwarps);
    int64_t r = walk.begin;
    const int64_t step = walk.step, rend = walk.end;
#pragma unroll
    for (int t = 0; t < kRowsPerStep; ++t) {
        wsc[t] = r + t < rend ? __half2float(a.w_scale[r + t]) : 0.0f;
#pragma unroll
        for (int i = 0; i < KCH; ++i) {
            const int c = lane + 32 * i;
            wv[t][i] = make_uint4(0, 0, 0, 0);
            if (r + t < rend && c < chunks) wv[t][i] = ld_stream(w4 + (r + t) * chunks + c);
        }
    }
    if (lane < kRowsPerStep * a.prefetch) {
        const int64_t pr = r + step * (1 + lane / kRowsPerStep) + (lane % kRowsPerStep);
        if (pr < rend) prefetch_l2(w4 + pr * chunks, static_cast<uint32_t>(a.K));
    }
    pdl_trigger();
    pdl_wait();
    quantize_rows_to_smem<M, (KCH + 3) / 4, kRowThreads>(a.x, a.K, reinterpret_cast<int8_t*>(xs), a.K, xscale_s,
                                                         nullptr, nullptr);
    __syncthreads();

    uint64_t best[M];
#pragma unroll
    for (int m = 0; m < M; ++m) best[m] = 0;

    while (r < rend) {
        int acc[kRowsPerStep][M];
#pragma unroll
        for (int t = 0; t < kRowsPerStep; ++t)
#pragma unroll
            for (int m = 0; m < M; ++m) acc[t][m] = 0;
#pragma unroll
        for (int i = 0; i < KCH; ++i) {
            const int c = lane + 32 * i;
            if (c < chunks) {
#pragma unroll
                for (int m = 0; m < M; ++m) {
                    const uint4 xv = xs[m * chunks + c];
#pragma unroll
                    for (int t = 0; t < kRowsPerStep; ++t) {
                        int v = acc[t][m];
                        v = __dp4a(static_cast<int>(wv[t][i].x), static_cast<int>(xv.x), v);
                        v = __dp4a(static_cast<int>(wv[t][i].y), static_cast<int>(xv.y), v);
                        v = __dp4a(static_cast<int>(wv[t][i].z), static_cast<int>(xv.z), v);
                        v = __dp4a(static_cast<int>(wv[t][i].w), static_cast<int>(xv.w), v);
                        acc[t][m] = v;
                    }
                }
            }
        }
        // issue the next step's loads before reducing this one
        const int64_t rn = r + step;
        if (lane < kRowsPerStep && a.prefetch > 0) {
            const int64_t pr = rn + step * a.prefetch + lane;
            if (pr < rend) prefetch_l2(w4 + pr * chunks, static_cast<uint32_t>(a.K));
        }
        float wsn[kRowsPerStep];
#pragma unroll
        for (int t = 0; t < kRowsPerStep; ++t) {
            wsn[t] = rn + t < rend ? __half2float(a.w_scale[rn + t]) : 0.0f;
#pragma unroll
            for (int i = 0; i < KCH; ++i) {
                const int c = lane + 32 * i;
                if (rn + t < rend && c < chunks) wv[t][i] = ld_stream(w4 + (rn + t) * chunks + c);
            }
        }
#pragma unroll
        for (int t = 0; t < kRowsPerStep; ++t) {
            const int64_t row = r + t;
#pragma unroll
            for (int m = 0; m < M; ++m) {
                int v = acc[t][m];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                if (row < rend) {
                    const __half h = __float2half_rn(__fmul_rn(__fmul_rn(__int2float_rn(v), wsc[t]), xscale_s[m]));
                    const uint64_t key = argmax_key(h2f_flush_subnormal(h), static_cast<uint32_t>(a.n_offset + row));
                    best[m] = key > best[m] ? key : best[m];
                }
            }
        }
#pragma unroll
        for (int t = 0; t < kRowsPerStep; ++t) wsc[t] = wsn[t];
        r = rn;
    }
    finish_argmax<M>(a, best, lane, warp);
}

template <int M>
int launch_rows_w8_m(int kch, const RowArgs& a, cudaStream_t s, int grid) {
    const size_t smem = static_cast<size_t>(M) * a.K;
    auto pick = [&](auto kern) -> int {
        if (smem > 48 * 1024) {
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(smem));
            if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(rows_w8_kernel)");
        }
        return launch(kern, dim3(grid), dim3(kRowThreads), smem, s, a);
    };
    switch (kch) {
        case 1: return pick(rows_w8_kernel<M, 1>);
        case 2: return pick(rows_w8_kernel<M, 2>);
        case 4: return pick(rows_w8_kernel<M, 4>);
        case 8: return pick(rows_w8_kernel<M, 8>);
        default: return fail(MCV_ERR_SHAPE, "lm_head_w8a8: K above 4096 unsupported");
    }
}

int launch_rows_w8(int64_t M, const RowArgs& a, cudaStream_t s, int grid) {
    const int chunks_per_lane = (a.K / 16 + 31) / 32;
    int kch = 1;
    while (kch < chunks_per_lane) kch *= 2;
    switch (M) {
        case 1: return launch_rows_w8_m<1>(kch, a, s, grid);
        case 2: return launch_rows_w8_m<2>(kch, a, s, grid);
        case 3: return launch_rows_w8_m<3>(kch, a, s, grid);
        case 4: return launch_rows_w8_m<4>(kch, a, s, grid);
        case 5: return launch_rows_w8_m<5>(kch, a, s, grid);
        case 6: return launch_rows_w8_m<6>(kch, a, s, grid);
        case 7: return launch_rows_w8_m<7>(kch, a, s, grid);
        default: return launch_rows_w8_m<8>(kch, a, s, grid);
    }
}

int check_rows(const void* x, const void* w, int64_t M, int64_t K, int64_t N) {
    if (!x || !w) return fail(MCV_ERR_NULL, "null x or w");
    if (M < 1 || M > 8) return fail(MCV_ERR_SHAPE, "M must be 1..8");
    if (K <= 0 || N <= 0 || K % 8 != 0) return fail(MCV_ERR_SHAPE, "K must be a positive multiple of 8 and N positive");
    if (K > 16384) return fail(MCV_ERR_SHAPE, "K above 16384 unsupported");
    if (!aligned16(x) || !aligned16(w)) return fail(MCV_ERR_ALIGN, "x and w must be 16-byte aligned");
    return MCV_OK;
}

}  // namespace

// Used by the collective entry points (collective.cu, p2p.cu).
// x_param (host memory, may be null): when set and M * K fits the launch
// parameters, the rows are passed by value in the launch and x is not read.
int lm_head_argmax_impl_p2p(const void* x, const void* w, void* out_key, void* out_index, int64_t M,
                            int64_t K, int64_t N, int64_t n_offset, int fp16_logits, void* ws,
                            size_t ws_bytes, cudaStream_t s, const P2PArgs* p2p, const void* x_param,
                            const NormArgs* norm) {
    const bool by_param = x_param != nullptr && M * K <= kXParamChunks * 8;
    int st = check_rows(by_param ? w : x, w, M, K, N);
    if (st) return st;
    if (n_offset < 0 || n_offset + N > 0xffffffffLL) return fail(MCV_ERR_SHAPE, "lm_head: global vocab index must fit 32 bits");
    if (!ws) return fail(MCV_ERR_WORKSPACE, "lm_head: workspace is null");
    if (ws_bytes < mcv_lm_head_workspace_size(M)) return fail(MCV_ERR_WORKSPACE, "lm_head: workspace too small");
    if (reinterpret_cast<uintptr_t>(ws) & 7u) return fail(MCV_ERR_ALIGN, "lm_head: workspace must be 8-byte aligned");
    const int grid = row_grid(N);
    RowArgs a{};
    a.prefetch = row_prefetch(N, grid);
    a.contiguous = row_contiguous();
    a.x = static_cast<const __half*>(x);
    a.w = static_cast<const __half*>(w);
    a.counter = static_cast<unsigned*>(ws);
    a.keys = reinterpret_cast<uint64_t*>(static_cast<char*>(ws) + 64);
    a.out_key = static_cast<uint64_t*>(out_key);
    a.out_index = static_cast<int64_t*>(out_index);
    a.N = N;
    a.K = static_cast<int>(K);
    a.n_offset = n_offset;
    if (p2p) a.p2p = *p2p;
    if (norm && norm->gamma) {
        if (norm->variant != 0 && norm->variant != 1) return fail(MCV_ERR_VALUE, "lm_head: norm variant must be 0 or 1");
        a.norm = *norm;
    }
    if (by_param) {
        RowArgsXP ax{};
        ax.a = a;
        ax.a.x = nullptr;
        std::memcpy(ax.x, x_param, static_cast<size_t>(M * K) * 2);
        return fp16_logits ? launch_rows<true, true>(M, ax, s, grid) : launch_rows<true, false>(M, ax, s, grid);
    }
    return fp16_logits ? launch_rows<true, true>(M, a, s, grid) : launch_rows<true, false>(M, a, s, grid);
}

// W8A8 lm_head: int8 weight rows [N][K] + fp16 per-row scales (see rows_w8_kernel).
int lm_head_argmax_w8a8_impl(const void* x, const void* w, const void* w_scale, void* out_key, void* out_index,
                             int64_t M, int64_t K, int64_t N, int64_t n_offset, void* ws, size_t ws_bytes,
                             cudaStream_t s, const P2PArgs* p2p) {
    if (!w_scale) return fail(MCV_ERR_NULL, "lm_head_w8a8: null weight scales");
    int st = check_rows(x, w, M, K, N);
    if (st) return st;
    if (K % 16 != 0 || K > 4096) return fail(MCV_ERR_SHAPE, "lm_head_w8a8: K must be a multiple of 16, at most 4096");
    if (n_offset < 0 || n_offset + N > 0xffffffffLL) return fail(MCV_ERR_SHAPE, "lm_head: global vocab index must fit 32 bits");
    if (!ws) return fail(MCV_ERR_WORKSPACE, "lm_head: workspace is null");
    if (ws_bytes < mcv_lm_head_workspace_size(M)) return fail(MCV_ERR_WORKSPACE, "lm_head: workspace too small");
    if (reinterpret_cast<uintptr_t>(ws) & 7u) return fail(MCV_ERR_ALIGN, "lm_head: workspace must be 8-byte aligned");
    // int8 rows are half as long as fp16 ones: 4 blocks per SM (48
    // registers) keep as many bytes in flight as the fp16 kernel's 2
    // (MCV_TUNE_ROWS_BLOCKS_PER_SM overrides)
    const int t = tuning(MCV_TUNE_ROWS_BLOCKS_PER_SM);
    const int64_t warps_needed = (N + kRowsPerStep - 1) / kRowsPerStep;
    const int64_t blocks_needed = (warps_needed + kRowWarps - 1) / kRowWarps;
    const int64_t cap = static_cast<int64_t>(sm_count()) * ((t >= 1 && t <= 4) ? t : 4);
    const int grid = static_cast<int>(blocks_needed < cap ? blocks_needed : cap);
    RowArgs a{};
    a.prefetch = row_prefetch(N, grid);
    a.contiguous = row_contiguous();
    a.x = static_cast<const __half*>(x);
    a.w = static_cast<const __half*>(w);
    a.w_scale = static_cast<const __half*>(w_scale);
    a.counter = static_cast<unsigned*>(ws);
    a.keys = reinterpret_cast<uint64_t*>(static_cast<char*>(ws) + 64);
    a.out_key = static_cast<uint64_t*>(out_key);
    a.out_index = static_cast<int64_t*>(out_index);
    a.N = N;
    a.K = static_cast<int>(K);
    a.n_offset = n_offset;
    if (p2p) a.p2p = *p2p;
    return launch_rows_w8(M, a, s, grid);
}

unsigned take_dense_device_error() {
    unsigned v = 0;
    if (cudaMemcpyFromSymbol(&v, g_dense_dev_error, sizeof(v)) != cudaSuccess) return ~0u;
    if (v) {
        const unsigned zero = 0;
        cudaMemcpyToSymbol(g_dense_dev_error, &zero, sizeof(zero));
    }
    return v;
}

int lm_head_argmax_impl(const void* x, const void* w, void* out_key, void* out_index, int64_t M,
                        int64_t K, int64_t N, int64_t n_offset, int fp16_logits, void* ws,
                        size_t ws_bytes, cudaStream_t s) {
    return lm_head_argmax_impl_p2p(x, w, out_key, out_index, M, K, N, n_offset, fp16_logits, ws, ws_bytes, s,
                                   nullptr, nullptr, nullptr);
}

int key_to_index_impl(const void* key, void* out_index, int64_t M, cudaStream_t s) {
    return launch(key_to_index_kernel, dim3(1), dim3(32), 0, s, static_cast<const uint64_t*>(key),
                  static_cast<int64_t*>(out_index), static_cast<int>(M));
}

}  // namespace mcv

using namespace mcv;

extern "C" {

int mcv_gemv_f16(const void* x, const void* w, void* out, int64_t M, int64_t K, int64_t N, int w_layout,
                 mcv_stream_t stream) {
    int st = check_rows(x, w, M, K, N);
    if (st) return st;
    if (!out) return fail(MCV_ERR_NULL, "gemv_f16: null out");
    auto s = static_cast<cudaStream_t>(stream);
    if (w_layout == 0) {
        if (N > 0x7fffffffLL) return fail(MCV_ERR_SHAPE, "gemv_f16: N too large");
        RowArgs a{};
        a.prefetch = row_prefetch(N, row_grid(N));
        a.contiguous = row_contiguous();
        a.x = static_cast<const __half*>(x);
        a.w = static_cast<const __half*>(w);
        a.out = static_cast<__half*>(out);
        a.N = N;
        a.K = static_cast<int>(K);
        return launch_rows<false, false>(M, a, s, row_grid(N));
    }
    if (w_layout != 1) return fail(MCV_ERR_VALUE, "gemv_f16: w_layout must be 0 ([N][K]) or 1 ([K][N])");
    if (N % 8 != 0) return fail(MCV_ERR_SHAPE, "gemv_f16: [K][N] layout needs N % 8 == 0");
    const dim3 grid(static_cast<unsigned>((N + kKnTx * 8 - 1) / (kKnTx * 8)));
    const dim3 block(kKnTx * kKnTy);
    const size_t smem = static_cast<size_t>(kKnTy) * M * kKnTx * 8 * sizeof(float);
    auto xs = static_cast<const __half*>(x);
    auto ws = static_cast<const __half*>(w);
    auto o = static_cast<__half*>(out);
    const int k = static_cast<int>(K), n = static_cast<int>(N);
    auto go = [&](auto kern) -> int {
        if (smem > 48 * 1024) {
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
            if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemv_kn)");
        }
        return launch(kern, grid, block, smem, s, xs, ws, o, k, n);
    };
    switch (M) {
        case 1: return go(gemv_kn_kernel<1>);
        case 2: return go(gemv_kn_kernel<2>);
        case 3: return go(gemv_kn_kernel<3>);
        case 4: return go(gemv_kn_kernel<4>);
        case 5: return go(gemv_kn_kernel<5>);
        case 6: return go(gemv_kn_kernel<6>);
        case 7: return go(gemv_kn_kernel<7>);
        default: return go(gemv_kn_kernel<8>);
    }
}

size_t mcv_lm_head_workspace_size(int64_t M) {
    if (M < 1) M = 1;
    // a 64-byte counter slot and one 64-bit key per row, in a 256-byte header
    (void)M;
    return 256;
}

int mcv_lm_head_argmax(const void* x, const void* w, void* out_key, void* out_index, int64_t M, int64_t K,
                       int64_t N_shard, int64_t n_offset, int fp16_logits, void* workspace,
                       size_t workspace_bytes, mcv_stream_t stream) {
    if (!out_key && !out_index) return fail(MCV_ERR_NULL, "lm_head_argmax: out_key and out_index both null");
    return lm_head_argmax_impl(x, w, out_key, out_index, M, K, N_shard, n_offset, fp16_logits, workspace,
                               workspace_bytes, static_cast<cudaStream_t>(stream));
}

int mcv_lm_head_argmax_rmsnorm(void* p2p_ctx, const void* x, const void* norm_gamma, float norm_eps,
                               int norm_variant, const void* w, void* out_key, void* out_index, int64_t M,
                               int64_t K, int64_t N_shard, int64_t n_offset, int fp16_logits, void* workspace,
                               size_t workspace_bytes, mcv_stream_t stream) {
    if (!out_key && !out_index) return fail(MCV_ERR_NULL, "lm_head_argmax_rmsnorm: out_key and out_index both null");
    if (!norm_gamma) return fail(MCV_ERR_NULL, "lm_head_argmax_rmsnorm: null gamma");
    if (norm_variant != 0 && norm_variant != 1) return fail(MCV_ERR_VALUE, "lm_head_argmax_rmsnorm: variant must be 0 or 1");
    const P2PArgs* pa = nullptr;
    if (p2p_ctx) {
        int st = MCV_OK;
        pa = p2p_args_checked(p2p_ctx, n_offset, N_shard, &st);
        if (st) return st;
    }
    const NormArgs na{static_cast<const __half*>(norm_gamma), norm_eps, norm_variant};
    return lm_head_argmax_impl_p2p(x, w, out_key, out_index, M, K, N_shard, n_offset, fp16_logits, workspace,
                                   workspace_bytes, static_cast<cudaStream_t>(stream), pa, nullptr, &na);
}

int mcv_argmax_last_dim_f16(const void* logits, void* out_index, int64_t M, int64_t V, mcv_stream_t stream) {
    if (!logits || !out_index) return fail(MCV_ERR_NULL, "argmax_last_dim: null pointer");
    if (M < 1 || M > 0x7fffffffLL || V < 1 || V > 0xffffffffLL) return fail(MCV_ERR_SHAPE, "argmax_last_dim: bad shape");
    return launch(argmax_rows_kernel, dim3(static_cast<unsigned>(M)), dim3(kArgThreads), 0,
                  static_cast<cudaStream_t>(stream), static_cast<const __half*>(logits),
                  static_cast<int64_t*>(out_index), V);
}

int mcv_argmax_key_to_index(const void* key, void* out_index, int64_t M, mcv_stream_t stream) {
    if (!key || !out_index) return fail(MCV_ERR_NULL, "argmax_key_to_index: null pointer");
    if (M < 1 || M > 32) return fail(MCV_ERR_SHAPE, "argmax_key_to_index: M must be 1..32");
    return key_to_index_impl(key, out_index, M, static_cast<cudaStream_t>(stream));
}


int mcv_lm_head_argmax_w8a8(const void* x, const void* w_int8, const void* w_scale, void* out_key, void* out_index,
                            int64_t M, int64_t K, int64_t N_shard, int64_t n_offset, void* workspace,
                            size_t workspace_bytes, mcv_stream_t stream) {
    if (!out_key && !out_index) return fail(MCV_ERR_NULL, "lm_head_argmax_w8a8: out_key and out_index both null");
    return lm_head_argmax_w8a8_impl(x, w_int8, w_scale, out_key, out_index, M, K, N_shard, n_offset, workspace,
                                    workspace_bytes, static_cast<cudaStream_t>(stream), nullptr);
}

}  // extern "C"
