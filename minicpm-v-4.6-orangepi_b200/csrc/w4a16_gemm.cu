// W4A16 GEMM for batched decode / prefill (M >= 16) on the 5th-generation
// tensor cores: tcgen05.mma with the fp32 accumulator in tensor memory.
//
// Reference counterpart: the reference has no quantized GEMM for M > 1 -
// prefill goes through matmul_b_transposed's dense aclnnMm / K-tiling path
// (src/csrc/lib/ops.cpp:215-322) and matmul_w4a16 is M=1 only (ops.cpp:1048).
// This kernel serves the same mcv-int4 weights as the decode GEMV.
//
// The product is computed transposed, out^T = W x^T: the 128 weight columns
// of a block are the MMA's M dimension and up to 256 rows of x its N
// dimension.  The dequantised weights never touch shared memory: they are
// written straight into tensor memory (tcgen05.st) and the MMA reads its A
// operand from there (tcgen05.mma ... [a_tmem]), so shared-memory bandwidth
// is left to the x tiles the MMA reads as its B operand.  A block has three
// roles that meet only on mbarriers (no block-wide barrier in the k loop):
//  * a producer thread requests, per 64-k stage, the x tile [rows x 64 k]
//    (TMA, 128-byte swizzle; rows past M are zero-filled) and the packed int4
//    tile (8 strips x 512 B, one 2-D TMA) into a 6-deep ring, refilling a
//    slot once the MMAs that read it are done; the weights of the first
//    slots are requested before the PDL wait, x after it;
//  * 512 dequantising threads - thread (warp w, lane l) owns weight column
//    32(w%4)+l of the tile and k 16(w/4)..+15 of the stage - turn their 16
//    nibbles into fp16 (q - zero) * scale and store them to their TMEM lane
//    with one tcgen05.st, then arrive on the stage's "weight ready" mbarrier;
//    scales and zeros sit in registers, fetched 8 groups at a time;
//  * an issuer thread runs four tcgen05.mma.kind::f16 (M=128, N=rows of x
//    rounded to 16, K=16) per stage and commits them to the stage's "done"
//    mbarrier;
//  * the epilogue reads the accumulator (TMEM lane = weight column, column =
//    row of x) with tcgen05.ld and writes fp16.
// When the output tiles leave SMs idle (small M), k is split over the CTAs
// of a thread-block cluster; the leader sums the slices' fp32 partials
// through distributed shared memory, so no global scratch is needed.
// Tensor memory: the accumulator (256 columns) plus a 6-deep ring of A
// operands (32 columns per stage), 512 columns allocated per block.
// Every wait is bounded (2 s); on a timeout the block records an error bit,
// waits (bounded) for its own copies and MMAs, frees its tensor memory and
// returns.  Single-GPU code: no multicast, no peer memory.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "tcgen05.cuh"

namespace mcv {
unsigned take_gemm_device_error();

namespace {

constexpr int kWCols = 128;                 // weight columns per block (MMA M)
constexpr int kXRows = 256;                 // rows of x per block (MMA N, at most)
constexpr int kBK = 64;                     // k per stage: one 128-byte swizzle row of x
constexpr int kStrips = kWCols / 16;        // 16-column strips of the mcv-int4 layout per tile
constexpr int kDqThreads = kWCols * kBK / 16;  // 512: 16 k of one weight column each
constexpr int kDqWarps = kDqThreads / 32;
constexpr int kThreads = kDqThreads + 64;   // + an MMA-issuing warp and a producer warp
constexpr int kXBytes = kXRows * kBK * 2;   // 32 KB x tile per stage (at most)
constexpr int kQBytes = kWCols * kBK / 2;   // 4 KB packed int4 weights per stage
constexpr int kStageBytes = kXBytes + kQBytes;
constexpr int kStages = 6;                  // ring depth
constexpr int kACols = kBK / 2;             // TMEM columns of one stage's A operand (fp16 pairs)
constexpr int kAccCols = kXRows;            // fp32 accumulator columns
constexpr int kTmemCols = 512;              // accumulator + A ring, rounded to a power of two
static_assert(kAccCols + kStages * kACols <= kTmemCols, "tensor memory budget");
constexpr int kSmemBytes = kStages * kStageBytes + 1024 + 256;
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
static_assert(kXRows * kWCols * 4 + 16 <= kStages * kStageBytes, "split-k partials (and the failure word) must fit the ring");

static __device__ unsigned g_gemm_dev_error;

// 8 consecutive 32-bit columns of this thread's TMEM lane (warp-collective).
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
                 "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Lane-uniform select of word (i & 3) of v, without dynamic register indexing.
__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) {
    const uint32_t lo = (i & 1) ? v.y : v.x, hi = (i & 1) ? v.w : v.z;
    return (i & 2) ? hi : lo;
}

// ---- weight dequantisation -----------------------------------------------

// One column's 16 consecutive k from a 16-byte lane vector of the mcv-int4
// layout (include/mcv_matmul.h): word j holds k = kb..kb+3 (kb = 16t + 4j)
// of row g in nibble slots 0,4,2,6 and of row g+8 in slots 1,5,3,7.  `w4`
// is the vector already shifted right by 4 for the row-(g+8) column, so
// both columns read slots 0,4 (k, k+1) and, after >> 8, 2,6 (k+2, k+3).
// Out: 8 fp16 pairs (q - zero) * scale in k order.
__device__ __forceinline__ void dequant_col(const uint4& w4, int zero, __half scale, uint32_t (&o)[8]) {
    constexpr uint32_t kMagic = 0x64006400u;  // fp16 1024: (1024 + q) exact for q < 16
    const __half z1 = __int2half_rn(1024 + zero);
    const __half2 zz = __halves2half2(z1, z1), ss = __halves2half2(scale, scale);
    const uint32_t w[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const __half2 a = __hsub2(u32_as_h2(lop3_and_or(w[j], 0x000f000fu, kMagic)), zz);
        const __half2 b = __hsub2(u32_as_h2(lop3_and_or(w[j] >> 8, 0x000f000fu, kMagic)), zz);
        o[2 * j] = h2_as_u32(__hmul2(a, ss));
        o[2 * j + 1] = h2_as_u32(__hmul2(b, ss));
    }
}

struct GemmArgs {
    const __half* s;
    const uint32_t* z;
    __half* out;
    int M, K, N, zero_bias;
    int x_box_rows;  // rows one x tile copy lands (256, or M rounded up to 16 when smaller)
    int splits;      // K slices = CTAs of a cluster along z (1: no split)
};

__global__ void __launch_bounds__(kThreads, 1)
w4a16_gemm_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap qmap,
                  const GemmArgs a) {
    extern __shared__ unsigned char smem_raw[];
    // 1024-byte alignment for the swizzle atoms
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    auto xt = [&](int b) { return smem + b * kStageBytes; };
    auto qt = [&](int b) { return smem + b * kStageBytes + kXBytes; };
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);  // [kStages] x + packed tile landed
    uint64_t* wready = full + kStages;   // [kStages] A operand in TMEM (kDqThreads arrivals)
    uint64_t* done = wready + kStages;   // [kStages] MMAs of the stage complete (tcgen05.commit)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + kStages);
    volatile int* failed = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * kWCols, m0 = blockIdx.y * kXRows;
    const int K = a.K, G = K / 128, Gp = (G + 7) & ~7, zw = (G + 7) >> 3;
    // this CTA's slice of the k stages: [i0, i0 + nst)
    const int split = blockIdx.z;
    const int i0 = static_cast<int>(static_cast<int64_t>(K / kBK) * split / a.splits);
    const int nst = static_cast<int>(static_cast<int64_t>(K / kBK) * (split + 1) / a.splits) - i0;
    const int rows = a.M - m0 < kXRows ? a.M - m0 : kXRows;  // rows of x in this block
    const int mma_n = (rows + 15) & ~15;                        // MMA N: rows rounded up to 16
    const int x_bytes = a.x_box_rows * kBK * 2;
    constexpr int kIssuerWarp = kDqWarps, kProducerWarp = kDqWarps + 1;

    if (warp == kIssuerWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&wready[i], kDqThreads);
            mbar_init(&done[i], 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        *failed = 0;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tmem_acc = tmem, tmem_a = tmem + kAccCols;
    pdl_trigger();

    if (warp == kProducerWarp) {
        // Stage j's x tile and packed weight tile go into slot j % kStages
        // once the MMAs of stage j - kStages have released it (which also
        // frees the slot's A operand in TMEM).
        if (lane == 0) {
            const int pre = nst < kStages ? nst : kStages;
            for (int j = 0; j < pre; ++j) {  // weights do not depend on the previous kernel
                mbar_expect_tx(&full[j], x_bytes + kQBytes);
                tma_load_2d(qt(j), &qmap, (i0 + j) * (kQBytes / kStrips / 4), n0 / 16, &full[j]);
            }
            pdl_wait();  // x may be the previous kernel's output
            int j = 0;
            for (; j < nst; ++j) {
                const int sj = j % kStages;
                if (j >= kStages) {
                    if (*failed || !mbar_wait(&done[sj], static_cast<uint32_t>((j - kStages) / kStages) & 1u)) {
                        *failed = 1;
                        break;
                    }
                    mbar_expect_tx(&full[sj], x_bytes + kQBytes);
                    tma_load_2d(qt(sj), &qmap, (i0 + j) * (kQBytes / kStrips / 4), n0 / 16, &full[sj]);
                }
                tma_load_2d(xt(sj), &xmap, (i0 + j) * kBK, m0, &full[sj]);
            }
            // Drain (bounded): every slot whose copies were fully requested
            // must land before the block frees its shared memory.
            for (int q = (j > kStages ? j - kStages : 0); q < j; ++q)
                if (!mbar_wait(&full[q % kStages], static_cast<uint32_t>(q / kStages) & 1u)) *failed = 1;
        }
        __syncwarp();
    } else if (warp == kIssuerWarp) {
        // Four MMAs (K = 16 each) per stage once the stage's x tile has
        // landed and its A operand is in TMEM; one commit per stage.
        if (lane == 0) {
            const uint32_t idesc = instr_desc_f16(kWCols, mma_n);
            // descriptor of slot 0; slot b, k-step kk adds (b * kStageBytes + 32 kk) / 16
            // to the start-address field (no carry: shared addresses stay below 256 KB)
            const uint64_t desc0 = smem_desc_sw128(smem_u32(xt(0)));
            int issued = 0, b = 0;
            uint32_t ph = 0;
            for (int i = 0; i < nst; ++i) {
                // "weight ready" implies the slot's x tile has landed: every
                // dequantising thread waited for the slot's full barrier
                // (TMA completion) before arriving
                if (*failed || !mbar_wait(&wready[b], ph)) {
                    *failed = 1;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < kBK / 16; ++kk)
                    mma_f16_ts(tmem_acc, tmem_a + b * kACols + kk * 8,
                               desc0 + static_cast<uint64_t>((b * kStageBytes + kk * 32) >> 4), idesc,
                               (i > 0 || kk > 0) ? 1u : 0u);
                mma_commit(&done[b]);
                issued = i + 1;
                if (++b == kStages) b = 0, ph ^= 1u;
            }
            // the last commit covers every MMA issued before it
            if (issued > 0 &&
                !mbar_wait(&done[(issued - 1) % kStages], static_cast<uint32_t>((issued - 1) / kStages) & 1u))
                *failed = 1;
            if (issued < nst) *failed = 1;
        }
        __syncwarp();
    } else {
        // Dequantising threads.  Warp w writes TMEM lanes 32(w%4)..+31 (the
        // lanes it may access), i.e. weight columns n = 32(w%4) + lane of the
        // tile, and k-chunk c = w/4 (16 k, 8 TMEM columns) of every stage.
        const int quarter = warp & 3, c = warp >> 2;
        const int n = quarter * 32 + lane;             // column within the tile
        const int sl = n >> 4, r = n & 15;             // strip and row within it
        const int vec = sl * 32 + 4 * (r & 7) + c;     // lane vector holding (column, chunk)
        const int shift = (r & 8) ? 4 : 0;             // rows g+8 sit one nibble higher
        const int col = n0 + n;
        const bool have_col = col < ((a.N + 15) & ~15);
        const int nchunks = (G + 7) / 8;
        const uint32_t lane_addr = tmem_a + (static_cast<uint32_t>(quarter * 32) << 16) + c * 8;
        // scales and zeros of this column, 8 groups at a time (one 16-byte
        // scale vector and one zero word), the next chunk loaded early
        auto load_chunk = [&](int ch, uint4& s, uint32_t& z) {
            if (have_col && ch < nchunks) {
                s = __ldg(reinterpret_cast<const uint4*>(a.s + static_cast<size_t>(col) * Gp) + ch);
                z = __ldg(a.z + static_cast<size_t>(col) * zw + ch);
            }
        };
        uint4 s_cur = make_uint4(0, 0, 0, 0), s_nxt = s_cur;
        uint32_t z_cur = 0, z_nxt = 0;
        load_chunk(i0 / 16, s_cur, z_cur);  // 16 stages of 64 k per 8-group chunk
        load_chunk(i0 / 16 + 1, s_nxt, z_nxt);
        for (int i = 0; i < nst; ++i) {
            const int b = i % kStages;
            const int grp = ((i0 + i) * kBK) / 128, gi = grp & 7;
            if (i > 0 && ((i0 + i) & 15) == 0) {  // first stage of a new 8-group chunk
                s_cur = s_nxt, z_cur = z_nxt;
                load_chunk(grp / 8 + 1, s_nxt, z_nxt);
            }
            // a landed slot implies its previous MMAs are done (the producer
            // waited for them), so the A ring slot is free too; the warp
            // leaves together, since tcgen05.st is warp-collective
            const bool ok = !*failed && mbar_wait(&full[b], static_cast<uint32_t>(i / kStages) & 1u);
            if (!__all_sync(0xffffffffu, ok)) {
                *failed = 1;
                break;
            }
            uint4 v = *reinterpret_cast<const uint4*>(qt(b) + vec * 16);
            v.x >>= shift, v.y >>= shift, v.z >>= shift, v.w >>= shift;
            const __half sc = __ushort_as_half(static_cast<unsigned short>(word_of(s_cur, gi >> 1) >> (16 * (gi & 1))));
            const int zero = static_cast<int>((z_cur >> (4 * gi)) & 0xfu) + a.zero_bias;
            uint32_t o[8];
            dequant_col(v, zero, sc, o);
            if (!have_col) {
#pragma unroll
                for (int e = 0; e < 8; ++e) o[e] = 0u;
            }
            tmem_st8(lane_addr + b * kACols, o);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tc_fence_before();
            mbar_arrive(&wready[b]);
        }
    }
    if (warp != kProducerWarp) pdl_wait();  // every thread passes the wait before exit
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const bool acc_ready = !*failed;
    if (!acc_ready && tid == 0) atomicOr(&g_gemm_dev_error, kDevErrTimeout);
    const int quarter = warp & 3;
    const uint32_t acc_lanes = tmem_acc + (static_cast<uint32_t>(quarter * 32) << 16);
    if (a.splits == 1) {
        // warp w reads TMEM lanes 32(w%4).. (weight columns) over columns
        // 16 j.. (rows of x) for j = w/4, w/4 + 4, ...; the issuer waited
        // for the last commit
        // fp16 outputs through a shared-memory tile (the ring is idle now:
        // every copy landed and every MMA completed), then 16-byte stores
        // of 8 columns: an eighth of the store instructions of writing each
        // thread's column directly (M = 1024, N = 4096: 12.1 vs 12.7 us)
        __half* tile = reinterpret_cast<__half*>(smem);  // [rows][kWCols]
        if (warp < kDqWarps) {
            if (acc_ready) {
#pragma unroll 1
                for (int j = warp >> 2; j * 16 < mma_n; j += kDqWarps / 4) {
                    float v[16];
                    tmem_ld16(acc_lanes + j * 16, v);
#pragma unroll
                    for (int e = 0; e < 16; ++e) tile[(j * 16 + e) * kWCols + quarter * 32 + lane] = __float2half_rn(v[e]);
                }
            }
            asm volatile("bar.sync 1, %0;" ::"r"(kDqThreads) : "memory");  // the dequantising warps only
            if (acc_ready) {
                const bool vec_ok = (a.N & 7) == 0 && (reinterpret_cast<uintptr_t>(a.out) & 15u) == 0;
                for (int idx = tid; idx < rows * (kWCols / 8); idx += kDqThreads) {
                    const int r = idx / (kWCols / 8), c8 = (idx % (kWCols / 8)) * 8, col = n0 + c8;
                    const __half* src = tile + r * kWCols + c8;
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
        // Split k: every CTA of the cluster parks its fp32 partial sums in
        // its own (now idle) ring memory as red[m][n]; after a cluster
        // barrier each CTA adds all slices' partials of its share of the
        // rows through distributed shared memory and writes fp16; a second
        // barrier keeps every CTA's memory alive until all are done.  Every
        // CTA reaches both barriers.
        float* red = reinterpret_cast<float*>(smem);
        int* red_failed = reinterpret_cast<int*>(smem + kStages * kStageBytes - 16);
        if (warp < kDqWarps) {
#pragma unroll 1
            for (int j = warp >> 2; j * 16 < mma_n; j += kDqWarps / 4) {
                float v[16];
                tmem_ld16(acc_lanes + j * 16, v);
#pragma unroll
                for (int e = 0; e < 16; ++e) red[(j * 16 + e) * kWCols + quarter * 32 + lane] = v[e];
            }
        }
        if (tid == 0) *red_failed = acc_ready ? 0 : 1;
        cluster_sync();
        // CTA `split` finishes rows m = split, split + S, ...: 32 threads per
        // row, 4 columns each; the slices' partials are all loaded before
        // they are added, in rank order (the same sum whichever CTA does it)
        int any_failed = 0;
        for (int r = 0; r < a.splits; ++r) any_failed |= ld_cluster_s32(cluster_smem_addr(red_failed, r));
        if (!any_failed && tid < kDqThreads) {
            const int n = 4 * (tid & 31), col = n0 + n;
            const bool vec_ok = (a.N & 3) == 0 && (reinterpret_cast<uintptr_t>(a.out) & 7u) == 0;
#pragma unroll 1
            for (int m = split + a.splits * (tid >> 5); m < rows; m += a.splits * (kDqThreads / 32)) {
                float4 part[8];
#pragma unroll
                for (int r = 0; r < 8; ++r)
                    if (r < a.splits) part[r] = ld_cluster_f32x4(cluster_smem_addr(red + m * kWCols + n, r));
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
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

}  // namespace

unsigned take_gemm_device_error() {
    unsigned v = 0;
    if (cudaMemcpyFromSymbol(&v, g_gemm_dev_error, sizeof(v)) != cudaSuccess) return ~0u;
    if (v) {
        const unsigned zero = 0;
        cudaMemcpyToSymbol(g_gemm_dev_error, &zero, sizeof(zero));
    }
    return v;
}

}  // namespace mcv

using namespace mcv;

extern "C" {

int mcv_w4a16_gemm(const void* x, const void* qweight, const void* scales, const void* zeros, int zero_bias,
                   void* out, int64_t M, int64_t K, int64_t N, int64_t group, mcv_stream_t stream) {
    if (!x || !qweight || !scales || !zeros || !out) return fail(MCV_ERR_NULL, "w4a16_gemm: null pointer");
    if (group != 128) return fail(MCV_ERR_SHAPE, "w4a16_gemm: group size must be 128");
    if (M < 1 || K < 128 || N < 1 || K % 128 != 0 || M > (1 << 24) || K > (1 << 16) || N > (1 << 24))
        return fail(MCV_ERR_SHAPE, "w4a16_gemm: need M >= 1, K a multiple of 128 (<= 65536), N >= 1");
    if (!aligned16(x) || !aligned16(qweight)) return fail(MCV_ERR_ALIGN, "w4a16_gemm: x and qweight must be 16-byte aligned");
    if ((reinterpret_cast<uintptr_t>(scales) & 15u) || (reinterpret_cast<uintptr_t>(zeros) & 3u) ||
        (reinterpret_cast<uintptr_t>(out) & 1u))
        return fail(MCV_ERR_ALIGN, "w4a16_gemm: scales must be 16-byte, zeros 4-byte and out 2-byte aligned");
    if (zero_bias < 0 || zero_bias > 1) return fail(MCV_ERR_VALUE, "w4a16_gemm: zero_bias must be 0 or 1");
    auto enc = encode_fn();
    if (!enc) return fail(MCV_ERR_CUDA, "w4a16_gemm: cuTensorMapEncodeTiled unavailable");
    // Split k over a cluster when the output tiles leave SMs idle: double
    // the slices while they still fit the SMs and keep >= 4 stages each
    // (MCV_TUNE_GEMM_SPLIT_K 1..8 overrides, limited by the stage count).
    const int64_t tiles_n = (N + kWCols - 1) / kWCols, tiles_m = (M + kXRows - 1) / kXRows;
    const int nst_all = static_cast<int>(K / kBK);
    int split_k = 1;
    const int forced = tuning(MCV_TUNE_GEMM_SPLIT_K);
    if (forced >= 1 && forced <= 8) {
        split_k = forced < nst_all ? forced : nst_all;
    } else {
        while (split_k < 8 && tiles_n * tiles_m * split_k * 2 <= sm_count() && nst_all / (split_k * 2) >= 4)
            split_k *= 2;
    }
    if (tiles_m > 65535) return fail(MCV_ERR_SHAPE, "w4a16_gemm: M too large");
    // x tile box: 256 rows, or M rounded up to 16 when smaller (rows of the
    // shared-memory tile past the box keep stale values; they only feed
    // accumulator columns >= M, which are never stored)
    const int box_rows = M >= kXRows ? kXRows : static_cast<int>((M + 15) & ~int64_t(15));
    CUtensorMap map, qmap;
    {
        const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(M)};
        const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
        const cuuint32_t box[2] = {kBK, static_cast<cuuint32_t>(box_rows)};
        const cuuint32_t estr[2] = {1, 1};
        CUresult r = enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(x), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return fail(MCV_ERR_CUDA, "w4a16_gemm: cuTensorMapEncodeTiled(x) failed");
    }
    {
        // packed weights as [strips][K/64 * 128] uint32: one 512-byte row
        // segment per strip and 64-k stage
        const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K) * 2, static_cast<cuuint64_t>((N + 15) / 16)};
        const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 8};
        const cuuint32_t box[2] = {kQBytes / kStrips / 4, kStrips};
        const cuuint32_t estr[2] = {1, 1};
        CUresult r = enc(&qmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(qweight), dims, strides, box,
                         estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return fail(MCV_ERR_CUDA, "w4a16_gemm: cuTensorMapEncodeTiled(qweight) failed");
    }
    cudaError_t e = cudaFuncSetAttribute(w4a16_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(w4a16_gemm)");
    GemmArgs ga{static_cast<const __half*>(scales), static_cast<const uint32_t*>(zeros), static_cast<__half*>(out),
                static_cast<int>(M), static_cast<int>(K), static_cast<int>(N), zero_bias, box_rows, split_k};
    return launch_clustered(w4a16_gemm_kernel, dim3(static_cast<unsigned>(tiles_n), static_cast<unsigned>(tiles_m), split_k),
                            dim3(kThreads), dim3(1, 1, split_k), kSmemBytes, static_cast<cudaStream_t>(stream), map,
                            qmap, ga);
}

}  // extern "C"
