// W4A16 GEMV for decode (M = 1..8, batched up to 64) over the mcv-int4 weight layout, plus the
// load-time host repackers from GPTQ / AWQ / the reference's tile layout.
//
// Reference behaviour replaced: matmul_w4a16 (src/csrc/lib/ops.cpp:1030-1095)
// and its AscendC kernel op_kernel/matmul_w4a16_custom.cpp:64-127, which
// computes out[n] = sum_g s[g,n] * sum_{k in g} x[k] * (q-z)[k,n] (group 128)
// on 8 AICore blocks with fp16 accumulation.  Here every group's partial sum
// is accumulated in fp32 and scaled in fp32.
//
// Design (HBM-bound: a 1024x3584 weight is 1.84 MB of int4):
//  * Layout.  Output columns form strips of 16.  A strip's weights are stored
//    k-block (16 k) after k-block, four k-blocks per 16-byte lane vector, and
//    lane l's 32-bit word of a k-block holds exactly the eight 4-bit values it
//    feeds to one m16n8k16 tensor-core MMA as its A fragment (rows = the 16
//    columns of the strip).  So one coalesced 16-byte load per lane brings the
//    fragments of four MMAs, and a warp-wide load reads 512 contiguous bytes.
//  * Work.  Three schedules (MCV_TUNE_W4A16_MODE picks one explicitly):
//    - K-split (default for a launch with few strips, i.e. one decode GEMV):
//      one block per strip, its 8 or 16 warps take the strip's 128-k groups
//      and meet in shared memory - one load latency on the critical path;
//    - bulk-copy streaming (default for large launches): a persistent grid,
//      each warp owns whole strips and walks them in 512-k chunks that land
//      in a warp-private 2-deep cp.async.bulk ring while the previous chunk
//      is computed (3 blocks of 8 warps per SM);
//    - register streaming: the same walk with the next chunk's eight 16-byte
//      loads per lane held in registers (2 blocks per SM).
//    Weights are requested before griddepcontrol.wait in all three, so under
//    programmatic dependent launch the weight stream overlaps the previous
//    kernel.
//  * Math.  int4 -> fp16 by the exponent-bias ("magic number") conversion
//    described for FasterTransformer-style mixed-input GEMMs (Kim et al.,
//    "Who Says Elephants Can't Run", 2022; Frantar et al., MARLIN, 2024):
//    OR-ing a nibble into the mantissa of fp16 1024.0 gives 1024+q exactly,
//    and one HSUB2/HFMA2 leaves (q - zero) exactly.  mma.sync m16n8k16 with
//    fp32 accumulation multiplies them by x (B operand, up to 8 rows); each
//    128-k group gets fresh accumulators that are scaled in fp32 and added to
//    the running sums.  The MMA is used here to keep the ALU instruction
//    count per weight low (~1.3) in an HBM-bound kernel, not for its FLOPs.
#include <algorithm>
#include <cstring>
#include <vector>

#include "common.cuh"
#include "neighbours.cuh"

namespace mcv {
namespace {

constexpr int kGroup = 128;        // quantization group along K (the reference's only size)
constexpr int kChunkK = 512;       // k per register buffer (8 lane vectors, 4 groups)
constexpr int kWarps = 8;
constexpr int kBlocksPerSm = 2;
constexpr int kMaxGroupProblems = 48;
constexpr int kMaxGemvRows = 64;  // rows of x on the GEMV schedules (M > 8: up to 8 MMAs per fragment)

__host__ __device__ inline int64_t padded_n(int64_t N) { return (N + 15) / 16 * 16; }
__host__ __device__ inline int64_t padded_g(int64_t G) { return (G + 7) / 8 * 8; }

// An MMA's dot product does not depend on the order of k, so k is permuted
// inside every 64-k quad, identically for weights and activations: lane
// (g = lane/4, t = lane%4) owns physical k = 16t .. 16t+15 of the quad, and
// k-block j of the quad uses its k = 16t + 4j .. 16t + 4j + 3.  Fragment
// element e of the lane's A word for k-block j is then
// (row, k) = (g, +0), (g, +1), (g+8, +0), (g+8, +1), (g, +2), (g, +3),
// (g+8, +2), (g+8, +3) relative to 16t + 4j, and the B fragment is x at the
// same four k - one 16-byte load of x covers two k-blocks.  Nibble slots are
// chosen so that LOP3 with 0x000F000F / 0x00F000F0 on the word and on
// word >> 8 yields the four half2 registers a0..a3 in order.
constexpr int kFragSlot[8] = {0, 4, 1, 5, 2, 6, 3, 7};
constexpr int kFragRow[8] = {0, 0, 8, 8, 0, 0, 8, 8};
constexpr int kFragK[8] = {0, 1, 0, 1, 2, 3, 2, 3};

__device__ __forceinline__ void mma_16816(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// fp16 bit patterns of the zero-point constants, built with integer ops
// (no int -> fp16 conversion): 1024 + z (z < 1024) is 0x6400 | z, and
// -(64 + z) for z < 64 is 0xD400 | (z << 4) (exponent 6, mantissa 16 z).
__device__ __forceinline__ uint32_t h2_bits_1024_plus(int z) { return (0x6400u | static_cast<uint32_t>(z)) * 0x10001u; }
__device__ __forceinline__ uint32_t h2_bits_neg_64_plus(int z) {
    return (0xD400u | (static_cast<uint32_t>(z) << 4)) * 0x10001u;
}

template <int M, int MATH>
__device__ __forceinline__ void group_mma(const uint4 (&v)[2], const __half* xg, int g, int zl_q, int zh_q,
                                          float d[4]);

// One 128-k group for one lane: v[0], v[1] are the lane's weight vectors of
// the group's two quads, xg points at x[row g][group start + 16t] (read only
// when g < M).  Dequantises and runs 8 MMAs on four independent accumulator
// chains; returns the group's fp32 sums for rows g, g+8 x columns 2t, 2t+1.
template <int M>
__device__ __forceinline__ void group_mma(const uint4 (&v)[2], const __half* xg, int g, int zl_q, int zh_q,
                                          float d[4]) {
    group_mma<M, 0>(v, xg, g, zl_q, zh_q, d);
}

template <int M, int MATH>
__device__ __forceinline__ void group_mma(const uint4 (&v)[2], const __half* xg, int g, int zl_q, int zh_q,
                                          float d[4]) {
  if constexpr (MATH == 1 || MATH == 2) {
    uint4 xv[2][2];
#pragma unroll
    for (int qd = 0; qd < 2; ++qd) {
        xv[qd][0] = xv[qd][1] = make_uint4(0, 0, 0, 0);
        if (g < M) {
            xv[qd][0] = *reinterpret_cast<const uint4*>(xg + qd * 64);
            xv[qd][1] = *reinterpret_cast<const uint4*>(xg + qd * 64 + 8);
        }
    }
    constexpr uint32_t kMagic = 0x64006400u;
    float c[2][4] = {};
    float ones_acc[4] = {};
    if constexpr (MATH == 1) {
        // exact (q - zero) in fp16 per weight, two accumulator chains
        const __half2 zl = u32_as_h2(h2_bits_1024_plus(zl_q)), zh = u32_as_h2(h2_bits_neg_64_plus(zh_q));
        const __half2 inv16 = u32_as_h2(0x2c002c00u);
#pragma unroll
        for (int kb = 0; kb < 8; ++kb) {
            const int qd = kb >> 2, j = kb & 3;
            const uint4 vv = v[qd];
            const uint32_t w = j == 0 ? vv.x : j == 1 ? vv.y : j == 2 ? vv.z : vv.w;
            const uint4 xx = xv[qd][j >> 1];
            const uint32_t b0 = (j & 1) ? xx.z : xx.x;
            const uint32_t b1 = (j & 1) ? xx.w : xx.y;
            const uint32_t w8 = w >> 8;
            uint32_t a[4];
            a[0] = h2_as_u32(__hsub2(u32_as_h2(lop3_and_or(w, 0x000f000fu, kMagic)), zl));
            a[1] = h2_as_u32(__hfma2(u32_as_h2(lop3_and_or(w, 0x00f000f0u, kMagic)), inv16, zh));
            a[2] = h2_as_u32(__hsub2(u32_as_h2(lop3_and_or(w8, 0x000f000fu, kMagic)), zl));
            a[3] = h2_as_u32(__hfma2(u32_as_h2(lop3_and_or(w8, 0x00f000f0u, kMagic)), inv16, zh));
            mma_16816(c[kb & 1], a, b0, b1);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) d[i] = c[0][i] + c[1][i];
    } else {
        // Zero point folded out of the per-weight work: the MMAs take the raw
        // exponent-bias values (1024 + q for rows g, 1024 + 16 q for rows g+8,
        // both exact in fp16) and a second MMA chain with an all-ones A
        // operand gives S = sum(x) over the group in every row; then
        //   sum x (q - z) = D_lo - (1024 + z) S = D_hi / 16 - (64 + z) S.
        // Four instructions per 8 weights instead of eight.
        const uint32_t ones[4] = {0x3c003c00u, 0x3c003c00u, 0x3c003c00u, 0x3c003c00u};
#pragma unroll
        for (int kb = 0; kb < 8; ++kb) {
            const int qd = kb >> 2, j = kb & 3;
            const uint4 vv = v[qd];
            const uint32_t w = j == 0 ? vv.x : j == 1 ? vv.y : j == 2 ? vv.z : vv.w;
            const uint4 xx = xv[qd][j >> 1];
            const uint32_t b0 = (j & 1) ? xx.z : xx.x;
            const uint32_t b1 = (j & 1) ? xx.w : xx.y;
            const uint32_t w8 = w >> 8;
            uint32_t a[4];
            a[0] = lop3_and_or(w, 0x000f000fu, kMagic);
            a[1] = lop3_and_or(w, 0x00f000f0u, kMagic);
            a[2] = lop3_and_or(w8, 0x000f000fu, kMagic);
            a[3] = lop3_and_or(w8, 0x00f000f0u, kMagic);
            mma_16816(c[kb & 1], a, b0, b1);
            mma_16816(ones_acc, ones, b0, b1);
        }
        const float S0 = ones_acc[0], S1 = ones_acc[1];  // columns 2t, 2t+1 (every row holds them)
        const float zl = -static_cast<float>(1024 + zl_q), zh = -static_cast<float>(64 + zh_q);
        d[0] = fmaf(zl, S0, c[0][0] + c[1][0]);
        d[1] = fmaf(zl, S1, c[0][1] + c[1][1]);
        d[2] = fmaf(c[0][2] + c[1][2], 0.0625f, zh * S0);
        d[3] = fmaf(c[0][3] + c[1][3], 0.0625f, zh * S1);
    }
  } else {
    uint4 xv[2][2];
#pragma unroll
    for (int qd = 0; qd < 2; ++qd) {
        xv[qd][0] = xv[qd][1] = make_uint4(0, 0, 0, 0);
        if (g < M) {
            xv[qd][0] = *reinterpret_cast<const uint4*>(xg + qd * 64);
            xv[qd][1] = *reinterpret_cast<const uint4*>(xg + qd * 64 + 8);
        }
    }
    const __half z1 = __int2half_rn(1024 + zl_q);   // rows g: 1024 + zero
    const __half z2 = __int2half_rn(-(64 + zh_q));  // rows g+8: -(64 + zero)
    const __half2 zl = __halves2half2(z1, z1), zh = __halves2half2(z2, z2);
    const __half2 inv16 = __halves2half2(__ushort_as_half(0x2c00), __ushort_as_half(0x2c00));
    float c[4][4] = {};
#pragma unroll
    for (int kb = 0; kb < 8; ++kb) {
        const int qd = kb >> 2, j = kb & 3;
        const uint4 vv = v[qd];
        const uint32_t w = j == 0 ? vv.x : j == 1 ? vv.y : j == 2 ? vv.z : vv.w;
        const uint4 xx = xv[qd][j >> 1];
        const uint32_t b0 = (j & 1) ? xx.z : xx.x;
        const uint32_t b1 = (j & 1) ? xx.w : xx.y;
        const uint32_t w8 = w >> 8;
        constexpr uint32_t kMagic = 0x64006400u;
        uint32_t a[4];
        a[0] = h2_as_u32(__hsub2(u32_as_h2(lop3_and_or(w, 0x000f000fu, kMagic)), zl));
        a[1] = h2_as_u32(__hfma2(u32_as_h2(lop3_and_or(w, 0x00f000f0u, kMagic)), inv16, zh));
        a[2] = h2_as_u32(__hsub2(u32_as_h2(lop3_and_or(w8, 0x000f000fu, kMagic)), zl));
        a[3] = h2_as_u32(__hfma2(u32_as_h2(lop3_and_or(w8, 0x00f000f0u, kMagic)), inv16, zh));
        mma_16816(c[kb & 3], a, b0, b1);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) d[i] = (c[0][i] + c[1][i]) + (c[2][i] + c[3][i]);
  }
}

struct Problem {
    const __half* x;
    const uint4* qw;
    const __half* s;   // [Npad][Gpad8]
    const uint32_t* z; // [Npad][ceil(G/8)]
    __half* out;
    int K, N, zero_bias;
    int strip_begin;   // first global strip index of this problem
};

struct GroupParams {
    int count;
    int total_strips;
    Problem p[kMaxGroupProblems];
};


// The problem owning a global strip: a binary search over the problems'
// first strips (at most 6 steps for 48 problems; a persistent warp's next
// strip is ~W strips on, often many problems away).
__device__ __forceinline__ int find_problem(const GroupParams& gp, int strip, int start) {
    int lo = start, hi = gp.count - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (gp.p[mid].strip_begin <= strip) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

// Register buffer of one (strip, 512-k chunk): eight lane vectors (32
// k-blocks), the scales of the chunk's 4 groups for the lane's two columns
// (rows g and g+8 of the MMA) and their zero nibbles.
struct Chunk {
    uint4 w[8];
    uint2 slo, shi;
    uint32_t zlo, zhi;
};

__device__ __forceinline__ void load_chunk(Chunk& b, const Problem& P, int sl, int c, int lane) {
    const int K = P.K, G = K / kGroup, Gp = (G + 7) & ~7, zw = (G + 7) >> 3;
    const int nq = min(8, (K - c * kChunkK) / 64);  // lane vectors in this chunk
    const size_t base = (static_cast<size_t>(sl) * (K / 64) + c * 8) * 32 + lane;
#pragma unroll
    for (int q = 0; q < 8; ++q) b.w[q] = q < nq ? ld_stream(P.qw + base + q * 32) : make_uint4(0, 0, 0, 0);
    const int col = sl * 16 + (lane >> 2);
    b.slo = *reinterpret_cast<const uint2*>(P.s + static_cast<size_t>(col) * Gp + c * 4);
    b.shi = *reinterpret_cast<const uint2*>(P.s + static_cast<size_t>(col + 8) * Gp + c * 4);
    const int sh = 16 * (c & 1);
    b.zlo = P.z[static_cast<size_t>(col) * zw + (c >> 1)] >> sh;
    b.zhi = P.z[static_cast<size_t>(col + 8) * zw + (c >> 1)] >> sh;
}

__device__ __forceinline__ float half_of(uint2 v, int i) {
    const uint32_t w = (i < 2) ? v.x : v.y;
    return __half2float(__ushort_as_half(static_cast<unsigned short>(w >> (16 * (i & 1)))));
}

// Computes one chunk into acc (rows g / g+8, columns 2t / 2t+1 of the MMA
// output tile = output columns n0+g, n0+g+8 of activation rows 2t, 2t+1).
template <int M>
__device__ __forceinline__ void compute_chunk(const Chunk& b, const Problem& P, int c, int lane, float acc[4]) {
    const int K = P.K;
    const int nq = min(8, (K - c * kChunkK) / 64);
    const int g = lane >> 2, t = lane & 3;
    const __half* xrow = P.x + static_cast<size_t>(g) * K + c * kChunkK + 16 * t;
#pragma unroll
    for (int gi = 0; gi < 4; ++gi) {
        if (2 * gi >= nq) break;
        const uint4 v[2] = {b.w[2 * gi], b.w[2 * gi + 1]};
        float d[4];
        group_mma<M>(v, xrow + gi * kGroup, g, static_cast<int>((b.zlo >> (4 * gi)) & 0xfu) + P.zero_bias,
                     static_cast<int>((b.zhi >> (4 * gi)) & 0xfu) + P.zero_bias, d);
        const float s_lo = half_of(b.slo, gi), s_hi = half_of(b.shi, gi);
        acc[0] = fmaf(d[0], s_lo, acc[0]);
        acc[1] = fmaf(d[1], s_lo, acc[1]);
        acc[2] = fmaf(d[2], s_hi, acc[2]);
        acc[3] = fmaf(d[3], s_hi, acc[3]);
    }
}

template <int M>
__device__ __forceinline__ void store_strip(const Problem& P, int sl, int lane, const float acc[4]) {
    const int g = lane >> 2, t = lane & 3;
    const int n0 = sl * 16;
    const size_t N = static_cast<size_t>(P.N);
    const int m0 = 2 * t;
    if (m0 < M) {
        if (n0 + g < P.N) P.out[m0 * N + n0 + g] = __float2half_rn(acc[0]);
        if (n0 + g + 8 < P.N) P.out[m0 * N + n0 + g + 8] = __float2half_rn(acc[2]);
    }
    if (m0 + 1 < M) {
        if (n0 + g < P.N) P.out[(m0 + 1) * N + n0 + g] = __float2half_rn(acc[1]);
        if (n0 + g + 8 < P.N) P.out[(m0 + 1) * N + n0 + g + 8] = __float2half_rn(acc[3]);
    }
}

// Warp w of block b is global warp (w * gridDim.x + b), so consecutive strips
// land on different SMs first; it owns strips gw, gw + W, gw + 2W, ...
template <int M>
__global__ void __launch_bounds__(kWarps * 32, kBlocksPerSm)
w4a16_gemv_kernel(const __grid_constant__ GroupParams gp) {
    const int lane = threadIdx.x & 31;
    const int W = static_cast<int>(gridDim.x) * kWarps;
    int strip = (threadIdx.x >> 5) * static_cast<int>(gridDim.x) + static_cast<int>(blockIdx.x);
    const int T = gp.total_strips;
    Chunk A, B;  // two named buffers: a dynamically indexed pair would live in local memory
    int pi = 0, c = 0;
    if (strip < T) {
        pi = find_problem(gp, strip, 0);
        load_chunk(A, gp.p[pi], strip - gp.p[pi].strip_begin, 0, lane);
    }
    pdl_trigger();
    pdl_wait();  // x may be the previous kernel's output
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    // one step: prefetch the (strip, chunk) after the current one into nb,
    // compute the current one from cb
    auto step = [&](Chunk& cb, Chunk& nb) {
        const Problem& P = gp.p[pi];
        const int nchunks = (P.K + kChunkK - 1) / kChunkK;
        int ns = strip, nc = c + 1, npi = pi;
        if (nc == nchunks) {
            ns = strip + W;
            nc = 0;
        }
        if (ns < T) {
            npi = find_problem(gp, ns, pi);
            load_chunk(nb, gp.p[npi], ns - gp.p[npi].strip_begin, nc, lane);
        }
        compute_chunk<M>(cb, P, c, lane, acc);
        if (nc == 0) {
            store_strip<M>(P, strip - P.strip_begin, lane, acc);
            acc[0] = acc[1] = acc[2] = acc[3] = 0.0f;
        }
        strip = ns;
        c = nc;
        pi = npi;
    };
#pragma unroll 1
    while (strip < T) {
        step(A, B);
        if (strip >= T) break;
        step(B, A);
    }
}

// ---------------------------------------------------------------------------
// Streaming variant with warp-private bulk-copy rings.  Each warp owns whole
// strips as above, but its (strip, 512-k chunk) items arrive in shared
// memory: lane 0 moves the chunk's weights (one contiguous <= 4 KB range)
// with cp.async.bulk, lanes copy the chunk's scales (8 bytes per column) and
// zero words with cp.async, and the stage's mbarrier completes when all of it
// has landed.  Each warp keeps kRing items in flight (128 KB per SM) without
// spending registers on them, and needs no synchronisation with other warps.
// The first kRing items are requested before griddepcontrol.wait.
// ---------------------------------------------------------------------------
#ifndef MCV_W4A16_RING
#define MCV_W4A16_RING 2
#endif
constexpr int kRing = MCV_W4A16_RING;
#ifndef MCV_W4A16_TMA_BPS
#define MCV_W4A16_TMA_BPS 3
#endif
constexpr int kTmaBlocksPerSm = MCV_W4A16_TMA_BPS;
constexpr int kStageW = 4096;                      // 8 lane vectors x 32 lanes
constexpr int kStageBytes = kStageW + 16 * 8 + 16 * 4 + 64;  // + scales + zeros, 4352
constexpr int kTmaSmem = kWarps * kRing * kStageBytes + kWarps * kRing * 8;

static __device__ unsigned g_w4a16_dev_error;

// A warp's walk over (strip, 512-k chunk) items: strips strided by the grid's
// warp count (measured faster than one contiguous strip range per warp,
// 0.50 vs 0.55 us per grouped GEMV), each strip's chunks in order; the chunk
// count of the current problem rides along.
struct ItemIter {
    int strip, c, pi, nchunks;
};

__device__ __forceinline__ int chunks_of(const GroupParams& gp, int pi) { return (gp.p[pi].K + kChunkK - 1) / kChunkK; }

__device__ __forceinline__ void next_item(const GroupParams& gp, ItemIter& it, int W) {
    if (++it.c == it.nchunks) {
        it.c = 0;
        it.strip += W;
        if (it.strip < gp.total_strips) {
            it.pi = find_problem(gp, it.strip, it.pi);
            it.nchunks = chunks_of(gp, it.pi);
        }
    }
}

// Requests item `it` into stage `st` (whole warp participates).
__device__ __forceinline__ void issue_item(const GroupParams& gp, const ItemIter& it, unsigned char* st,
                                           uint64_t* bar, int lane) {
    const Problem& P = gp.p[it.pi];
    const int K = P.K, G = K / kGroup, Gp = (G + 7) & ~7, zw = (G + 7) >> 3;
    const int sl = it.strip - P.strip_begin;
    const int nq = min(8, (K - it.c * kChunkK) / 64);
    if (lane == 0) {
        const uint32_t bytes = static_cast<uint32_t>(nq) * 32u * 16u;
        mbar_expect_tx(bar, bytes);
        bulk_load(st, P.qw + (static_cast<size_t>(sl) * (K / 64) + it.c * 8) * 32, bytes, bar);
    }
    const int col = sl * 16 + (lane & 15);
    if (lane < 16) cp_async8(st + kStageW + lane * 8, P.s + static_cast<size_t>(col) * Gp + it.c * 4);
    else cp_async4(st + kStageW + 128 + (lane - 16) * 4, P.z + static_cast<size_t>(col) * zw + (it.c >> 1));
    cp_async_mbar_arrive(bar);
}

template <int M, int MATH>
__global__ void __launch_bounds__(kWarps * 32, kTmaBlocksPerSm)
w4a16_tma_kernel(const __grid_constant__ GroupParams gp) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    unsigned char* ring = smem + warp * kRing * kStageBytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kWarps * kRing * kStageBytes) + warp * kRing;
    const int W = static_cast<int>(gridDim.x) * kWarps;
    const int T = gp.total_strips;
    ItemIter cur{warp * static_cast<int>(gridDim.x) + static_cast<int>(blockIdx.x), 0, 0, 1};
    if (cur.strip < T) {
        cur.pi = find_problem(gp, cur.strip, 0);
        cur.nchunks = chunks_of(gp, cur.pi);
    }
    if (lane == 0)
        for (int s = 0; s < kRing; ++s) mbar_init(&bars[s], 1 + 32);  // bulk arrival + 32 cp.async lanes
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncwarp();
    ItemIter iss = cur;
    int issued = 0;
    for (; issued < kRing && iss.strip < T; ++issued) {
        issue_item(gp, iss, ring + issued * kStageBytes, &bars[issued], lane);
        next_item(gp, iss, W);
    }
    pdl_trigger();
    pdl_wait();  // x may be the previous kernel's output
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 1
    for (int k = 0; cur.strip < T; ++k) {
        const int s = k % kRing;
        if (!mbar_wait(&bars[s], static_cast<uint32_t>(k / kRing) & 1u)) {
            if (lane == 0) atomicOr(&g_w4a16_dev_error, kDevErrTimeout);
            // let this warp's other copies in flight land (each wait bounded)
            // before the block can leave and its shared memory be reused
            for (int it = k + 1; it < issued; ++it)
                (void)mbar_wait(&bars[it % kRing], static_cast<uint32_t>(it / kRing) & 1u);
            return;
        }
        const Problem& P = gp.p[cur.pi];
        const int K = P.K;
        const int nq = min(8, (K - cur.c * kChunkK) / 64);
        const unsigned char* st = ring + s * kStageBytes;
        const uint2 slo = *reinterpret_cast<const uint2*>(st + kStageW + g * 8);
        const uint2 shi = *reinterpret_cast<const uint2*>(st + kStageW + (g + 8) * 8);
        const int sh = 16 * (cur.c & 1);
        const uint32_t zlo = *reinterpret_cast<const uint32_t*>(st + kStageW + 128 + g * 4) >> sh;
        const uint32_t zhi = *reinterpret_cast<const uint32_t*>(st + kStageW + 128 + (g + 8) * 4) >> sh;
        const __half* xrow = P.x + static_cast<size_t>(g) * K + cur.c * kChunkK + 16 * t;
#pragma unroll
        for (int gi = 0; gi < 4; ++gi) {
            if (2 * gi >= nq) break;
            const uint4 v[2] = {*reinterpret_cast<const uint4*>(st + (2 * gi * 32 + lane) * 16),
                                *reinterpret_cast<const uint4*>(st + ((2 * gi + 1) * 32 + lane) * 16)};
            float d[4];
            group_mma<M, MATH>(v, xrow + gi * kGroup, g, static_cast<int>((zlo >> (4 * gi)) & 0xfu) + P.zero_bias,
                         static_cast<int>((zhi >> (4 * gi)) & 0xfu) + P.zero_bias, d);
            const float s_lo = half_of(slo, gi), s_hi = half_of(shi, gi);
            acc[0] = fmaf(d[0], s_lo, acc[0]);
            acc[1] = fmaf(d[1], s_lo, acc[1]);
            acc[2] = fmaf(d[2], s_hi, acc[2]);
            acc[3] = fmaf(d[3], s_hi, acc[3]);
        }
        if (cur.c + 1 == cur.nchunks) {
            store_strip<M>(P, cur.strip - P.strip_begin, lane, acc);
            acc[0] = acc[1] = acc[2] = acc[3] = 0.0f;
        }
        // refill this stage with the item kRing ahead
        fence_proxy_async_smem();
        __syncwarp();
        if (iss.strip < T) {
            issue_item(gp, iss, ring + s * kStageBytes, &bars[s], lane);
            next_item(gp, iss, W);
            ++issued;
        }
        next_item(gp, cur, W);
    }
}

// ---------------------------------------------------------------------------
// K-split variant for launches with few strips (a single decode GEMV): one
// block per strip, its W warps (8, or 16 above 1024 k) take the strip's 128-k
// groups round-robin (at most KG each), load all their weight vectors, scales
// and zeros before griddepcontrol.wait, and meet in shared memory for the
// final sum.  This keeps a lone GEMV's critical path to one load latency plus
// 1/W of its math.
// ---------------------------------------------------------------------------
template <int M, int KG, int MATH, int W>
__global__ void __launch_bounds__(W * 32)
w4a16_ksplit_kernel(const __grid_constant__ GroupParams gp) {
    __shared__ float4 red[W][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int strip = static_cast<int>(blockIdx.x);
    const int pi = find_problem(gp, strip, 0);
    const Problem& P = gp.p[pi];
    const int K = P.K, G = K / kGroup, Gp = (G + 7) & ~7, zw = (G + 7) >> 3;
    const int sl = strip - P.strip_begin;
    const int col = sl * 16 + g;
    uint4 v[KG][2];
    float slo[KG], shi[KG];
    int zlo[KG], zhi[KG];
#pragma unroll
    for (int j = 0; j < KG; ++j) {
        const int gi = warp + j * W;
        v[j][0] = v[j][1] = make_uint4(0, 0, 0, 0);
        slo[j] = shi[j] = 0.0f;
        zlo[j] = zhi[j] = 0;
        if (gi < G) {
            const size_t base = (static_cast<size_t>(sl) * (K / 64) + 2 * gi) * 32 + lane;
            v[j][0] = ld_stream(P.qw + base);
            v[j][1] = ld_stream(P.qw + base + 32);
            slo[j] = __half2float(P.s[static_cast<size_t>(col) * Gp + gi]);
            shi[j] = __half2float(P.s[static_cast<size_t>(col + 8) * Gp + gi]);
            zlo[j] = static_cast<int>((P.z[static_cast<size_t>(col) * zw + (gi >> 3)] >> (4 * (gi & 7))) & 0xfu);
            zhi[j] = static_cast<int>((P.z[static_cast<size_t>(col + 8) * zw + (gi >> 3)] >> (4 * (gi & 7))) & 0xfu);
        }
    }
    pdl_trigger();
    pdl_wait();  // x may be the previous kernel's output
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < KG; ++j) {
        const int gi = warp + j * W;
        if (gi >= G) break;
        float d[4];
        group_mma<M, MATH>(v[j], P.x + static_cast<size_t>(g) * K + gi * kGroup + 16 * t, g, zlo[j] + P.zero_bias,
                     zhi[j] + P.zero_bias, d);
        acc[0] = fmaf(d[0], slo[j], acc[0]);
        acc[1] = fmaf(d[1], slo[j], acc[1]);
        acc[2] = fmaf(d[2], shi[j], acc[2]);
        acc[3] = fmaf(d[3], shi[j], acc[3]);
    }
    red[warp][lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    __syncthreads();
    if (warp == 0) {
        float4 sum = red[0][lane];
#pragma unroll
        for (int w = 1; w < W; ++w) {
            const float4 r = red[w][lane];
            sum.x += r.x;
            sum.y += r.y;
            sum.z += r.z;
            sum.w += r.w;
        }
        const float out4[4] = {sum.x, sum.y, sum.z, sum.w};
        store_strip<M>(P, sl, lane, out4);
    }
}

// Batched decode, M = 9..64 rows of x: the K-split schedule with each
// dequantised A fragment feeding MT = ceil(M / 8) MMAs, one per 8 rows of x
// (the MMA's N), so the dequant work per weight is paid once for up to 64
// rows.  Lane (g, t) supplies x row 8T + g of tile T and ends with the
// outputs of rows 8T + 2t, 8T + 2t + 1 for columns g, g + 8 of the strip.
template <int MT, int KG>
__global__ void __launch_bounds__(kWarps * 32)
w4a16_ksplit_wide_kernel(const __grid_constant__ GroupParams gp, int M) {
    __shared__ float4 red[kWarps][MT][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int strip = static_cast<int>(blockIdx.x);
    const int pi = find_problem(gp, strip, 0);
    const Problem& P = gp.p[pi];
    const int K = P.K, G = K / kGroup, Gp = (G + 7) & ~7, zw = (G + 7) >> 3;
    const int sl = strip - P.strip_begin;
    const int col = sl * 16 + g;
    uint4 v[KG][2];
    float slo[KG], shi[KG];
    int zlo[KG], zhi[KG];
#pragma unroll
    for (int j = 0; j < KG; ++j) {
        const int gi = warp + j * kWarps;
        v[j][0] = v[j][1] = make_uint4(0, 0, 0, 0);
        slo[j] = shi[j] = 0.0f;
        zlo[j] = zhi[j] = 0;
        if (gi < G) {
            const size_t base = (static_cast<size_t>(sl) * (K / 64) + 2 * gi) * 32 + lane;
            v[j][0] = ld_stream(P.qw + base);
            v[j][1] = ld_stream(P.qw + base + 32);
            slo[j] = __half2float(P.s[static_cast<size_t>(col) * Gp + gi]);
            shi[j] = __half2float(P.s[static_cast<size_t>(col + 8) * Gp + gi]);
            zlo[j] = static_cast<int>((P.z[static_cast<size_t>(col) * zw + (gi >> 3)] >> (4 * (gi & 7))) & 0xfu);
            zhi[j] = static_cast<int>((P.z[static_cast<size_t>(col + 8) * zw + (gi >> 3)] >> (4 * (gi & 7))) & 0xfu);
        }
    }
    pdl_trigger();
    pdl_wait();  // x may be the previous kernel's output
    float acc[MT][4];
#pragma unroll
    for (int T = 0; T < MT; ++T) acc[T][0] = acc[T][1] = acc[T][2] = acc[T][3] = 0.0f;
    constexpr uint32_t kMagic = 0x64006400u;
    const __half2 inv16 = u32_as_h2(0x2c002c00u);
#pragma unroll
    for (int j = 0; j < KG; ++j) {
        const int gi = warp + j * kWarps;
        if (gi >= G) break;
        const __half2 zl = u32_as_h2(h2_bits_1024_plus(zlo[j] + P.zero_bias));
        const __half2 zh = u32_as_h2(h2_bits_neg_64_plus(zhi[j] + P.zero_bias));
        float c[MT][4];
#pragma unroll
        for (int T = 0; T < MT; ++T) c[T][0] = c[T][1] = c[T][2] = c[T][3] = 0.0f;
#pragma unroll
        for (int qd = 0; qd < 2; ++qd) {
            uint4 xv[MT][2];
#pragma unroll
            for (int T = 0; T < MT; ++T) {
                xv[T][0] = xv[T][1] = make_uint4(0, 0, 0, 0);
                const int row = 8 * T + g;
                if (row < M) {
                    const __half* xg = P.x + static_cast<size_t>(row) * K + gi * kGroup + qd * 64 + 16 * t;
                    xv[T][0] = *reinterpret_cast<const uint4*>(xg);
                    xv[T][1] = *reinterpret_cast<const uint4*>(xg + 8);
                }
            }
            const uint4 vv = v[j][qd];
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                const uint32_t w = jj == 0 ? vv.x : jj == 1 ? vv.y : jj == 2 ? vv.z : vv.w;
                const uint32_t w8 = w >> 8;
                uint32_t a[4];
                a[0] = h2_as_u32(__hsub2(u32_as_h2(lop3_and_or(w, 0x000f000fu, kMagic)), zl));
                a[1] = h2_as_u32(__hfma2(u32_as_h2(lop3_and_or(w, 0x00f000f0u, kMagic)), inv16, zh));
                a[2] = h2_as_u32(__hsub2(u32_as_h2(lop3_and_or(w8, 0x000f000fu, kMagic)), zl));
                a[3] = h2_as_u32(__hfma2(u32_as_h2(lop3_and_or(w8, 0x00f000f0u, kMagic)), inv16, zh));
#pragma unroll
                for (int T = 0; T < MT; ++T) {
                    const uint4 xx = xv[T][jj >> 1];
                    mma_16816(c[T], a, (jj & 1) ? xx.z : xx.x, (jj & 1) ? xx.w : xx.y);
                }
            }
        }
#pragma unroll
        for (int T = 0; T < MT; ++T) {
            acc[T][0] = fmaf(c[T][0], slo[j], acc[T][0]);
            acc[T][1] = fmaf(c[T][1], slo[j], acc[T][1]);
            acc[T][2] = fmaf(c[T][2], shi[j], acc[T][2]);
            acc[T][3] = fmaf(c[T][3], shi[j], acc[T][3]);
        }
    }
#pragma unroll
    for (int T = 0; T < MT; ++T) red[warp][T][lane] = make_float4(acc[T][0], acc[T][1], acc[T][2], acc[T][3]);
    __syncthreads();
    // warps 0..MT-1 each finish one tile of 8 rows
    if (warp < MT) {
        const int T = warp;
        float4 sum = red[0][T][lane];
#pragma unroll
        for (int w = 1; w < kWarps; ++w) {
            const float4 r = red[w][T][lane];
            sum.x += r.x;
            sum.y += r.y;
            sum.z += r.z;
            sum.w += r.w;
        }
        const int n0 = sl * 16;
        const size_t N = static_cast<size_t>(P.N);
        const int m0 = 8 * T + 2 * t;
        if (m0 < M) {
            if (n0 + g < P.N) P.out[m0 * N + n0 + g] = __float2half_rn(sum.x);
            if (n0 + g + 8 < P.N) P.out[m0 * N + n0 + g + 8] = __float2half_rn(sum.z);
        }
        if (m0 + 1 < M) {
            if (n0 + g < P.N) P.out[(m0 + 1) * N + n0 + g] = __float2half_rn(sum.y);
            if (n0 + g + 8 < P.N) P.out[(m0 + 1) * N + n0 + g + 8] = __float2half_rn(sum.w);
        }
    }
}

int assign_strips(GroupParams& gp);

template <int MT>
int launch_wide_mt(GroupParams& gp, int M, cudaStream_t st) {
    const int strips = assign_strips(gp);
    int maxG = 0;
    for (int i = 0; i < gp.count; ++i) maxG = std::max(maxG, gp.p[i].K / kGroup);
    const int per_warp = (maxG + kWarps - 1) / kWarps;
    auto go = [&](auto kern) { return launch(kern, dim3(strips), dim3(kWarps * 32), 0, st, gp, M); };
    if (per_warp <= 1) return go(w4a16_ksplit_wide_kernel<MT, 1>);
    if (per_warp <= 2) return go(w4a16_ksplit_wide_kernel<MT, 2>);
    if (per_warp <= 4) return go(w4a16_ksplit_wide_kernel<MT, 4>);
    if (per_warp <= 8) return go(w4a16_ksplit_wide_kernel<MT, 8>);
    return fail(MCV_ERR_SHAPE, "w4a16_gemv: M > 8 needs K <= 8192");
}

int run_group_wide(GroupParams& gp, int M, cudaStream_t st) {
    if (M <= 16) return launch_wide_mt<2>(gp, M, st);
    if (M <= 24) return launch_wide_mt<3>(gp, M, st);
    if (M <= 32) return launch_wide_mt<4>(gp, M, st);
    if (M <= 48) return launch_wide_mt<6>(gp, M, st);
    return launch_wide_mt<8>(gp, M, st);
}

// The MLP's gate and up projections with SwiGLU in the epilogue
// (decoder_layer.cpp:1186-1203): act = silu_mul(x . Wg, x . Wu).  Block b
// computes strip b of both weights with 2W warps - warps 0..W-1 the gate,
// W..2W-1 the up projection (W = 8, or 16 above 1024 k), each half splitting
// K exactly as the K-split kernel does,
// so the sums (and, after rounding to fp16, the projections' outputs) are the
// separate GEMVs' bit for bit.  silu_mul's arithmetic then runs on the two
// fp16 values, so one launch replaces the gate/up launch plus the silu_mul
// launch, and the fp16 gate and up never travel through memory.
template <int M, int KG, int W>
__global__ void __launch_bounds__(2 * W * 32)
w4a16_gate_up_silu_kernel(const __grid_constant__ GroupParams gp) {
    __shared__ float4 red[2 * W][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int strip = static_cast<int>(blockIdx.x);
    const int wq = warp & (W - 1);
    const Problem& P = gp.p[warp / W];  // 0: gate, 1: up
    const int K = P.K, G = K / kGroup, Gp = (G + 7) & ~7, zw = (G + 7) >> 3;
    const int col = strip * 16 + g;
    uint4 v[KG][2];
    float slo[KG], shi[KG];
    int zlo[KG], zhi[KG];
#pragma unroll
    for (int j = 0; j < KG; ++j) {
        const int gi = wq + j * W;
        v[j][0] = v[j][1] = make_uint4(0, 0, 0, 0);
        slo[j] = shi[j] = 0.0f;
        zlo[j] = zhi[j] = 0;
        if (gi < G) {
            const size_t base = (static_cast<size_t>(strip) * (K / 64) + 2 * gi) * 32 + lane;
            v[j][0] = ld_stream(P.qw + base);
            v[j][1] = ld_stream(P.qw + base + 32);
            slo[j] = __half2float(P.s[static_cast<size_t>(col) * Gp + gi]);
            shi[j] = __half2float(P.s[static_cast<size_t>(col + 8) * Gp + gi]);
            zlo[j] = static_cast<int>((P.z[static_cast<size_t>(col) * zw + (gi >> 3)] >> (4 * (gi & 7))) & 0xfu);
            zhi[j] = static_cast<int>((P.z[static_cast<size_t>(col + 8) * zw + (gi >> 3)] >> (4 * (gi & 7))) & 0xfu);
        }
    }
    pdl_trigger();
    pdl_wait();  // x may be the previous kernel's output
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < KG; ++j) {
        const int gi = wq + j * W;
        if (gi >= G) break;
        float d[4];
        group_mma<M>(v[j], P.x + static_cast<size_t>(g) * K + gi * kGroup + 16 * t, g, zlo[j] + P.zero_bias,
                     zhi[j] + P.zero_bias, d);
        acc[0] = fmaf(d[0], slo[j], acc[0]);
        acc[1] = fmaf(d[1], slo[j], acc[1]);
        acc[2] = fmaf(d[2], shi[j], acc[2]);
        acc[3] = fmaf(d[3], shi[j], acc[3]);
    }
    red[warp][lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    __syncthreads();
    if (warp == 0) {
        float4 gs = red[0][lane], us = red[W][lane];
#pragma unroll
        for (int w = 1; w < W; ++w) {
            const float4 a = red[w][lane], b = red[W + w][lane];
            gs.x += a.x, gs.y += a.y, gs.z += a.z, gs.w += a.w;
            us.x += b.x, us.y += b.y, us.z += b.z, us.w += b.w;
        }
        const Problem& Q = gp.p[0];
        const int n0 = strip * 16;
        const size_t N = static_cast<size_t>(Q.N);
        const int m0 = 2 * t;
        auto put = [&](int m, int n, float gv, float uv) {
            if (m < M && n < Q.N) Q.out[m * N + n] = silu_mul1(__float2half_rn(gv), __float2half_rn(uv));
        };
        put(m0, n0 + g, gs.x, us.x);
        put(m0, n0 + g + 8, gs.z, us.z);
        put(m0 + 1, n0 + g, gs.y, us.y);
        put(m0 + 1, n0 + g + 8, gs.w, us.w);
    }
}

template <int M>
int launch_gate_up_m(GroupParams& gp, cudaStream_t st) {
    const int strips = static_cast<int>(padded_n(gp.p[0].N) / 16);
    const int G = gp.p[0].K / kGroup;
    // warps per half as the single-GEMV kernel picks them (8, or 16 above
    // 1024 k), so the two give the same sums
    const int W = G > kWarps ? 2 * kWarps : kWarps;
    const int per_warp = (G + W - 1) / W;
    auto go = [&](auto kern) { return launch(kern, dim3(strips), dim3(2 * W * 32), 0, st, gp); };
    if (W == kWarps) {
        if (per_warp <= 1) return go(w4a16_gate_up_silu_kernel<M, 1, kWarps>);
        if (per_warp <= 2) return go(w4a16_gate_up_silu_kernel<M, 2, kWarps>);
        return go(w4a16_gate_up_silu_kernel<M, 4, kWarps>);
    }
    if (per_warp <= 1) return go(w4a16_gate_up_silu_kernel<M, 1, 2 * kWarps>);
    return go(w4a16_gate_up_silu_kernel<M, 2, 2 * kWarps>);
}

int assign_strips(GroupParams& gp) {
    int t = 0;
    for (int i = 0; i < gp.count; ++i) {
        gp.p[i].strip_begin = t;
        t += static_cast<int>(padded_n(gp.p[i].N) / 16);
    }
    gp.total_strips = t;
    return t;
}

// MATH < 0: each schedule's measured default - the K-split kernel's
// four-chain arithmetic (variant 0; 1.73 vs 1.76 us per dependent GEMV) and
// the bulk-copy ring's two chains with integer-built zero constants (variant
// 1; 0.500 vs 0.516 us per GEMV in a 48-GEMV launch).
template <int M, int MATH_ARG>
int launch_m(GroupParams& gp, cudaStream_t st) {
    constexpr int MATH = MATH_ARG < 0 ? 0 : MATH_ARG;
    constexpr int RING_MATH = MATH_ARG < 0 ? 1 : MATH_ARG;
    const int strips = assign_strips(gp);
    const int mode = tuning(MCV_TUNE_W4A16_MODE);
    // few strips: one block per strip with K split over its warps; many
    // strips: the persistent streaming kernel fed by warp-private bulk-copy
    // rings (3 blocks of 8 warps per SM: 0.549 vs 0.589 us per config-0 GEMV
    // in a 48-GEMV launch against the register-buffered kernel, measured on B200)
    if (mode == 2 || (mode == 0 && strips < sm_count() * 4)) {
        int maxG = 0;
        for (int i = 0; i < gp.count; ++i) maxG = std::max(maxG, gp.p[i].K / kGroup);
        const int tw = tuning(MCV_TUNE_W4A16_KSPLIT_WARPS);
        // warps per strip: one per 128-k group up to 16 (K = 2048 / 3584 on 16
        // warps: more loads in flight per strip before the wait; measured on
        // the decode step's launch sequence); MCV_TUNE_W4A16_KSPLIT_WARPS
        // = 8 / 16 / 32 forces one
        int W = maxG > kWarps ? 2 * kWarps : kWarps;
        if (tw == 8 || tw == 16 || tw == 32) W = tw;
        if (MATH != 0) W = kWarps;
        const int per_warp = (maxG + W - 1) / W;
        auto go = [&](auto kern, int w) { return launch(kern, dim3(strips), dim3(w * 32), 0, st, gp); };
        if (W == 8) {
            if (per_warp <= 1) return go(w4a16_ksplit_kernel<M, 1, MATH, 8>, 8);
            if (per_warp <= 2) return go(w4a16_ksplit_kernel<M, 2, MATH, 8>, 8);
            if (per_warp <= 4) return go(w4a16_ksplit_kernel<M, 4, MATH, 8>, 8);
            if (per_warp <= 8) return go(w4a16_ksplit_kernel<M, 8, MATH, 8>, 8);
        } else if constexpr (MATH == 0) {
            if (W == 16) {
                if (per_warp <= 1) return go(w4a16_ksplit_kernel<M, 1, 0, 16>, 16);
                if (per_warp <= 2) return go(w4a16_ksplit_kernel<M, 2, 0, 16>, 16);
                if (per_warp <= 4) return go(w4a16_ksplit_kernel<M, 4, 0, 16>, 16);
            } else {
                if (per_warp <= 1) return go(w4a16_ksplit_kernel<M, 1, 0, 32>, 32);
                if (per_warp <= 2) return go(w4a16_ksplit_kernel<M, 2, 0, 32>, 32);
            }
        }
        // larger K: the streaming kernel has no K limit
    }
    if (mode == 1) {
        // register-buffered streaming kernel; at most kBlocksPerSm blocks per SM
        const int blocks = std::min(strips, sm_count() * kBlocksPerSm);
        return launch(w4a16_gemv_kernel<M>, dim3(blocks), dim3(kWarps * 32), 0, st, gp);
    }
    auto kern = w4a16_tma_kernel<M, RING_MATH>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kTmaSmem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(w4a16_tma)");
    // As many warps as fit (3 blocks of 8 per SM): the stream is bound by
    // bytes in flight per warp, so fewer warps with an even strip count each
    // measured slower (48 config-0 GEMVs: 0.66 us per GEMV on 336 blocks
    // against 0.55 us on 444, although 96 of the 3552 warps take a 4th strip).
    const int max_blocks = sm_count() * kTmaBlocksPerSm;
    int blocks = std::min((strips + kWarps - 1) / kWarps, max_blocks);
    const int t = tuning(MCV_TUNE_W4A16_GRID);
    if (t > 0) blocks = std::min(t, max_blocks);
    return launch(kern, dim3(blocks), dim3(kWarps * 32), static_cast<size_t>(kTmaSmem), st, gp);
}

template <int MATH>
int run_group_math(GroupParams& gp, int64_t M, cudaStream_t st) {
    switch (M) {
        case 1: return launch_m<1, MATH>(gp, st);
        case 2: return launch_m<2, MATH>(gp, st);
        case 3: return launch_m<3, MATH>(gp, st);
        case 4: return launch_m<4, MATH>(gp, st);
        case 5: return launch_m<5, MATH>(gp, st);
        case 6: return launch_m<6, MATH>(gp, st);
        case 7: return launch_m<7, MATH>(gp, st);
        default: return launch_m<8, MATH>(gp, st);
    }
}

int run_group(GroupParams& gp, int64_t M, cudaStream_t st) {
    if (M > 8) return run_group_wide(gp, static_cast<int>(M), st);
    switch (tuning(MCV_TUNE_W4A16_MATH)) {
        case 1: return run_group_math<0>(gp, M, st);
        case 2: return run_group_math<1>(gp, M, st);
        case 3: return run_group_math<2>(gp, M, st);
        default: return run_group_math<-1>(gp, M, st);
    }
}

int check_layout_dims(int64_t K, int64_t N, int64_t group) {
    if (K <= 0 || N <= 0 || group <= 0) return fail(MCV_ERR_SHAPE, "w4a16: K, N, group must be positive");
    if (group != kGroup) return fail(MCV_ERR_SHAPE, "w4a16: group size must be 128 (as in the reference)");
    if (K % group != 0) return fail(MCV_ERR_SHAPE, "w4a16: K must be a multiple of 128");
    if (K > (1 << 20) || N > (1 << 28)) return fail(MCV_ERR_SHAPE, "w4a16: dimension too large");
    return MCV_OK;
}

// Writes the three mcv-int4 arrays from a logical accessor q(k,n) (0..15)
// and zero z(g,n) (0..15); padding columns get q = z = 0 and scale 0.
template <typename QF, typename ZF>
void pack_layout(QF q, ZF z, const uint16_t* scales_gn, int64_t K, int64_t N, int64_t group,
                 uint32_t* qw, uint16_t* sc, uint32_t* zw) {
    const int64_t G = K / group, Gp = padded_g(G), Np = padded_n(N), KQ = K / 64;
    const int64_t zwords = (G + 7) / 8;
    for (int64_t strip = 0; strip < Np / 16; ++strip)
        for (int64_t kq = 0; kq < KQ; ++kq)
            for (int lane = 0; lane < 32; ++lane)
                for (int j = 0; j < 4; ++j) {  // k-block 4*kq + j -> component j of the lane vector
                    const int gg = lane >> 2, t = lane & 3;
                    uint32_t word = 0;
                    for (int e = 0; e < 8; ++e) {
                        const int64_t n = strip * 16 + gg + kFragRow[e];
                        const int64_t k = kq * 64 + 16 * t + 4 * j + kFragK[e];
                        const uint32_t v = n < N ? (static_cast<uint32_t>(q(k, n)) & 0xfu) : 0u;
                        word |= v << (4 * kFragSlot[e]);
                    }
                    qw[((strip * KQ + kq) * 32 + lane) * 4 + j] = word;
                }
    for (int64_t n = 0; n < Np; ++n) {
        for (int64_t g = 0; g < Gp; ++g) sc[n * Gp + g] = (n < N && g < G) ? scales_gn[g * N + n] : 0;
        for (int64_t t = 0; t < zwords; ++t) zw[n * zwords + t] = 0;
        if (n < N)
            for (int64_t g = 0; g < G; ++g)
                zw[n * zwords + g / 8] |= (static_cast<uint32_t>(z(g, n)) & 0xfu) << (4 * (g % 8));
    }
}

}  // namespace

unsigned take_w4a16_device_error() {
    unsigned v = 0;
    if (cudaMemcpyFromSymbol(&v, g_w4a16_dev_error, sizeof(v)) != cudaSuccess) return ~0u;
    if (v) {
        const unsigned zero = 0;
        cudaMemcpyToSymbol(g_w4a16_dev_error, &zero, sizeof(zero));
    }
    return v;
}

}  // namespace mcv

using namespace mcv;

extern "C" {

int mcv_w4a16_layout_bytes(int64_t K, int64_t N, int64_t group, size_t* qb, size_t* sb, size_t* zb) {
    int st = check_layout_dims(K, N, group);
    if (st) return st;
    const int64_t G = K / group, Np = padded_n(N);
    if (qb) *qb = static_cast<size_t>(Np) * (K / 8) * 4;
    if (sb) *sb = static_cast<size_t>(Np) * padded_g(G) * 2;
    if (zb) *zb = static_cast<size_t>(Np) * ((G + 7) / 8) * 4;
    return MCV_OK;
}

int mcv_w4a16_pack_host(const uint8_t* q_kn, const uint8_t* z_gn, const uint16_t* scales_gn,
                        int64_t K, int64_t N, int64_t group, uint32_t* qw, uint16_t* sc,
                        uint32_t* zw) {
    if (!q_kn || !z_gn || !scales_gn || !qw || !sc || !zw) return fail(MCV_ERR_NULL, "w4a16_pack_host: null pointer");
    int st = check_layout_dims(K, N, group);
    if (st) return st;
    pack_layout([&](int64_t k, int64_t n) { return q_kn[k * N + n]; },
                [&](int64_t g, int64_t n) { return z_gn[g * N + n]; }, scales_gn, K, N, group, qw, sc, zw);
    return MCV_OK;
}

int mcv_w4a16_unpack_host(const uint32_t* qw, const uint16_t* sc, const uint32_t* zw, int zero_bias, int64_t K,
                          int64_t N, int64_t group, int8_t* w_kn, uint16_t* scales_gn) {
    if (!qw || !sc || !zw || !w_kn || !scales_gn) return fail(MCV_ERR_NULL, "w4a16_unpack_host: null pointer");
    int st = check_layout_dims(K, N, group);
    if (st) return st;
    const int64_t G = K / group, Gp = padded_g(G), KQ = K / 64, zwords = (G + 7) / 8;
    // inverse of pack_layout: nibble slot kFragSlot[e] of word j of lane
    // vector (strip, kq, lane) holds (n, k) = (16 strip + g + kFragRow[e],
    // 64 kq + 16 t + 4 j + kFragK[e])
    for (int64_t strip = 0; strip < padded_n(N) / 16; ++strip)
        for (int64_t kq = 0; kq < KQ; ++kq)
            for (int lane = 0; lane < 32; ++lane)
                for (int j = 0; j < 4; ++j) {
                    const uint32_t word = qw[((strip * KQ + kq) * 32 + lane) * 4 + j];
                    const int gg = lane >> 2, t = lane & 3;
                    for (int e = 0; e < 8; ++e) {
                        const int64_t n = strip * 16 + gg + kFragRow[e];
                        const int64_t k = kq * 64 + 16 * t + 4 * j + kFragK[e];
                        if (n >= N) continue;
                        const int q = static_cast<int>((word >> (4 * kFragSlot[e])) & 0xfu);
                        const int z = static_cast<int>((zw[n * zwords + (k / group) / 8] >> (4 * ((k / group) % 8))) & 0xfu) +
                                      zero_bias;
                        w_kn[k * N + n] = static_cast<int8_t>(q - z);
                    }
                }
    for (int64_t g = 0; g < G; ++g)
        for (int64_t n = 0; n < N; ++n) scales_gn[g * N + n] = sc[n * Gp + g];
    return MCV_OK;
}

int mcv_w4a16_pack_gptq_host(const int32_t* qweight, const int32_t* qzeros, const int32_t* g_idx,
                             const uint16_t* scales, int64_t K, int64_t N, int64_t group,
                             uint32_t* qw, uint16_t* sc, uint32_t* zw, int* zero_bias_out) {
    if (!qweight || !qzeros || !scales || !qw || !sc || !zw) return fail(MCV_ERR_NULL, "w4a16_pack_gptq_host: null pointer");
    int st = check_layout_dims(K, N, group);
    if (st) return st;
    if (N % 8 != 0) return fail(MCV_ERR_SHAPE, "w4a16_pack_gptq_host: N must be a multiple of 8");
    if (g_idx) {
        for (int64_t k = 0; k < K; ++k)
            if (g_idx[k] != k / group)
                return fail(MCV_ERR_VALUE, "w4a16_pack_gptq_host: g_idx is not k/group (act-order GPTQ unsupported)");
    }
    // GPTQ: qweight word (k/8, n) holds k at nibble k%8; qzeros word (g, n/8)
    // holds column n at nibble n%8, true zero = stored + 1
    // (src/csrc/lib/quantized_weight.cpp:104-114).
    pack_layout([&](int64_t k, int64_t n) { return (static_cast<uint32_t>(qweight[(k / 8) * N + n]) >> (4 * (k % 8))) & 0xfu; },
                [&](int64_t g, int64_t n) { return (static_cast<uint32_t>(qzeros[g * (N / 8) + n / 8]) >> (4 * (n % 8))) & 0xfu; },
                scales, K, N, group, qw, sc, zw);
    if (zero_bias_out) *zero_bias_out = 1;
    return MCV_OK;
}

int mcv_w4a16_pack_awq_host(const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                            int64_t K, int64_t N, int64_t group, uint32_t* qw, uint16_t* sc,
                            uint32_t* zw, int* zero_bias_out) {
    if (!qweight || !qzeros || !scales || !qw || !sc || !zw) return fail(MCV_ERR_NULL, "w4a16_pack_awq_host: null pointer");
    int st = check_layout_dims(K, N, group);
    if (st) return st;
    if (N % 8 != 0) return fail(MCV_ERR_SHAPE, "w4a16_pack_awq_host: N must be a multiple of 8");
    // AWQ: column j*8 + {0,2,4,6,1,3,5,7}[s] sits in slot s of word (k, j)
    // (src/csrc/lib/quantized_weight.cpp:17, 147-156); invert that order.
    static const int slot_of_col[8] = {0, 4, 1, 5, 2, 6, 3, 7};
    const int64_t np = N / 8;
    pack_layout([&](int64_t k, int64_t n) { return (static_cast<uint32_t>(qweight[k * np + n / 8]) >> (4 * slot_of_col[n % 8])) & 0xfu; },
                [&](int64_t g, int64_t n) { return (static_cast<uint32_t>(qzeros[g * np + n / 8]) >> (4 * slot_of_col[n % 8])) & 0xfu; },
                scales, K, N, group, qw, sc, zw);
    if (zero_bias_out) *zero_bias_out = 0;
    return MCV_OK;
}

int mcv_w4a16_pack_from_tiles_host(const int8_t* packed, int64_t tile_len, const uint16_t* scales_gn,
                                   int64_t K, int64_t N, uint32_t* qw, uint16_t* sc, uint32_t* zw,
                                   int* zero_bias_out) {
    if (!packed || !scales_gn || !qw || !sc || !zw) return fail(MCV_ERR_NULL, "w4a16_pack_from_tiles_host: null pointer");
    const int64_t group = 128;
    int st = check_layout_dims(K, N, group);
    if (st) return st;
    if (tile_len <= 0 || tile_len > 448 || tile_len % 16 != 0)
        return fail(MCV_ERR_SHAPE, "w4a16_pack_from_tiles_host: tile_len must be a multiple of 16 and <= 448");
    // Undo the (group, core, tile, k) tile pack of quantized_weight.cpp:48-73.
    const int64_t block_len = (N + 7) / 8;
    const int64_t tpb = (block_len + tile_len - 1) / tile_len;
    std::vector<int8_t> w(static_cast<size_t>(K) * N);
    for (int64_t g = 0; g < K / group; ++g)
        for (int64_t b = 0; b < 8; ++b) {
            const int64_t bstart = b * block_len;
            const int64_t bvalid = std::max<int64_t>(0, std::min<int64_t>(block_len, N - bstart));
            for (int64_t t = 0; t < tpb; ++t) {
                const int64_t tstart = t * tile_len;
                const int64_t tvalid = std::max<int64_t>(0, std::min<int64_t>(tile_len, bvalid - tstart));
                const int64_t base = (((g * 8 + b) * tpb + t) * group) * tile_len;
                for (int64_t kk = 0; kk < group; ++kk)
                    for (int64_t i = 0; i < tvalid; ++i)
                        w[(g * group + kk) * N + bstart + tstart + i] = packed[base + kk * tile_len + i];
            }
        }
    // Per (group, column): values v = q - zero must map to q in 0..15.
    const int64_t G = K / group;
    std::vector<int> lo(static_cast<size_t>(G) * N, 127), hi(static_cast<size_t>(G) * N, -128);
    for (int64_t k = 0; k < K; ++k)
        for (int64_t n = 0; n < N; ++n) {
            const int v = w[k * N + n];
            const size_t i = static_cast<size_t>(k / group) * N + n;
            lo[i] = std::min(lo[i], v);
            hi[i] = std::max(hi[i], v);
        }
    int bias = 0;
    for (size_t i = 0; i < lo.size(); ++i) {
        if (hi[i] - lo[i] > 15) return fail(MCV_ERR_VALUE, "w4a16_pack_from_tiles_host: a group spans more than 16 levels");
        if (-lo[i] > 15) bias = 1;
    }
    std::vector<uint8_t> z(lo.size());
    for (size_t i = 0; i < lo.size(); ++i) {
        // zero in [max(-lo, bias), min(15 - hi, 15 + bias)]
        const int zmin = std::max(-lo[i], bias);
        const int zmax = std::min(15 - hi[i], 15 + bias);
        if (zmin > zmax) return fail(MCV_ERR_VALUE, "w4a16_pack_from_tiles_host: no 4-bit zero fits a group");
        z[i] = static_cast<uint8_t>(zmin - bias);
    }
    pack_layout([&](int64_t k, int64_t n) { return static_cast<uint32_t>(w[k * N + n] + z[(k / group) * N + n] + bias); },
                [&](int64_t g, int64_t n) { return static_cast<uint32_t>(z[g * N + n]); },
                scales_gn, K, N, group, qw, sc, zw);
    if (zero_bias_out) *zero_bias_out = bias;
    return MCV_OK;
}

int mcv_w4a16_gemv(const void* x, const void* qweight, const void* scales, const void* zeros,
                   int zero_bias, void* out, int64_t M, int64_t K, int64_t N, int64_t group,
                   mcv_stream_t stream) {
    if (K > (1 << 20) || N > (1 << 28)) return fail(MCV_ERR_SHAPE, "w4a16: dimension too large");
    mcv_w4a16_problem p{x, qweight, scales, zeros, out, static_cast<int32_t>(K), static_cast<int32_t>(N),
                        static_cast<int32_t>(group), zero_bias};
    return mcv_w4a16_gemv_grouped(&p, 1, M, stream);
}

int mcv_w4a16_gemv_gate_up_silu(const void* x, const mcv_w4a16_problem* gate, const mcv_w4a16_problem* up, void* act,
                                int64_t M, mcv_stream_t stream) {
    if (!x || !gate || !up || !act) return fail(MCV_ERR_NULL, "w4a16_gate_up_silu: null pointer");
    if (M < 1 || M > 8) return fail(MCV_ERR_SHAPE, "w4a16_gate_up_silu: M must be 1..8");
    const mcv_w4a16_problem* ps[2] = {gate, up};
    for (const mcv_w4a16_problem* p : ps) {
        if (!p->qweight || !p->scales || !p->zeros) return fail(MCV_ERR_NULL, "w4a16_gate_up_silu: null weight pointer");
        int st = check_layout_dims(p->K, p->N, p->group);
        if (st) return st;
        if (!aligned16(p->qweight) || !aligned16(p->scales))
            return fail(MCV_ERR_ALIGN, "w4a16_gate_up_silu: qweight and scales must be 16-byte aligned");
        if (reinterpret_cast<uintptr_t>(p->zeros) & 3u) return fail(MCV_ERR_ALIGN, "w4a16_gate_up_silu: zeros must be 4-byte aligned");
        if (p->zero_bias < 0 || p->zero_bias > 1) return fail(MCV_ERR_VALUE, "w4a16_gate_up_silu: zero_bias must be 0 or 1");
    }
    if (gate->K != up->K || gate->N != up->N) return fail(MCV_ERR_SHAPE, "w4a16_gate_up_silu: gate and up shapes differ");
    if (gate->K > 32 * kGroup) return fail(MCV_ERR_SHAPE, "w4a16_gate_up_silu: K above 4096 unsupported");
    if (!aligned16(x)) return fail(MCV_ERR_ALIGN, "w4a16_gate_up_silu: x must be 16-byte aligned");
    GroupParams gp{};
    gp.count = 2;
    for (int i = 0; i < 2; ++i)
        gp.p[i] = Problem{static_cast<const __half*>(x), static_cast<const uint4*>(ps[i]->qweight),
                          static_cast<const __half*>(ps[i]->scales), static_cast<const uint32_t*>(ps[i]->zeros),
                          static_cast<__half*>(act), ps[i]->K, ps[i]->N, ps[i]->zero_bias, 0};
    auto s = static_cast<cudaStream_t>(stream);
    switch (M) {
        case 1: return launch_gate_up_m<1>(gp, s);
        case 2: return launch_gate_up_m<2>(gp, s);
        case 3: return launch_gate_up_m<3>(gp, s);
        case 4: return launch_gate_up_m<4>(gp, s);
        case 5: return launch_gate_up_m<5>(gp, s);
        case 6: return launch_gate_up_m<6>(gp, s);
        case 7: return launch_gate_up_m<7>(gp, s);
        default: return launch_gate_up_m<8>(gp, s);
    }
}

int mcv_w4a16_gemv_grouped(const mcv_w4a16_problem* problems, int count, int64_t M, mcv_stream_t stream) {
    if (!problems || count < 1) return fail(MCV_ERR_NULL, "w4a16_gemv: no problems");
    if (M < 1 || M > kMaxGemvRows) return fail(MCV_ERR_SHAPE, "w4a16_gemv: M must be 1..64");
    for (int i = 0; i < count; ++i) {
        const mcv_w4a16_problem& p = problems[i];
        if (!p.x || !p.qweight || !p.scales || !p.zeros || !p.out) return fail(MCV_ERR_NULL, "w4a16_gemv: null pointer");
        int st = check_layout_dims(p.K, p.N, p.group);
        if (st) return st;
        if (!aligned16(p.qweight) || !aligned16(p.scales) || !aligned16(p.x))
            return fail(MCV_ERR_ALIGN, "w4a16_gemv: x, qweight and scales must be 16-byte aligned");
        if (reinterpret_cast<uintptr_t>(p.zeros) & 3u)
            return fail(MCV_ERR_ALIGN, "w4a16_gemv: zeros must be 4-byte aligned");
        if (p.zero_bias < 0 || p.zero_bias > 1) return fail(MCV_ERR_VALUE, "w4a16_gemv: zero_bias must be 0 or 1");
    }
    auto st = static_cast<cudaStream_t>(stream);
    for (int base = 0; base < count; base += kMaxGroupProblems) {
        GroupParams gp{};
        gp.count = std::min(kMaxGroupProblems, count - base);
        for (int i = 0; i < gp.count; ++i) {
            const mcv_w4a16_problem& q = problems[base + i];
            gp.p[i] = Problem{static_cast<const __half*>(q.x), static_cast<const uint4*>(q.qweight),
                              static_cast<const __half*>(q.scales), static_cast<const uint32_t*>(q.zeros),
                              static_cast<__half*>(q.out), q.K, q.N, q.zero_bias, 0};
        }
        int rc = run_group(gp, M, st);
        if (rc) return rc;
    }
    return MCV_OK;
}

}  // extern "C"
