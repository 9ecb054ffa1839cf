// W4A16 GEMM for batched decode / prefill (M >= 16) on the 5th-generation
// tensor cores: tcgen05.mma with the fp32 accumulator in tensor memory.
//
// Reference counterpart: the reference has no quantized GEMM for M > 1 -
// prefill goes through matmul_b_transposed's dense aclnnMm / K-tiling path
// (src/csrc/lib/ops.cpp:215-322) and matmul_w4a16 is M=1 only (ops.cpp:1048).
// This kernel serves the same mcv-int4 weights as the decode GEMV.
//
// One block computes a 128 (rows of x) x 256 (output columns) tile with
// three roles that meet only on mbarriers (no block-wide barrier inside the
// k loop):
//  * a producer thread requests the x tiles [128 rows x 64 k] by TMA
//    (cp.async.bulk.tensor, 128-byte swizzle; rows past M are zero-filled by
//    the copy engine) into a 3-deep ring, refilling a slot once the MMAs that
//    read it are done;
//  * 512 dequantising threads each fetch (cp.async, three stages ahead) and
//    dequantise one 16-byte lane vector of the mcv-int4 layout per stage -
//    16 consecutive k of two columns - to fp16 (q - zero) * scale, store it
//    in the same 128-byte-swizzled K-major layout and arrive on the stage's
//    "weight ready" mbarrier;
//  * an issuer thread runs four tcgen05.mma.kind::f16 (M=128, N=256, K=16)
//    per 64-k stage once both operands are ready and commits them to the
//    stage's "done" mbarrier;
//  * the epilogue (the 16 dequantising warps) reads the accumulator with
//    tcgen05.ld (warp w owns TMEM lanes 32(w%4).. = rows, and a quarter of
//    the columns) and writes fp16.
// Every wait is bounded (2 s); on a timeout the block records an error bit,
// waits (bounded) for its own MMAs, frees its tensor memory and returns.
// Single-GPU code: no multicast, no peer memory.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace mcv {
unsigned take_gemm_device_error();

namespace {

constexpr int kBM = 128;         // rows of x per block (MMA M)
constexpr int kBN = 256;         // output columns per block (MMA N)
constexpr int kBK = 64;          // k per stage: one 128-byte swizzle row
constexpr int kStrips = kBN / 16;          // 16-column strips of the mcv-int4 layout per tile
constexpr int kDqThreads = kBN * 2;        // dequantising threads: one lane vector of the tile each
constexpr int kThreads = kDqThreads + 64;  // + an MMA-issuing warp and a producer warp
constexpr int kXBytes = kBM * kBK * 2;     // 16 KB x tile per stage
constexpr int kWBytes = kBN * kBK * 2;     // 32 KB dequantised weight tile per stage
constexpr int kQBytes = kBN * kBK / 2;     // 8 KB packed int4 weights per stage
constexpr int kStageBytes = kXBytes + kWBytes + kQBytes;
constexpr int kStages = 4;                 // ring depth
constexpr int kSmemBytes = kStages * kStageBytes + 1024 + 256;
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");

static __device__ unsigned g_gemm_dev_error;

// ---- tcgen05 / TMA primitives ------------------------------------------

// UMMA shared-memory descriptor for a K-major operand in the 128-byte
// swizzle layout: rows of 128 bytes, 8-row atoms 1024 bytes apart.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3fffu);         // start address
    d |= static_cast<uint64_t>(1u) << 16;                          // leading byte offset (unused here)
    d |= static_cast<uint64_t>((1024u >> 4) & 0x3fffu) << 32;     // stride byte offset: 8 rows
    d |= static_cast<uint64_t>(1u) << 46;                          // descriptor version
    d |= static_cast<uint64_t>(2u) << 61;                          // swizzle: 128 B
    return d;
}

// Instruction descriptor: kind::f16, fp16 A and B (both K-major), fp32 D.
__host__ __device__ constexpr uint32_t instr_desc_f16(int m, int n) {
    return (1u << 4)                                 // D format: f32
           | (0u << 7) | (0u << 10)                  // A, B format: f16
           | (static_cast<uint32_t>(n >> 3) << 17)   // N / 8
           | (static_cast<uint32_t>(m >> 4) << 24);  // M / 16
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

// 16 consecutive fp32 columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// ---- weight dequantisation into the swizzled K-major tile ----------------

// Lane vector (strip, quad, lane) -> 16 k of column g and of column g+8,
// written as fp16 (q - zero) * scale.  See include/mcv_matmul.h for the
// layout: word j holds k = 16t + 4j + {0,1,2,3} of rows g and g+8.
__device__ __forceinline__ void dequant_store(uint4 v, unsigned char* tile, int row_lo, int t, int zlo, int zhi,
                                              __half slo, __half shi) {
    constexpr uint32_t kMagic = 0x64006400u;
    const __half2 inv16 = __halves2half2(__ushort_as_half(0x2c00), __ushort_as_half(0x2c00));
    const __half z1 = __int2half_rn(1024 + zlo);
    const __half z2 = __int2half_rn(-(64 + zhi));
    const __half2 zl = __halves2half2(z1, z1), zh = __halves2half2(z2, z2);
    const __half2 sl = __halves2half2(slo, slo), sh = __halves2half2(shi, shi);
    uint32_t lo[8], hi[8];  // 16 halves of each row, in k order
    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t w = w4[j], w8 = w >> 8;
        const __half2 a0 = __hsub2(u32_as_h2(lop3_and_or(w, 0x000f000fu, kMagic)), zl);
        const __half2 a1 = __hfma2(u32_as_h2(lop3_and_or(w, 0x00f000f0u, kMagic)), inv16, zh);
        const __half2 a2 = __hsub2(u32_as_h2(lop3_and_or(w8, 0x000f000fu, kMagic)), zl);
        const __half2 a3 = __hfma2(u32_as_h2(lop3_and_or(w8, 0x00f000f0u, kMagic)), inv16, zh);
        lo[2 * j] = h2_as_u32(__hmul2(a0, sl));
        lo[2 * j + 1] = h2_as_u32(__hmul2(a2, sl));
        hi[2 * j] = h2_as_u32(__hmul2(a1, sh));
        hi[2 * j + 1] = h2_as_u32(__hmul2(a3, sh));
    }
    // k = 16t .. 16t+15 is 16-byte chunks 2t and 2t+1 of the 128-byte row;
    // 128-byte swizzle: chunk c of row r is stored at chunk c ^ (r & 7)
    const int rh = row_lo + 8;  // row_lo & 7 == rh & 7
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        const int chunk = (2 * t + c) ^ (row_lo & 7);
        *reinterpret_cast<uint4*>(tile + row_lo * 128 + chunk * 16) =
            make_uint4(lo[4 * c], lo[4 * c + 1], lo[4 * c + 2], lo[4 * c + 3]);
        *reinterpret_cast<uint4*>(tile + rh * 128 + chunk * 16) =
            make_uint4(hi[4 * c], hi[4 * c + 1], hi[4 * c + 2], hi[4 * c + 3]);
    }
}

struct GemmArgs {
    const uint4* qw;
    const __half* s;
    const uint32_t* z;
    __half* out;
    int M, K, N, zero_bias;
};

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Lane-uniform select of word (i & 3) of v, without dynamic register indexing.
__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) {
    const uint32_t lo = (i & 1) ? v.y : v.x, hi = (i & 1) ? v.w : v.z;
    return (i & 2) ? hi : lo;
}

__global__ void __launch_bounds__(kThreads, 1)
w4a16_gemm_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap qmap,
                  const GemmArgs a) {
    extern __shared__ unsigned char smem_raw[];
    // 1024-byte alignment for the swizzle atoms
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    // per ring slot: x tile, dequantised weight tile, packed weight tile
    auto xt = [&](int b) { return smem + b * kStageBytes; };
    auto wt = [&](int b) { return smem + b * kStageBytes + kXBytes; };
    auto qt = [&](int b) { return smem + b * kStageBytes + kXBytes + kWBytes; };
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);  // [kStages] x + packed tile landed
    uint64_t* wready = full + kStages;   // [kStages] weight tile dequantised (kDqThreads arrivals)
    uint64_t* done = wready + kStages;   // [kStages] MMAs of the stage complete (tcgen05.commit)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + kStages);
    volatile int* failed = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * kBN;
    const int K = a.K, G = K / 128, Gp = (G + 7) & ~7, zw = (G + 7) >> 3;
    const int nst = K / kBK;
    const int strips_total = (a.N + 15) / 16;
    constexpr int kIssuerWarp = kDqThreads / 32, kProducerWarp = kIssuerWarp + 1;

    if (warp == kIssuerWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kBN)
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
    pdl_trigger();

    if (warp == kProducerWarp) {
        // Stage j's x tile and packed weight tile (16 strips x 512 B, one
        // TMA each) go into slot j % kStages once the MMAs of stage
        // j - kStages have released it.  The weights never depend on the
        // previous kernel: the first slots are requested before the PDL wait.
        if (lane == 0) {
            auto request_q = [&](int j) {
                const int sj = j % kStages;
                mbar_expect_tx(&full[sj], kXBytes + kQBytes);
                tma_load_2d(qt(sj), &qmap, j * (kQBytes / kStrips / 4), n0 / 16, &full[sj]);
            };
            const int pre = nst < kStages ? nst : kStages;
            for (int j = 0; j < pre; ++j) request_q(j);
            pdl_wait();  // x may be the previous kernel's output
            int j = 0;
            for (; j < nst; ++j) {
                const int sj = j % kStages;
                if (j >= kStages) {
                    if (*failed || !mbar_wait(&done[sj], static_cast<uint32_t>((j - kStages) / kStages) & 1u)) {
                        *failed = 1;
                        break;
                    }
                    request_q(j);
                }
                tma_load_2d(xt(sj), &xmap, j * kBK, m0, &full[sj]);
            }
            // Drain (bounded): the newest copies of each slot must land before
            // the block frees its shared memory; older ones were consumed.
            const int last = j > pre ? j : pre;  // stages whose copies were requested
            for (int q = (last > kStages ? last - kStages : 0); q < last; ++q)
                if (!mbar_wait(&full[q % kStages], static_cast<uint32_t>(q / kStages) & 1u)) *failed = 1;
        }
        __syncwarp();
    } else if (warp == kIssuerWarp) {
        // Four tcgen05.mma (K = 16 each) per stage once its x tile has landed
        // and its weight tile is dequantised; one commit per stage frees the slot.
        if (lane == 0) {
            const uint32_t idesc = instr_desc_f16(kBM, kBN);
            int issued = 0;
            for (int i = 0; i < nst; ++i) {
                const int b = i % kStages;
                const uint32_t ph = static_cast<uint32_t>(i / kStages) & 1u;
                if (*failed || !mbar_wait(&full[b], ph) || !mbar_wait(&wready[b], ph)) {
                    *failed = 1;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < kBK / 16; ++kk) {
                    const uint64_t ad = smem_desc_sw128(smem_u32(xt(b)) + kk * 32);
                    const uint64_t bd = smem_desc_sw128(smem_u32(wt(b)) + kk * 32);
                    mma_f16(tmem, ad, bd, idesc, (i > 0 || kk > 0) ? 1u : 0u);
                }
                mma_commit(&done[b]);
                issued = i + 1;
            }
            // the last commit covers every MMA issued before it
            if (issued > 0 &&
                !mbar_wait(&done[(issued - 1) % kStages], static_cast<uint32_t>((issued - 1) / kStages) & 1u))
                *failed = 1;
            if (issued < nst) *failed = 1;
        }
        __syncwarp();
    } else {
        // Dequantising threads: strip `warp` of the tile, lane vector `lane`.
        // A landed slot implies its previous MMAs are done (the producer
        // waited for them), so one barrier per stage suffices.  Scales and
        // zeros of the thread's two columns come from global memory in
        // chunks of 8 groups (one 16-byte scale vector and one zero word per
        // column), the next chunk loaded while the current one is in use.
        const int sl = warp, g = lane >> 2, t = lane & 3;
        const int strip = (n0 >> 4) + sl;
        const bool have_strip = strip < strips_total;
        const int col = strip * 16 + g;
        const int nchunks = (G + 7) / 8;
        auto load_chunk = [&](int c, uint4& slo, uint4& shi, uint32_t& zlo, uint32_t& zhi) {
            if (have_strip && c < nchunks) {
                slo = __ldg(reinterpret_cast<const uint4*>(a.s + static_cast<size_t>(col) * Gp) + c);
                shi = __ldg(reinterpret_cast<const uint4*>(a.s + static_cast<size_t>(col + 8) * Gp) + c);
                zlo = __ldg(a.z + static_cast<size_t>(col) * zw + c);
                zhi = __ldg(a.z + static_cast<size_t>(col + 8) * zw + c);
            }
        };
        uint4 s_lo = make_uint4(0, 0, 0, 0), s_hi = s_lo, n_lo = s_lo, n_hi = s_lo;
        uint32_t z_lo = 0, z_hi = 0, nz_lo = 0, nz_hi = 0;
        load_chunk(0, s_lo, s_hi, z_lo, z_hi);
        load_chunk(1, n_lo, n_hi, nz_lo, nz_hi);
        for (int i = 0; i < nst; ++i) {
            const int b = i % kStages;
            const int grp = (i * kBK) / 128;
            if (i > 0 && (grp & 7) == 0 && (i & 1) == 0) {  // first stage of a new chunk
                s_lo = n_lo, s_hi = n_hi, z_lo = nz_lo, z_hi = nz_hi;
                load_chunk(grp / 8 + 1, n_lo, n_hi, nz_lo, nz_hi);
            }
            if (*failed || !mbar_wait(&full[b], static_cast<uint32_t>(i / kStages) & 1u)) {
                *failed = 1;
                break;
            }
            const uint4 v = *reinterpret_cast<const uint4*>(qt(b) + tid * 16);
            const int gi = grp & 7;
            const __half slo = __ushort_as_half(static_cast<unsigned short>(word_of(s_lo, gi >> 1) >> (16 * (gi & 1))));
            const __half shi = __ushort_as_half(static_cast<unsigned short>(word_of(s_hi, gi >> 1) >> (16 * (gi & 1))));
            const int zl = static_cast<int>((z_lo >> (4 * gi)) & 0xfu) + a.zero_bias;
            const int zh = static_cast<int>((z_hi >> (4 * gi)) & 0xfu) + a.zero_bias;
            dequant_store(v, wt(b), sl * 16 + g, t, zl, zh, slo, shi);
            // generic-proxy stores -> visible to the tensor core, then signal
            fence_proxy_async_smem();
            mbar_arrive(&wready[b]);
        }
    }
    if (warp != kProducerWarp) pdl_wait();  // every thread passes the wait before exit
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const bool acc_ready = !*failed;
    if (!acc_ready && tid == 0) atomicOr(&g_gemm_dev_error, kDevErrTimeout);
    if (acc_ready && warp < kIssuerWarp) {
        // warp w reads TMEM lanes 32 (w % 4) .. + 31 (= rows) and its share
        // of the columns; the issuer waited for the last commit
        constexpr int kColsPerWarp = kBN / (kIssuerWarp / 4);
        const int quarter = warp & 3, c0 = (warp >> 2) * kColsPerWarp;
        const int m = m0 + quarter * 32 + lane;
        const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll 1
        for (int c = c0; c < c0 + kColsPerWarp; c += 16) {
            float v[16];
            tmem_ld16(lane_addr + c, v);
            const int n = n0 + c;
            if (m < a.M && n < a.N) {
                uint32_t h[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) h[e] = h2_as_u32(__floats2half2_rn(v[2 * e], v[2 * e + 1]));
                __half* o = a.out + static_cast<size_t>(m) * a.N + n;
                if (n + 16 <= a.N && (a.N & 7) == 0) {
                    reinterpret_cast<uint4*>(o)[0] = make_uint4(h[0], h[1], h[2], h[3]);
                    reinterpret_cast<uint4*>(o)[1] = make_uint4(h[4], h[5], h[6], h[7]);
                } else {
#pragma unroll
                    for (int e = 0; e < 16; ++e)
                        if (n + e < a.N) o[e] = __float2half_rn(v[e]);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kIssuerWarp)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kBN) : "memory");
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static std::once_flag once;
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
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
    CUtensorMap map, qmap;
    {
        const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(M)};
        const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
        const cuuint32_t box[2] = {kBK, kBM};
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
    GemmArgs ga{static_cast<const uint4*>(qweight), static_cast<const __half*>(scales),
                static_cast<const uint32_t*>(zeros), static_cast<__half*>(out), static_cast<int>(M),
                static_cast<int>(K), static_cast<int>(N), zero_bias};
    const dim3 grid(static_cast<unsigned>((N + kBN - 1) / kBN), static_cast<unsigned>((M + kBM - 1) / kBM));
    return launch(w4a16_gemm_kernel, grid, dim3(kThreads), kSmemBytes, static_cast<cudaStream_t>(stream), map, qmap,
                  ga);
}

}  // extern "C"
