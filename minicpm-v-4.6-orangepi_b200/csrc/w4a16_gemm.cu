// W4A16 GEMM for batched decode / prefill (M >= 16) on the 5th-generation
// tensor cores: tcgen05.mma with the fp32 accumulator in tensor memory.
//
// Reference counterpart: the reference has no quantized GEMM for M > 1 -
// prefill goes through matmul_b_transposed's dense aclnnMm / K-tiling path
// (src/csrc/lib/ops.cpp:215-322) and matmul_w4a16 is M=1 only (ops.cpp:1048).
// This kernel serves the same mcv-int4 weights as the decode GEMV.
//
// One block computes a 128 (rows of x) x 128 (output columns) tile:
//  * x tiles [128 rows x 64 k] arrive by TMA (cp.async.bulk.tensor, 128-byte
//    swizzle; rows past M are zero-filled by the copy engine);
//  * 256 dequantising threads each fetch (cp.async, five stages ahead) and
//    dequantise one 16-byte lane vector of the mcv-int4 layout per stage -
//    16 consecutive k of two columns - to fp16 (q - zero) * scale, store it
//    in the same 128-byte-swizzled K-major layout and arrive on the stage's
//    "weight ready" mbarrier;
//  * one thread of a ninth warp requests the x tiles (four stages ahead) and
//    issues four tcgen05.mma.kind::f16 (M=128, N=128, K=16) per 64-k stage
//    once both operands of the stage are ready, committing them to the
//    stage's "done" mbarrier, which frees the 5-deep tile ring slot.  The
//    roles meet only on mbarriers: no block-wide barrier inside the k loop;
//  * the epilogue (warps 0-3) reads the accumulator with tcgen05.ld (warp w
//    owns TMEM lanes 32w..32w+31 = rows) and writes fp16.
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
constexpr int kBN = 128;         // output columns per block (MMA N)
constexpr int kBK = 64;          // k per stage: one 128-byte swizzle row
constexpr int kDqThreads = 256;  // dequantising threads: one lane vector of the tile each
constexpr int kThreads = kDqThreads + 32;  // + one warp that issues the TMA copies and the MMAs
constexpr int kTileBytes = kBM * kBK * 2;  // 16 KB (both operands)
constexpr int kStages = 5;                 // x / weight tile ring depth
constexpr int kRawStages = 6;              // per-thread raw operand ring depth
constexpr int kRawBytes = kDqThreads * 32; // per raw stage: each thread's int4 vector, scales, zeros
constexpr int kSmemBytes = kStages * 2 * kTileBytes + kRawStages * kRawBytes + 1024 + 512;

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

__global__ void __launch_bounds__(kThreads, 1)
w4a16_gemm_kernel(const __grid_constant__ CUtensorMap xmap, const GemmArgs a) {
    extern __shared__ unsigned char smem_raw[];
    // 1024-byte alignment for the swizzle atoms
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    // x tiles and dequantised weight tiles (kStages each), then the raw ring
    // where every dequantising thread lands its own int4 vector, scales and zeros
    auto xt = [&](int b) { return smem + b * kTileBytes; };
    auto wt = [&](int b) { return smem + (kStages + b) * kTileBytes; };
    auto raw = [&](int b) { return smem + 2 * kStages * kTileBytes + b * kRawBytes; };
    uint64_t* xfull = reinterpret_cast<uint64_t*>(smem + 2 * kStages * kTileBytes + kRawStages * kRawBytes);
    uint64_t* wready = xfull + kStages;  // [kStages] weight tile dequantised (kDqThreads arrivals)
    uint64_t* done = wready + kStages;   // [kStages] MMAs of the stage complete (tcgen05.commit)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + kStages);
    volatile int* failed = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * kBN;
    const int K = a.K, G = K / 128, Gp = (G + 7) & ~7, zw = (G + 7) >> 3;
    const int nst = K / kBK;
    const int strips_total = (a.N + 15) / 16;
    constexpr int kIssuerWarp = kDqThreads / 32;

    if (warp == kIssuerWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kBN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&xfull[i], 1);
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
    pdl_wait();  // x may be the previous kernel's output

    if (warp == kIssuerWarp) {
        // Producer of x tiles and issuer of the MMAs.  Stage j's x tile goes
        // into slot j % kStages once the MMAs of stage j - kStages are done;
        // the refill for stage i + kStages - 1 is requested right after the
        // MMAs of stage i are queued, so the tensor pipe always holds queued
        // work while this thread waits.
        if (lane == 0) {
            const uint32_t idesc = instr_desc_f16(kBM, kBN);
            auto request_x = [&](int j) {
                const int sj = j % kStages;
                mbar_expect_tx(&xfull[sj], kTileBytes);
                tma_load_2d(xt(sj), &xmap, j * kBK, m0, &xfull[sj]);
            };
            int x_issued = 0, mma_issued = 0;
            for (; x_issued < kStages - 1 && x_issued < nst; ++x_issued) request_x(x_issued);
            for (int i = 0; i < nst; ++i) {
                const int b = i % kStages;
                const uint32_t ph = static_cast<uint32_t>(i / kStages) & 1u;
                if (*failed || !mbar_wait(&xfull[b], ph) || !mbar_wait(&wready[b], ph)) {
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
                mma_issued = i + 1;
                if (x_issued < nst) {
                    // slot of stage x_issued = i + kStages - 1 was used by stage i - 1
                    if (i >= 1 && !mbar_wait(&done[(i - 1) % kStages], static_cast<uint32_t>((i - 1) / kStages) & 1u)) {
                        *failed = 1;
                        break;
                    }
                    request_x(x_issued++);
                }
            }
            // Drain (bounded): outstanding x copies and the issued MMAs must
            // land before the block can free its shared and tensor memory.
            for (int j = mma_issued; j < x_issued; ++j)
                if (!mbar_wait(&xfull[j % kStages], static_cast<uint32_t>(j / kStages) & 1u)) *failed = 1;
            if (mma_issued > 0 &&
                !mbar_wait(&done[(mma_issued - 1) % kStages], static_cast<uint32_t>((mma_issued - 1) / kStages) & 1u))
                *failed = 1;
            if (mma_issued < nst) *failed = 1;
        }
        __syncwarp();
    } else {
        // Dequantising threads: strip tid / 32 of the tile, lane vector lane.
        // Each thread fetches its own raw operands kRawStages - 1 stages
        // ahead (one cp.async group per stage) and reads them back itself, so
        // the raw ring needs no barrier; the weight tile slot is reused once
        // the MMAs of stage i - kStages are done.
        const int sl = warp, g = lane >> 2, t = lane & 3;
        const int strip = (n0 >> 4) + sl;
        const bool have_strip = strip < strips_total;
        const int col = strip * 16 + g;
        auto request_raw = [&](int j) {
            if (have_strip && j < nst) {
                unsigned char* r = raw(j % kRawStages) + tid * 32;
                const int grp = (j * kBK) / 128;
                cp_async16(r, a.qw + (static_cast<size_t>(strip) * (K / 64) + j) * 32 + lane);
                cp_async4(r + 16, a.s + static_cast<size_t>(col) * Gp + (grp & ~1));
                cp_async4(r + 20, a.s + static_cast<size_t>(col + 8) * Gp + (grp & ~1));
                cp_async4(r + 24, a.z + static_cast<size_t>(col) * zw + (grp >> 3));
                cp_async4(r + 28, a.z + static_cast<size_t>(col + 8) * zw + (grp >> 3));
            }
            cp_async_commit();  // one group per stage, empty past the end
        };
#pragma unroll 1
        for (int j = 0; j < kRawStages - 1; ++j) request_raw(j);
        for (int i = 0; i < nst; ++i) {
            const int b = i % kStages;
            request_raw(i + kRawStages - 1);
            cp_async_wait<kRawStages - 1>();  // this stage's group has landed
            if (*failed ||
                (i >= kStages && !mbar_wait(&done[b], (static_cast<uint32_t>(i / kStages) & 1u) ^ 1u))) {
                *failed = 1;
                break;
            }
            const unsigned char* r = raw(i % kRawStages) + tid * 32;
            const int grp = (i * kBK) / 128;
            uint4 v = make_uint4(0, 0, 0, 0);
            int zl = 0, zh = 0;
            __half slo = __ushort_as_half(0), shi = __ushort_as_half(0);
            if (have_strip) {
                v = *reinterpret_cast<const uint4*>(r);
                const uint32_t sp_lo = *reinterpret_cast<const uint32_t*>(r + 16);
                const uint32_t sp_hi = *reinterpret_cast<const uint32_t*>(r + 20);
                slo = __ushort_as_half(static_cast<unsigned short>(sp_lo >> (16 * (grp & 1))));
                shi = __ushort_as_half(static_cast<unsigned short>(sp_hi >> (16 * (grp & 1))));
                zl = static_cast<int>((*reinterpret_cast<const uint32_t*>(r + 24) >> (4 * (grp & 7))) & 0xfu) + a.zero_bias;
                zh = static_cast<int>((*reinterpret_cast<const uint32_t*>(r + 28) >> (4 * (grp & 7))) & 0xfu) + a.zero_bias;
            }
            dequant_store(v, wt(b), sl * 16 + g, t, zl, zh, slo, shi);
            // generic-proxy stores -> visible to the tensor core, then signal
            fence_proxy_async_smem();
            mbar_arrive(&wready[b]);
        }
        cp_async_wait<0>();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const bool acc_ready = !*failed;
    if (!acc_ready && tid == 0) atomicOr(&g_gemm_dev_error, kDevErrTimeout);
    if (acc_ready && warp < 4) {
        // the issuer waited for the last commit, which covers every MMA
        const int m = m0 + warp * 32 + lane;
        const uint32_t lane_addr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
#pragma unroll 1
        for (int c = 0; c < kBN; c += 16) {
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
    if ((reinterpret_cast<uintptr_t>(scales) & 3u) || (reinterpret_cast<uintptr_t>(zeros) & 3u) ||
        (reinterpret_cast<uintptr_t>(out) & 1u))
        return fail(MCV_ERR_ALIGN, "w4a16_gemm: misaligned scales, zeros or out");
    if (zero_bias < 0 || zero_bias > 1) return fail(MCV_ERR_VALUE, "w4a16_gemm: zero_bias must be 0 or 1");
    auto enc = encode_fn();
    if (!enc) return fail(MCV_ERR_CUDA, "w4a16_gemm: cuTensorMapEncodeTiled unavailable");
    CUtensorMap map;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(M)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
    const cuuint32_t box[2] = {kBK, kBM};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(x), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(MCV_ERR_CUDA, "w4a16_gemm: cuTensorMapEncodeTiled failed");
    cudaError_t e = cudaFuncSetAttribute(w4a16_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(w4a16_gemm)");
    GemmArgs ga{static_cast<const uint4*>(qweight), static_cast<const __half*>(scales),
                static_cast<const uint32_t*>(zeros), static_cast<__half*>(out), static_cast<int>(M),
                static_cast<int>(K), static_cast<int>(N), zero_bias};
    const dim3 grid(static_cast<unsigned>((N + kBN - 1) / kBN), static_cast<unsigned>((M + kBM - 1) / kBM));
    return launch(w4a16_gemm_kernel, grid, dim3(kThreads), kSmemBytes, static_cast<cudaStream_t>(stream), map, ga);
}

}  // extern "C"
