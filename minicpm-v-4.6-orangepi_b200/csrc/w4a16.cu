// W4A16 GEMV for decode (M = 1..8) over the mcv-int4 weight layout, plus the
// load-time host repackers from GPTQ / AWQ / the reference's tile layout.
//
// Reference behaviour replaced: matmul_w4a16 (src/csrc/lib/ops.cpp:1030-1095)
// and its AscendC kernel op_kernel/matmul_w4a16_custom.cpp:64-127, which
// computes out[n] = sum_g s[g,n] * sum_{k in g} x[k] * (q-z)[k,n] on 8 AICore
// blocks with fp16 accumulation.  Here the same sum is accumulated in fp32.
//
// Kernel design (HBM-bound; a 1024x3584 weight is 1.84 MB of int4):
//  * one warp owns CPW output columns; lane l streams 16-byte chunks
//    (32 consecutive k of one column) c = l, l+32, ... so each warp-wide load
//    instruction reads 512 contiguous bytes;
//  * every weight, scale and zero load of the thread is issued up front,
//    before griddepcontrol.wait, so under programmatic dependent launch the
//    weight stream of this GEMV overlaps the previous kernel's tail;
//  * int4 -> fp16 with the exponent-bias ("magic number") conversion
//    described for FasterTransformer-style mixed-input GEMMs (Kim et al.,
//    "Who Says Elephants Can't Run", 2022; Frantar et al., MARLIN, 2024):
//    OR-ing a nibble into the mantissa of fp16 1024.0 gives 1024+q exactly,
//    and one HSUB2 / HFMA2 removes 1024+zero, leaving (q - zero) exactly;
//  * products are accumulated in fp32 by the sm_100 mixed-precision FMA
//    (fp16 x fp16 + fp32), per 32-weight chunk, then scaled by the group
//    scale; a 5-step xor-shuffle reduces over the warp.
#include <algorithm>
#include <cstring>
#include <vector>

#include "common.cuh"

namespace mcv {
namespace {

constexpr int kWarps = 4;
constexpr int kCpw = 2;  // columns per warp
constexpr int kSlot[8] = {0, 4, 1, 5, 2, 6, 3, 7};

// Four half2 values (q - z) for k = 8j..8j+7 of one word (see kSlot).
__device__ __forceinline__ void dequant8(uint32_t w, __half2 zlo, __half2 zhi, uint32_t h[4]) {
    constexpr uint32_t kMagic = 0x64006400u;  // fp16 1024.0 in both lanes
    const __half2 inv16 = __halves2half2(__ushort_as_half(0x2c00), __ushort_as_half(0x2c00));
    const uint32_t w8 = w >> 8;
    const __half2 a = u32_as_h2(lop3_and_or(w, 0x000f000fu, kMagic));
    const __half2 b = u32_as_h2(lop3_and_or(w, 0x00f000f0u, kMagic));
    const __half2 c = u32_as_h2(lop3_and_or(w8, 0x000f000fu, kMagic));
    const __half2 d = u32_as_h2(lop3_and_or(w8, 0x00f000f0u, kMagic));
    h[0] = h2_as_u32(__hsub2(a, zlo));
    h[1] = h2_as_u32(__hfma2(b, inv16, zhi));
    h[2] = h2_as_u32(__hsub2(c, zlo));
    h[3] = h2_as_u32(__hfma2(d, inv16, zhi));
}

template <int M, int KCH>
__global__ void __launch_bounds__(kWarps * 32)
w4a16_gemv_kernel(const __half* __restrict__ x, const uint32_t* __restrict__ qw,
                  const __half* __restrict__ scales, const uint32_t* __restrict__ zeros,
                  int zero_bias, __half* __restrict__ out, int K, int N, int group) {
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int n0 = (blockIdx.x * kWarps + warp) * kCpw;
    const int chunks = K >> 5;
    const int kwords = K >> 3;
    const int G = K / group;
    const int zwords = (G + 7) >> 3;

    // ---- prefetch everything that does not depend on the previous kernel ----
    uint4 wv[kCpw][KCH];
    float sc[kCpw][KCH];
    int zq[kCpw][KCH];
#pragma unroll
    for (int j = 0; j < kCpw; ++j) {
        const int n = n0 + j;
#pragma unroll
        for (int i = 0; i < KCH; ++i) {
            const int c = lane + 32 * i;
            wv[j][i] = make_uint4(0, 0, 0, 0);
            sc[j][i] = 0.0f;
            zq[j][i] = 0;
            if (n < N && c < chunks) {
                wv[j][i] = ld_stream(qw + static_cast<size_t>(n) * kwords + c * 4);
                const int g = (c * 32) / group;
                sc[j][i] = __half2float(scales[static_cast<size_t>(n) * G + g]);
                const uint32_t zw = zeros[static_cast<size_t>(n) * zwords + (g >> 3)];
                zq[j][i] = static_cast<int>((zw >> (4 * (g & 7))) & 0xfu) + zero_bias;
            }
        }
    }
    pdl_trigger();
    pdl_wait();

    float acc[kCpw][M];
#pragma unroll
    for (int j = 0; j < kCpw; ++j)
#pragma unroll
        for (int m = 0; m < M; ++m) acc[j][m] = 0.0f;

#pragma unroll
    for (int i = 0; i < KCH; ++i) {
        const int c = lane + 32 * i;
        if (c >= chunks) break;
        float pa[kCpw][M], pb[kCpw][M];
#pragma unroll
        for (int j = 0; j < kCpw; ++j)
#pragma unroll
            for (int m = 0; m < M; ++m) pa[j][m] = pb[j][m] = 0.0f;
        __half2 zlo[kCpw], zhi[kCpw];
#pragma unroll
        for (int j = 0; j < kCpw; ++j) {
            const __half z1 = __int2half_rn(1024 + zq[j][i]);
            const __half z2 = __int2half_rn(-(64 + zq[j][i]));
            zlo[j] = __halves2half2(z1, z1);
            zhi[j] = __halves2half2(z2, z2);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            uint4 xv[M];
#pragma unroll
            for (int m = 0; m < M; ++m)
                xv[m] = *reinterpret_cast<const uint4*>(x + static_cast<size_t>(m) * K + c * 32 + q * 8);
#pragma unroll
            for (int j = 0; j < kCpw; ++j) {
                const uint32_t w = q == 0 ? wv[j][i].x : q == 1 ? wv[j][i].y : q == 2 ? wv[j][i].z : wv[j][i].w;
                uint32_t h[4];
                dequant8(w, zlo[j], zhi[j], h);
#pragma unroll
                for (int m = 0; m < M; ++m) {
                    fma2_f16_f32(pa[j][m], pb[j][m], h[0], xv[m].x);
                    fma2_f16_f32(pa[j][m], pb[j][m], h[1], xv[m].y);
                    fma2_f16_f32(pa[j][m], pb[j][m], h[2], xv[m].z);
                    fma2_f16_f32(pa[j][m], pb[j][m], h[3], xv[m].w);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < kCpw; ++j)
#pragma unroll
            for (int m = 0; m < M; ++m) acc[j][m] = fmaf(pa[j][m] + pb[j][m], sc[j][i], acc[j][m]);
    }

#pragma unroll
    for (int j = 0; j < kCpw; ++j)
#pragma unroll
        for (int m = 0; m < M; ++m) {
            const float v = warp_sum(acc[j][m]);
            const int n = n0 + j;
            if (lane == ((j * M + m) & 31) && n < N)
                out[static_cast<size_t>(m) * N + n] = __float2half_rn(v);
        }
}

template <int M>
int dispatch_k(int kch, const __half* x, const uint32_t* qw, const __half* s, const uint32_t* z,
               int zb, __half* out, int K, int N, int group, cudaStream_t st) {
    const dim3 grid((N + kWarps * kCpw - 1) / (kWarps * kCpw));
    const dim3 block(kWarps * 32);
    switch (kch) {
        case 1: return launch(w4a16_gemv_kernel<M, 1>, grid, block, 0, st, x, qw, s, z, zb, out, K, N, group);
        case 2: return launch(w4a16_gemv_kernel<M, 2>, grid, block, 0, st, x, qw, s, z, zb, out, K, N, group);
        case 4: return launch(w4a16_gemv_kernel<M, 4>, grid, block, 0, st, x, qw, s, z, zb, out, K, N, group);
        case 8: return launch(w4a16_gemv_kernel<M, 8>, grid, block, 0, st, x, qw, s, z, zb, out, K, N, group);
        default: return fail(MCV_ERR_SHAPE, "w4a16_gemv: K above 8192 unsupported");
    }
}

int check_layout_dims(int64_t K, int64_t N, int64_t group) {
    if (K <= 0 || N <= 0 || group <= 0) return fail(MCV_ERR_SHAPE, "w4a16: K, N, group must be positive");
    if (group % 32 != 0) return fail(MCV_ERR_SHAPE, "w4a16: group must be a multiple of 32");
    if (K % group != 0) return fail(MCV_ERR_SHAPE, "w4a16: K must be a multiple of group");
    if (K > (1 << 24) || N > (1 << 30)) return fail(MCV_ERR_SHAPE, "w4a16: dimension too large");
    return MCV_OK;
}

// Writes the three mcv-int4 arrays from a logical accessor q(k,n) (0..15)
// and zero z(g,n) (0..15).
template <typename QF, typename ZF>
void pack_layout(QF q, ZF z, const uint16_t* scales_gn, int64_t K, int64_t N, int64_t group,
                 uint32_t* qw, uint16_t* sc, uint32_t* zw) {
    const int64_t G = K / group;
    const int64_t kwords = K / 8;
    const int64_t zwords = (G + 7) / 8;
    for (int64_t n = 0; n < N; ++n) {
        for (int64_t j = 0; j < kwords; ++j) {
            uint32_t word = 0;
            for (int i = 0; i < 8; ++i)
                word |= (static_cast<uint32_t>(q(8 * j + i, n)) & 0xfu) << (4 * kSlot[i]);
            qw[n * kwords + j] = word;
        }
        for (int64_t g = 0; g < G; ++g) sc[n * G + g] = scales_gn[g * N + n];
        for (int64_t t = 0; t < zwords; ++t) zw[n * zwords + t] = 0;
        for (int64_t g = 0; g < G; ++g)
            zw[n * zwords + g / 8] |= (static_cast<uint32_t>(z(g, n)) & 0xfu) << (4 * (g % 8));
    }
}

}  // namespace
}  // namespace mcv

using namespace mcv;

extern "C" {

int mcv_w4a16_layout_bytes(int64_t K, int64_t N, int64_t group, size_t* qb, size_t* sb, size_t* zb) {
    int st = check_layout_dims(K, N, group);
    if (st) return st;
    const int64_t G = K / group;
    if (qb) *qb = static_cast<size_t>(N) * (K / 8) * 4;
    if (sb) *sb = static_cast<size_t>(N) * G * 2;
    if (zb) *zb = static_cast<size_t>(N) * ((G + 7) / 8) * 4;
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
    if (!x || !qweight || !scales || !zeros || !out) return fail(MCV_ERR_NULL, "w4a16_gemv: null pointer");
    int st = check_layout_dims(K, N, group);
    if (st) return st;
    if (M < 1 || M > 8) return fail(MCV_ERR_SHAPE, "w4a16_gemv: M must be 1..8");
    if (!aligned16(qweight) || !aligned16(x)) return fail(MCV_ERR_ALIGN, "w4a16_gemv: x and qweight must be 16-byte aligned");
    if (zero_bias < 0 || zero_bias > 1) return fail(MCV_ERR_VALUE, "w4a16_gemv: zero_bias must be 0 or 1");
    const int chunks_per_lane = static_cast<int>((K / 32 + 31) / 32);
    int kch = 1;
    while (kch < chunks_per_lane) kch *= 2;
    auto* xs = static_cast<const __half*>(x);
    auto* qw = static_cast<const uint32_t*>(qweight);
    auto* sc = static_cast<const __half*>(scales);
    auto* zw = static_cast<const uint32_t*>(zeros);
    auto* o = static_cast<__half*>(out);
    auto s = static_cast<cudaStream_t>(stream);
    const int k = static_cast<int>(K), n = static_cast<int>(N), g = static_cast<int>(group);
    switch (M) {
        case 1: return dispatch_k<1>(kch, xs, qw, sc, zw, zero_bias, o, k, n, g, s);
        case 2: return dispatch_k<2>(kch, xs, qw, sc, zw, zero_bias, o, k, n, g, s);
        case 3: return dispatch_k<3>(kch, xs, qw, sc, zw, zero_bias, o, k, n, g, s);
        case 4: return dispatch_k<4>(kch, xs, qw, sc, zw, zero_bias, o, k, n, g, s);
        case 5: return dispatch_k<5>(kch, xs, qw, sc, zw, zero_bias, o, k, n, g, s);
        case 6: return dispatch_k<6>(kch, xs, qw, sc, zw, zero_bias, o, k, n, g, s);
        case 7: return dispatch_k<7>(kch, xs, qw, sc, zw, zero_bias, o, k, n, g, s);
        default: return dispatch_k<8>(kch, xs, qw, sc, zw, zero_bias, o, k, n, g, s);
    }
}

}  // extern "C"
