// W8A8 decode path: per-token int8 activation quantization, int8 x int8 ->
// int32 GEMV (bit-exact), per-channel x per-token dequant to fp16, and the
// per-channel weight quantizer.
//
// Reference behaviour replaced (src/csrc/lib/ops.cpp:1097-1210 and the
// AscendC kernels it launches):
//  * w8a8_quantize  (op_kernel/w8a8_quantize_custom.cpp:25-41): scale =
//    max|x|/127 in fp32, clamped to >= 1e-8, inv = 1/scale, q = (int)(clamp(
//    x*inv, -128, 127) +/- 0.5), scale stored as fp16.  Done per row here.
//  * matmul_w8a8_i32 (op_kernel/matmul_w8a8_i32_custom.cpp): exact int32.
//  * w8a8_dequant   (op_kernel/w8a8_dequant_custom.cpp:52-59): fp16 RN of
//    (float(acc) * float(w_scale)) * float(x_scale).
//  * quantize_dense_weight_w8a8 (src/csrc/lib/quantized_weight.cpp:231-268).
// Every floating-point step uses an explicitly rounded intrinsic
// (__fdiv_rn, __fmul_rn, __fadd_rn, __float2half_rn) so results are
// bit-identical to the fp32 C restatement of those formulas.
//
// Fast layout: weights int8 [N][K] (K contiguous).  One warp owns two output
// columns; lane l loads 16-byte chunks (16 k) l, l+32, ...; DP4A multiplies
// four int8 pairs per instruction; a 5-step shuffle sums the warp.  The fused
// kernel quantizes x inside every block (x is a few KB in L2), prefetches its
// weights before the PDL wait, and writes fp16 outputs directly.
#include "common.cuh"
#include "w8a8_quant.cuh"

namespace mcv {
namespace {

constexpr int kQThreads = 256;
constexpr int kW8Warps = 8;
constexpr int kW8Cpw = 2;

// Block-wide max of non-negative floats (bit pattern order == value order).
__device__ __forceinline__ float block_max_nonneg(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float r = 0.0f;
    for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) r = fmaxf(r, red[i]);
    return r;
}

// ---- standalone per-row quantizer --------------------------------------------
__global__ void __launch_bounds__(kQThreads)
quantize_rows_kernel(const __half* __restrict__ x, int8_t* __restrict__ xq, __half* __restrict__ xs, int K) {
    __shared__ float red[kQThreads / 32];
    pdl_trigger();
    pdl_wait();
    const __half* row = x + static_cast<int64_t>(blockIdx.x) * K;
    float m = 0.0f;
    for (int i = threadIdx.x; i < K; i += kQThreads) m = fmaxf(m, fabsf(__half2float(row[i])));
    const float max_abs = block_max_nonneg(m, red);
    const float scale = scale_from_absmax(max_abs);
    const float inv = __fdiv_rn(1.0f, scale);
    for (int i = threadIdx.x; i < K; i += kQThreads)
        xq[static_cast<int64_t>(blockIdx.x) * K + i] = quant_act(__half2float(row[i]), inv);
    if (threadIdx.x == 0) xs[blockIdx.x] = __float2half_rn(scale);
}

// ---- int8 GEMV over [N][K] weights, optionally fused ----------------------------
struct W8Args {
    const void* x;          // FUSED: fp16 [M][K]; else int8 [M][K]
    const int8_t* w;        // [N][K]
    const __half* w_scale;  // [N] (FUSED)
    __half* out;            // [M][N] (FUSED)
    int32_t* acc;           // [M][N] (optional when FUSED)
    int8_t* xq_out;         // [M][K] (optional, FUSED, written by block 0)
    __half* xs_out;         // [M]    (optional, FUSED, written by block 0)
    const __half* xs_in;    // [M] scales of an int8 x (not FUSED): with w_scale and out, dequantize in the epilogue
    int K;
    int N;
};

// Independent GEMVs of one launch (same K and M): problem i owns blocks
// [block_begin[i], block_begin[i + 1]).  A single GEMV is a group of one.
constexpr int kW8MaxProblems = 16;
struct W8Group {
    int count;
    int block_begin[kW8MaxProblems + 1];
    W8Args p[kW8MaxProblems];
};

__device__ __forceinline__ int w8_problem_of(const W8Group& gr, int block) {
    int pi = 0;
    while (pi + 1 < gr.count && block >= gr.block_begin[pi + 1]) ++pi;
    return pi;
}

// Fused prologue: quantizes the M activation rows of a.x into xq8 (row
// stride `stride` bytes) and their fp16-rounded scales into xscale_s, per
// row exactly as w8a8_quantize; block 0 also writes the optional copies.
template <int M, int VPT>
__device__ __forceinline__ void fused_quantize_x(const W8Args& a, int8_t* xq8, int stride, float* xscale_s) {
    quantize_rows_to_smem<M, VPT, kW8Warps * 32>(static_cast<const __half*>(a.x), a.K, xq8, stride, xscale_s,
                                                 a.xq_out, a.xs_out);
}

template <int M, int KCH, bool FUSED>
__global__ void __launch_bounds__(kW8Warps * 32)
w8_rows_kernel(const __grid_constant__ W8Group gr) {
    extern __shared__ uint4 xq_s[];  // int8 x as [M][K/16] 16-byte chunks
    __shared__ float xscale_s[M];
    const int pi = w8_problem_of(gr, static_cast<int>(blockIdx.x));
    const W8Args& a = gr.p[pi];
    const int bid = static_cast<int>(blockIdx.x) - gr.block_begin[pi];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int n0 = (bid * kW8Warps + warp) * kW8Cpw;
    const int chunks = a.K >> 4;

    uint4 wv[kW8Cpw][KCH];
    float wsc[kW8Cpw];
#pragma unroll
    for (int j = 0; j < kW8Cpw; ++j) {
        const int n = n0 + j;
        wsc[j] = 0.0f;
#pragma unroll
        for (int i = 0; i < KCH; ++i) {
            const int c = lane + 32 * i;
            wv[j][i] = make_uint4(0, 0, 0, 0);
            if (n < a.N && c < chunks) wv[j][i] = ld_stream(a.w + static_cast<int64_t>(n) * a.K + c * 16);
        }
        if (FUSED || a.xs_in) {
            if (n < a.N) wsc[j] = __half2float(a.w_scale[n]);
        }
    }
    pdl_trigger();
    pdl_wait();

    int8_t* xq8 = reinterpret_cast<int8_t*>(xq_s);
    if constexpr (FUSED) {
        fused_quantize_x<M, (KCH + 3) / 4>(a, xq8, a.K, xscale_s);
    } else {
        const uint4* src = static_cast<const uint4*>(a.x);
        for (int idx = threadIdx.x; idx < M * chunks; idx += kW8Warps * 32) xq_s[idx] = src[idx];
        if (a.xs_in && threadIdx.x < M) xscale_s[threadIdx.x] = __half2float(a.xs_in[threadIdx.x]);
    }
    __syncthreads();

    int acc[kW8Cpw][M];
#pragma unroll
    for (int j = 0; j < kW8Cpw; ++j)
#pragma unroll
        for (int m = 0; m < M; ++m) acc[j][m] = 0;
#pragma unroll
    for (int i = 0; i < KCH; ++i) {
        const int c = lane + 32 * i;
        if (c < chunks) {
#pragma unroll
            for (int m = 0; m < M; ++m) {
                const uint4 xv = xq_s[m * chunks + c];
#pragma unroll
                for (int j = 0; j < kW8Cpw; ++j) {
                    int s = acc[j][m];
                    s = __dp4a(static_cast<int>(wv[j][i].x), static_cast<int>(xv.x), s);
                    s = __dp4a(static_cast<int>(wv[j][i].y), static_cast<int>(xv.y), s);
                    s = __dp4a(static_cast<int>(wv[j][i].z), static_cast<int>(xv.z), s);
                    s = __dp4a(static_cast<int>(wv[j][i].w), static_cast<int>(xv.w), s);
                    acc[j][m] = s;
                }
            }
        }
    }
#pragma unroll
    for (int j = 0; j < kW8Cpw; ++j)
#pragma unroll
        for (int m = 0; m < M; ++m) {
            int v = acc[j][m];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            const int n = n0 + j;
            if (lane == ((j * M + m) & 31) && n < a.N) {
                const int64_t o = static_cast<int64_t>(m) * a.N + n;
                if (a.acc) a.acc[o] = v;
                if (FUSED || a.xs_in) {
                    const float d = __fmul_rn(__fmul_rn(__int2float_rn(v), wsc[j]), xscale_s[m]);
                    a.out[o] = __float2half_rn(d);
                }
            }
        }
}

// ---- int8 GEMV over [N][K] weights on the integer tensor cores ----------------
// mma.sync m16n8k32 s8 x s8 -> s32: a block owns 16 weight rows (the MMA's M)
// and its 8 warps split K in 64-k blocks.  Lane (g = lane/4, t = lane%4)
// loads 16 bytes of rows g and g+8 at k = 64 kb + 16 t; k is permuted
// identically for weights and activations inside each 64-k block (an integer
// dot product does not depend on the order of k), so those bytes are directly
// the A fragments of two MMAs and one 16-byte shared-memory load of x row g is
// the matching B fragments.  The activation rows are the MMA's N (M <= 8).
// int32 sums are exact in any order: the cross-warp sum in shared memory and
// the dequant epilogue give the DP4A kernel's bits.
constexpr int kXqPad = 16;  // bytes between x rows in shared memory (bank spread)

__device__ __forceinline__ void mma_s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <int M, int KB, bool FUSED>
__global__ void __launch_bounds__(kW8Warps * 32)
w8_mma_kernel(const __grid_constant__ W8Group gr) {
    extern __shared__ uint4 xq_s[];  // int8 x, M rows of K + kXqPad bytes
    __shared__ float xscale_s[M];
    __shared__ int4 red[kW8Warps][32];
    const int pi = w8_problem_of(gr, static_cast<int>(blockIdx.x));
    const W8Args& a = gr.p[pi];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int n0 = (static_cast<int>(blockIdx.x) - gr.block_begin[pi]) * 16;
    const int K = a.K, nkb = (K + 63) / 64, stride = K + kXqPad;
    const bool lo_ok = n0 + g < a.N, hi_ok = n0 + g + 8 < a.N;

    // this warp's weight bytes of rows g and g+8 (all before the PDL wait)
    uint4 wlo[KB], whi[KB];
#pragma unroll
    for (int j = 0; j < KB; ++j) {
        const int kb = warp + j * kW8Warps;
        const int k = kb * 64 + 16 * t;
        wlo[j] = whi[j] = make_uint4(0, 0, 0, 0);
        if (kb < nkb && k < K) {
            if (lo_ok) wlo[j] = ld_stream(a.w + static_cast<int64_t>(n0 + g) * K + k);
            if (hi_ok) whi[j] = ld_stream(a.w + static_cast<int64_t>(n0 + g + 8) * K + k);
        }
    }
    float wsc_lo = 0.0f, wsc_hi = 0.0f;
    if (FUSED || a.xs_in) {
        if (lo_ok) wsc_lo = __half2float(a.w_scale[n0 + g]);
        if (hi_ok) wsc_hi = __half2float(a.w_scale[n0 + g + 8]);
    }
    pdl_trigger();
    pdl_wait();

    int8_t* xq8 = reinterpret_cast<int8_t*>(xq_s);
    if constexpr (FUSED) {
        fused_quantize_x<M, (KB + 3) / 4>(a, xq8, stride, xscale_s);
    } else {
        const uint4* src = static_cast<const uint4*>(a.x);
        const int cpr = K >> 4;  // 16-byte chunks per row
        for (int idx = threadIdx.x; idx < M * cpr; idx += kW8Warps * 32) {
            const int m = idx / cpr, c = idx - m * cpr;
            *reinterpret_cast<uint4*>(xq8 + m * stride + c * 16) = src[idx];
        }
        if (a.xs_in && threadIdx.x < M) xscale_s[threadIdx.x] = __half2float(a.xs_in[threadIdx.x]);
    }
    __syncthreads();

    int d[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < KB; ++j) {
        const int kb = warp + j * kW8Warps;
        const int k = kb * 64 + 16 * t;
        if (kb >= nkb) break;
        uint4 xv = make_uint4(0, 0, 0, 0);
        if (g < M && k < K) xv = *reinterpret_cast<const uint4*>(xq8 + g * stride + k);
        mma_s8(d, wlo[j].x, whi[j].x, wlo[j].y, whi[j].y, xv.x, xv.y);
        mma_s8(d, wlo[j].z, whi[j].z, wlo[j].w, whi[j].w, xv.z, xv.w);
    }
    red[warp][lane] = make_int4(d[0], d[1], d[2], d[3]);
    __syncthreads();
    if (warp == 0) {
        int4 sum = red[0][lane];
#pragma unroll
        for (int w = 1; w < kW8Warps; ++w) {
            const int4 r = red[w][lane];
            sum.x += r.x, sum.y += r.y, sum.z += r.z, sum.w += r.w;
        }
        // D rows g / g+8 = weight rows n0+g / n0+g+8, columns 2t / 2t+1 = activation rows
        const int vals[4] = {sum.x, sum.y, sum.z, sum.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int m = 2 * t + (e & 1);
            const int n = n0 + g + 8 * (e >> 1);
            if (m >= M || n >= a.N) continue;
            const int64_t o = static_cast<int64_t>(m) * a.N + n;
            if (a.acc) a.acc[o] = vals[e];
            if (FUSED || a.xs_in) {
                const float wsc = (e >> 1) ? wsc_hi : wsc_lo;
                a.out[o] = __float2half_rn(__fmul_rn(__fmul_rn(__int2float_rn(vals[e]), wsc), xscale_s[m]));
            }
        }
    }
}

// ---- int8 GEMV over the reference's [K][N] weights --------------------------------
// Thread = 16 consecutive columns (one 16-byte load per k row); four rows are
// loaded together and transposed with byte permutes so DP4A can consume
// column words.  4 threads span 64 columns, 64 threads split K.
constexpr int kKnTx = 4;
constexpr int kKnTy = 64;

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

template <int M>
__global__ void __launch_bounds__(kKnTx * kKnTy)
w8_kn_kernel(const int8_t* __restrict__ xq, const int8_t* __restrict__ w, int32_t* __restrict__ acc_out,
             int K, int N) {
    extern __shared__ int red_i[];  // [kKnTy/8 warps][M][64]
    const int tx = threadIdx.x % kKnTx;
    const int ty = threadIdx.x / kKnTx;
    const int nb = blockIdx.x * (kKnTx * 16);
    const int n0 = nb + tx * 16;
    pdl_trigger();
    pdl_wait();
    int acc[M][16];
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
        for (int e = 0; e < 16; ++e) acc[m][e] = 0;
    if (n0 < N) {
        for (int k = ty * 4; k < K; k += kKnTy * 4) {
            uint4 r[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) r[t] = ld_stream(w + static_cast<int64_t>(k + t) * N + n0);
            uint32_t xw[M];
#pragma unroll
            for (int m = 0; m < M; ++m) xw[m] = *reinterpret_cast<const uint32_t*>(xq + static_cast<int64_t>(m) * K + k);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t a0 = q == 0 ? r[0].x : q == 1 ? r[0].y : q == 2 ? r[0].z : r[0].w;
                const uint32_t a1 = q == 0 ? r[1].x : q == 1 ? r[1].y : q == 2 ? r[1].z : r[1].w;
                const uint32_t a2 = q == 0 ? r[2].x : q == 1 ? r[2].y : q == 2 ? r[2].z : r[2].w;
                const uint32_t a3 = q == 0 ? r[3].x : q == 1 ? r[3].y : q == 2 ? r[3].z : r[3].w;
                // 4x4 byte transpose: column c of this word group = bytes c of a0..a3
                const uint32_t t0 = prmt(a0, a1, 0x5140);
                const uint32_t t1 = prmt(a2, a3, 0x5140);
                const uint32_t t2 = prmt(a0, a1, 0x7362);
                const uint32_t t3 = prmt(a2, a3, 0x7362);
                const uint32_t c0 = prmt(t0, t1, 0x5410);
                const uint32_t c1 = prmt(t0, t1, 0x7632);
                const uint32_t c2 = prmt(t2, t3, 0x5410);
                const uint32_t c3 = prmt(t2, t3, 0x7632);
#pragma unroll
                for (int m = 0; m < M; ++m) {
                    acc[m][4 * q + 0] = __dp4a(static_cast<int>(c0), static_cast<int>(xw[m]), acc[m][4 * q + 0]);
                    acc[m][4 * q + 1] = __dp4a(static_cast<int>(c1), static_cast<int>(xw[m]), acc[m][4 * q + 1]);
                    acc[m][4 * q + 2] = __dp4a(static_cast<int>(c2), static_cast<int>(xw[m]), acc[m][4 * q + 2]);
                    acc[m][4 * q + 3] = __dp4a(static_cast<int>(c3), static_cast<int>(xw[m]), acc[m][4 * q + 3]);
                }
            }
        }
    }
    // reduce over the 8 ty values inside each warp (lanes differing in bits 2..4)
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
        for (int e = 0; e < 16; ++e) {
            int v = acc[m][e];
            v += __shfl_xor_sync(0xffffffffu, v, 4);
            v += __shfl_xor_sync(0xffffffffu, v, 8);
            v += __shfl_xor_sync(0xffffffffu, v, 16);
            acc[m][e] = v;
        }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane < kKnTx) {
#pragma unroll
        for (int m = 0; m < M; ++m)
#pragma unroll
            for (int e = 0; e < 16; ++e) red_i[(warp * M + m) * 64 + lane * 16 + e] = acc[m][e];
    }
    __syncthreads();
    for (int o = threadIdx.x; o < M * 64; o += kKnTx * kKnTy) {
        const int m = o / 64, col = o % 64;
        int s = 0;
        for (int wi = 0; wi < (kKnTx * kKnTy) / 32; ++wi) s += red_i[(wi * M + m) * 64 + col];
        const int n = nb + col;
        if (n < N) acc_out[static_cast<int64_t>(m) * N + n] = s;
    }
}

__global__ void dequant_kernel(const int32_t* __restrict__ acc, const __half* __restrict__ xs,
                               const __half* __restrict__ ws, __half* __restrict__ out, int M, int N) {
    pdl_trigger();
    pdl_wait();
    const int64_t total = static_cast<int64_t>(M) * N;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int m = static_cast<int>(i / N), n = static_cast<int>(i % N);
        const float d = __fmul_rn(__fmul_rn(__int2float_rn(acc[i]), __half2float(ws[n])), __half2float(xs[m]));
        out[i] = __float2half_rn(d);
    }
}

// fp32 -> fp16 by truncation, underflow to signed zero: the reference's
// host-side scale conversion (src/csrc/lib/quantized_weight.cpp:186-195).
__device__ __forceinline__ uint16_t f32_to_f16_trunc(float f) {
    const uint32_t x = __float_as_uint(f);
    const uint16_t sign = static_cast<uint16_t>((x >> 16) & 0x8000u);
    const int e = static_cast<int>((x >> 23) & 0xffu) - 112;
    if (e <= 0) return sign;
    if (e >= 31) return static_cast<uint16_t>(sign | 0x7c00u);
    return static_cast<uint16_t>(sign | (e << 10) | ((x & 0x7fffffu) >> 13));
}

// One thread per output column n; reads the [K][N] fp16 source coalesced.
// No early PDL trigger here: this kernel writes weights, and the GEMV kernels
// read their weights before griddepcontrol.wait, so a dependent launch may only
// start once every block of this one has finished its stores (the implicit
// trigger at exit).
__global__ void quantize_weight_kernel(const __half* __restrict__ w, int8_t* __restrict__ wq,
                                       __half* __restrict__ w_scale, int K, int N, int layout) {
    pdl_wait();
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= N) return;
    // layout 2 reads row n of an [N][K] weight; 0 and 1 read column n of [K][N]
    auto in = [&](int k) { return layout == 2 ? w[static_cast<int64_t>(n) * K + k] : w[static_cast<int64_t>(k) * N + n]; };
    float mx = 0.0f;
    for (int k = 0; k < K; ++k) mx = fmaxf(mx, fabsf(__half2float(in(k))));
    const float scale = scale_from_absmax(mx);
    const float inv = __fdiv_rn(1.0f, scale);
    w_scale[n] = __ushort_as_half(f32_to_f16_trunc(scale));
    for (int k = 0; k < K; ++k) {
        float q = __fmul_rn(__half2float(in(k)), inv);
        q = q > 127.0f ? 127.0f : q;
        q = q < -128.0f ? -128.0f : q;
        q = q >= 0.0f ? __fadd_rn(q, 0.5f) : __fsub_rn(q, 0.5f);
        const int8_t v = static_cast<int8_t>(__float2int_rz(q));
        if (layout != 1) wq[static_cast<int64_t>(n) * K + k] = v;
        else wq[static_cast<int64_t>(k) * N + n] = v;
    }
}

// Fills the group's block ranges for blocks of `cols` output columns.
int w8_assign_blocks(W8Group& gr, int cols) {
    int b = 0;
    for (int i = 0; i < gr.count; ++i) {
        gr.block_begin[i] = b;
        b += (gr.p[i].N + cols - 1) / cols;
    }
    gr.block_begin[gr.count] = b;
    return b;
}

template <int M, bool FUSED>
int launch_w8_mma_m(W8Group& gr, cudaStream_t s) {
    const W8Args& a = gr.p[0];
    const int nkb = (a.K + 63) / 64;
    const int per_warp = (nkb + kW8Warps - 1) / kW8Warps;
    const dim3 grid(w8_assign_blocks(gr, 16));
    const dim3 block(kW8Warps * 32);
    const size_t smem = static_cast<size_t>(M) * (a.K + kXqPad);
    auto go = [&](auto kern) -> int {
        if (smem > 48 * 1024) {
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
            if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(w8_mma)");
        }
        return launch(kern, grid, block, smem, s, gr);
    };
    if (per_warp <= 1) return go(w8_mma_kernel<M, 1, FUSED>);
    if (per_warp <= 2) return go(w8_mma_kernel<M, 2, FUSED>);
    if (per_warp <= 4) return go(w8_mma_kernel<M, 4, FUSED>);
    if (per_warp <= 8) return go(w8_mma_kernel<M, 8, FUSED>);
    return fail(MCV_ERR_SHAPE, "w8a8: K above 4096 unsupported on the [N][K] path");
}

template <int M, bool FUSED>
int launch_w8_rows_m(W8Group& gr, cudaStream_t s) {
    // one activation row: DP4A is quicker (1.93 vs 2.18 us at N=3584); from
    // four rows the tensor cores are (2.73 vs 4.05 us at M=4, N=3584), B200
    const int t = tuning(MCV_TUNE_W8A8_KERNEL);
    if (t == 2 || (t != 1 && M >= 2)) return launch_w8_mma_m<M, FUSED>(gr, s);
    const W8Args& a = gr.p[0];
    const int chunks_per_lane = (a.K / 16 + 31) / 32;
    int kch = 1;
    while (kch < chunks_per_lane) kch *= 2;
    const dim3 grid(w8_assign_blocks(gr, kW8Warps * kW8Cpw));
    const dim3 block(kW8Warps * 32);
    const size_t smem = static_cast<size_t>(M) * a.K;
    auto go = [&](auto kern) -> int {
        if (smem > 48 * 1024) {
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
            if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(w8_rows)");
        }
        return launch(kern, grid, block, smem, s, gr);
    };
    switch (kch) {
        case 1: return go(w8_rows_kernel<M, 1, FUSED>);
        case 2: return go(w8_rows_kernel<M, 2, FUSED>);
        case 4: return go(w8_rows_kernel<M, 4, FUSED>);
        case 8: return go(w8_rows_kernel<M, 8, FUSED>);
        default: return fail(MCV_ERR_SHAPE, "w8a8: K above 4096 unsupported on the [N][K] path");
    }
}

template <bool FUSED>
int launch_w8_group(int64_t M, W8Group& gr, cudaStream_t s) {
    switch (M) {
        case 1: return launch_w8_rows_m<1, FUSED>(gr, s);
        case 2: return launch_w8_rows_m<2, FUSED>(gr, s);
        case 3: return launch_w8_rows_m<3, FUSED>(gr, s);
        case 4: return launch_w8_rows_m<4, FUSED>(gr, s);
        case 5: return launch_w8_rows_m<5, FUSED>(gr, s);
        case 6: return launch_w8_rows_m<6, FUSED>(gr, s);
        case 7: return launch_w8_rows_m<7, FUSED>(gr, s);
        default: return launch_w8_rows_m<8, FUSED>(gr, s);
    }
}

template <bool FUSED>
int launch_w8_rows(int64_t M, const W8Args& a, cudaStream_t s) {
    W8Group gr{};
    gr.count = 1;
    gr.p[0] = a;
    return launch_w8_group<FUSED>(M, gr, s);
}

int launch_w8_kn(int64_t M, const int8_t* xq, const int8_t* w, int32_t* acc, int K, int N, cudaStream_t s) {
    const dim3 grid((N + kKnTx * 16 - 1) / (kKnTx * 16));
    const dim3 block(kKnTx * kKnTy);
    const size_t smem = static_cast<size_t>((kKnTx * kKnTy) / 32) * M * 64 * sizeof(int);
    switch (M) {
        case 1: return launch(w8_kn_kernel<1>, grid, block, smem, s, xq, w, acc, K, N);
        case 2: return launch(w8_kn_kernel<2>, grid, block, smem, s, xq, w, acc, K, N);
        case 3: return launch(w8_kn_kernel<3>, grid, block, smem, s, xq, w, acc, K, N);
        case 4: return launch(w8_kn_kernel<4>, grid, block, smem, s, xq, w, acc, K, N);
        case 5: return launch(w8_kn_kernel<5>, grid, block, smem, s, xq, w, acc, K, N);
        case 6: return launch(w8_kn_kernel<6>, grid, block, smem, s, xq, w, acc, K, N);
        case 7: return launch(w8_kn_kernel<7>, grid, block, smem, s, xq, w, acc, K, N);
        default: return launch(w8_kn_kernel<8>, grid, block, smem, s, xq, w, acc, K, N);
    }
}

int check_mkn(int64_t M, int64_t K, int64_t N) {
    if (M < 1 || M > 8) return fail(MCV_ERR_SHAPE, "w8a8: M must be 1..8");
    if (K <= 0 || N <= 0 || K % 16 != 0) return fail(MCV_ERR_SHAPE, "w8a8: K must be a positive multiple of 16, N positive");
    if (K > 16384 || N > (1 << 30)) return fail(MCV_ERR_SHAPE, "w8a8: dimension too large");
    return MCV_OK;
}

int launch_dequant(const void* acc, const void* xs, const void* ws, void* out, int64_t M, int64_t N, cudaStream_t s) {
    const int64_t total = M * N;
    int64_t blocks = (total + 255) / 256;
    const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
    if (blocks > cap) blocks = cap;
    return launch(dequant_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, s,
                  static_cast<const int32_t*>(acc), static_cast<const __half*>(xs),
                  static_cast<const __half*>(ws), static_cast<__half*>(out), static_cast<int>(M),
                  static_cast<int>(N));
}

}  // namespace
}  // namespace mcv

using namespace mcv;

extern "C" {

int mcv_w8a8_quantize(const void* x, void* x_int8, void* x_scale, int64_t M, int64_t K, mcv_stream_t stream) {
    if (!x || !x_int8 || !x_scale) return fail(MCV_ERR_NULL, "w8a8_quantize: null pointer");
    if (M < 1 || M > 65535 || K < 1 || K > (1 << 30)) return fail(MCV_ERR_SHAPE, "w8a8_quantize: bad shape");
    return launch(quantize_rows_kernel, dim3(static_cast<unsigned>(M)), dim3(kQThreads), 0,
                  static_cast<cudaStream_t>(stream), static_cast<const __half*>(x), static_cast<int8_t*>(x_int8),
                  static_cast<__half*>(x_scale), static_cast<int>(K));
}

int mcv_w8a8_gemm_i32(const void* x_int8, const void* w_int8, void* acc, int64_t M, int64_t K, int64_t N,
                      int w_layout, mcv_stream_t stream) {
    if (!x_int8 || !w_int8 || !acc) return fail(MCV_ERR_NULL, "w8a8_gemm_i32: null pointer");
    int st = check_mkn(M, K, N);
    if (st) return st;
    auto s = static_cast<cudaStream_t>(stream);
    if (w_layout == 0) {
        if (!aligned16(x_int8) || !aligned16(w_int8)) return fail(MCV_ERR_ALIGN, "w8a8_gemm_i32: x and w must be 16-byte aligned");
        W8Args a{};
        a.x = x_int8;
        a.w = static_cast<const int8_t*>(w_int8);
        a.acc = static_cast<int32_t*>(acc);
        a.K = static_cast<int>(K);
        a.N = static_cast<int>(N);
        return launch_w8_rows<false>(M, a, s);
    }
    if (w_layout != 1) return fail(MCV_ERR_VALUE, "w8a8_gemm_i32: w_layout must be 0 ([N][K]) or 1 ([K][N])");
    if (N % 16 != 0) return fail(MCV_ERR_SHAPE, "w8a8_gemm_i32: [K][N] layout needs N % 16 == 0");
    if (!aligned16(w_int8) || (reinterpret_cast<uintptr_t>(x_int8) & 3u))
        return fail(MCV_ERR_ALIGN, "w8a8_gemm_i32: w must be 16-byte and x 4-byte aligned");
    return launch_w8_kn(M, static_cast<const int8_t*>(x_int8), static_cast<const int8_t*>(w_int8),
                        static_cast<int32_t*>(acc), static_cast<int>(K), static_cast<int>(N), s);
}

int mcv_w8a8_dequant(const void* acc, const void* x_scale, const void* w_scale, void* out, int64_t M, int64_t N,
                     mcv_stream_t stream) {
    if (!acc || !x_scale || !w_scale || !out) return fail(MCV_ERR_NULL, "w8a8_dequant: null pointer");
    if (M < 1 || N < 1 || M * N > (int64_t(1) << 40) || N > (1 << 30) || M > (1 << 30))
        return fail(MCV_ERR_SHAPE, "w8a8_dequant: bad shape");
    return launch_dequant(acc, x_scale, w_scale, out, M, N, static_cast<cudaStream_t>(stream));
}

int mcv_w8a8_fused(const void* x, const void* w_int8, const void* w_scale, void* out, void* acc_out,
                   void* x_int8_out, void* x_scale_out, int64_t M, int64_t K, int64_t N, int w_layout,
                   mcv_stream_t stream) {
    if (!x || !w_int8 || !w_scale || !out) return fail(MCV_ERR_NULL, "w8a8_fused: null pointer");
    int st = check_mkn(M, K, N);
    if (st) return st;
    auto s = static_cast<cudaStream_t>(stream);
    if (w_layout == 0) {
        if (!aligned16(w_int8) || !aligned16(x)) return fail(MCV_ERR_ALIGN, "w8a8_fused: x and w must be 16-byte aligned");
        if (reinterpret_cast<uintptr_t>(x_int8_out) & 7u) return fail(MCV_ERR_ALIGN, "w8a8_fused: x_int8_out must be 8-byte aligned");
        W8Args a{};
        a.x = x;
        a.w = static_cast<const int8_t*>(w_int8);
        a.w_scale = static_cast<const __half*>(w_scale);
        a.out = static_cast<__half*>(out);
        a.acc = static_cast<int32_t*>(acc_out);
        a.xq_out = static_cast<int8_t*>(x_int8_out);
        a.xs_out = static_cast<__half*>(x_scale_out);
        a.K = static_cast<int>(K);
        a.N = static_cast<int>(N);
        return launch_w8_rows<true>(M, a, s);
    }
    if (w_layout != 1) return fail(MCV_ERR_VALUE, "w8a8_fused: w_layout must be 0 or 1");
    if (!acc_out || !x_int8_out || !x_scale_out)
        return fail(MCV_ERR_WORKSPACE, "w8a8_fused: the [K][N] path needs acc_out, x_int8_out and x_scale_out buffers");
    st = mcv_w8a8_quantize(x, x_int8_out, x_scale_out, M, K, stream);
    if (st) return st;
    st = mcv_w8a8_gemm_i32(x_int8_out, w_int8, acc_out, M, K, N, 1, stream);
    if (st) return st;
    return launch_dequant(acc_out, x_scale_out, w_scale, out, M, N, s);
}

int mcv_w8a8_gemv_prequant(const void* x_int8, const void* x_scale, const void* w_int8, const void* w_scale, void* out,
                           void* acc_out, int64_t M, int64_t K, int64_t N, mcv_stream_t stream) {
    if (!x_int8 || !x_scale || !w_int8 || !w_scale || !out) return fail(MCV_ERR_NULL, "w8a8_gemv_prequant: null pointer");
    int st = check_mkn(M, K, N);
    if (st) return st;
    if (!aligned16(w_int8) || !aligned16(x_int8))
        return fail(MCV_ERR_ALIGN, "w8a8_gemv_prequant: x_int8 and w must be 16-byte aligned");
    W8Args a{};
    a.x = x_int8;
    a.w = static_cast<const int8_t*>(w_int8);
    a.w_scale = static_cast<const __half*>(w_scale);
    a.xs_in = static_cast<const __half*>(x_scale);
    a.out = static_cast<__half*>(out);
    a.acc = static_cast<int32_t*>(acc_out);
    a.K = static_cast<int>(K);
    a.N = static_cast<int>(N);
    return launch_w8_rows<false>(M, a, static_cast<cudaStream_t>(stream));
}

int mcv_w8a8_fused_grouped(const mcv_w8a8_problem* problems, int count, int64_t M, int64_t K, mcv_stream_t stream) {
    if (!problems || count < 1) return fail(MCV_ERR_NULL, "w8a8_fused_grouped: no problems");
    if (count > kW8MaxProblems) return fail(MCV_ERR_SHAPE, "w8a8_fused_grouped: at most 16 problems per launch");
    int st = check_mkn(M, K, 16);
    if (st) return st;
    W8Group gr{};
    gr.count = count;
    for (int i = 0; i < count; ++i) {
        const mcv_w8a8_problem& q = problems[i];
        if (!q.x || !q.w_int8 || !q.w_scale || !q.out) return fail(MCV_ERR_NULL, "w8a8_fused_grouped: null pointer");
        if (q.N < 1 || q.N > (1 << 30)) return fail(MCV_ERR_SHAPE, "w8a8_fused_grouped: bad N");
        if (!aligned16(q.x) || !aligned16(q.w_int8)) return fail(MCV_ERR_ALIGN, "w8a8_fused_grouped: x and w must be 16-byte aligned");
        W8Args& a = gr.p[i];
        a.x = q.x;
        a.w = static_cast<const int8_t*>(q.w_int8);
        a.w_scale = static_cast<const __half*>(q.w_scale);
        a.out = static_cast<__half*>(q.out);
        a.K = static_cast<int>(K);
        a.N = static_cast<int>(q.N);
    }
    return launch_w8_group<true>(M, gr, static_cast<cudaStream_t>(stream));
}

int mcv_w8a8_quantize_weight(const void* w_kn, void* wq, void* w_scale, int64_t K, int64_t N, int w_layout,
                             mcv_stream_t stream) {
    if (!w_kn || !wq || !w_scale) return fail(MCV_ERR_NULL, "w8a8_quantize_weight: null pointer");
    if (K < 1 || N < 1 || K > (1 << 30) || N > (1 << 30)) return fail(MCV_ERR_SHAPE, "w8a8_quantize_weight: bad shape");
    if (w_layout < 0 || w_layout > 2) return fail(MCV_ERR_VALUE, "w8a8_quantize_weight: w_layout must be 0, 1 or 2");
    return launch(quantize_weight_kernel, dim3(static_cast<unsigned>((N + 127) / 128)), dim3(128), 0,
                  static_cast<cudaStream_t>(stream), static_cast<const __half*>(w_kn), static_cast<int8_t*>(wq),
                  static_cast<__half*>(w_scale), static_cast<int>(K), static_cast<int>(N), w_layout);
}

}  // extern "C"
