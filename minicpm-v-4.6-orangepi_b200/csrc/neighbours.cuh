// Device helpers for the element-wise neighbours of the decode GEMVs, fused
// into the GEMV prologues (and used by the stand-alone kernels of
// neighbours.cu):
//
//  * rms_norm, two variants:
//    0 - the engine's rms_norm (src/csrc/lib/ops.cpp:564-737), applied by
//        lm_head_greedy before the lm_head (src/csrc/lib/language_model.cpp:423)
//        and by every decoder layer before its projections.  It is a chain of
//        fp16 tensor ops, so every intermediate is rounded to fp16:
//        sq = x*x, mean = sum(sq)/H, ms = mean + eps, rstd = 1/sqrt(ms),
//        scaled = x*rstd, gp1 = gamma + 1, out = scaled * gp1.
//        The sum of the fp16 squares is taken exactly (in double: fp16 values
//        span fewer than 53 bits, so no order changes it), then rounded to
//        fp32 and divided by H - one defined result where the reference's
//        aclnnMean leaves the order open.
//    1 - the rms_norm1024 custom kernel (op_kernel/rms_norm1024_custom.cpp:57-70):
//        fp32, inv = 1/sqrt(sum(x^2)/H + eps), out = RN((x*inv)*gamma).
//    Every float step is an explicitly rounded intrinsic, so the result is the
//    CPU restatement's bit for bit.
//  * silu_mul (op_kernel/silu_mul_custom.cpp:63-72): fp32
//    s = g / (1 + exp(-g)), out = RN(s * u).  exp is CUDA's expf.
#pragma once

#include "common.cuh"

namespace mcv {

__device__ __forceinline__ __half rn16(float f) { return __float2half_rn(f); }

__device__ __forceinline__ double warp_sum_f64(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Normalises M rows of H fp16 values (row stride H) from src into dst, with
// all threads of the block (blockDim.x a multiple of 32, at most 1024).
// src and dst may be global or shared memory, but must not overlap.  When
// H <= kNormCache * blockDim.x (e.g. a 1024-wide row on 256 threads) src is
// read once and kept in registers between the two passes.  Ends with a
// __syncthreads().
constexpr int kNormCache = 4;

template <int M>
__device__ __forceinline__ void rms_norm_rows_block(const __half* src, __half* dst, int H, const NormArgs& na) {
    __shared__ double part[32][M];
    __shared__ float rstd_s[M];
    const int tid = threadIdx.x, nthr = blockDim.x;
    const int lane = tid & 31, warp = tid >> 5, nwarps = nthr >> 5;
    const bool cached = H <= kNormCache * nthr;
    float xc[kNormCache][M];
    double s[M];
#pragma unroll
    for (int m = 0; m < M; ++m) s[m] = 0.0;
    auto sq = [&](float x) {
        return na.variant == 0 ? static_cast<double>(__half2float(rn16(__fmul_rn(x, x))))
                               : static_cast<double>(x) * static_cast<double>(x);
    };
    if (cached) {
#pragma unroll
        for (int i = 0; i < kNormCache; ++i) {
            const int h = tid + i * nthr;
#pragma unroll
            for (int m = 0; m < M; ++m) {
                xc[i][m] = h < H ? __half2float(src[static_cast<int64_t>(m) * H + h]) : 0.0f;
                s[m] += sq(xc[i][m]);
            }
        }
    } else {
        for (int h = tid; h < H; h += nthr) {
#pragma unroll
            for (int m = 0; m < M; ++m) s[m] += sq(__half2float(src[static_cast<int64_t>(m) * H + h]));
        }
    }
#pragma unroll
    for (int m = 0; m < M; ++m) {
        const double w = warp_sum_f64(s[m]);
        if (lane == 0) part[warp][m] = w;
    }
    __syncthreads();
    if (tid < M) {
        const int m = tid;
        double t = 0.0;
        for (int w = 0; w < nwarps; ++w) t += part[w][m];
        const float sum = __double2float_rn(t);
        float r;
        if (na.variant == 0) {
            const __half mean = rn16(__fdiv_rn(sum, static_cast<float>(H)));
            const __half ms = rn16(__fadd_rn(__half2float(mean), na.eps));
            r = __half2float(rn16(__fdiv_rn(1.0f, __fsqrt_rn(__half2float(ms)))));
        } else {
            r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(sum, __fdiv_rn(1.0f, static_cast<float>(H))), na.eps)));
        }
        rstd_s[m] = r;
    }
    __syncthreads();
    auto put = [&](int h, int m, float x) {
        const float g = __half2float(na.gamma[h]);
        __half o;
        if (na.variant == 0)
            o = rn16(__fmul_rn(__half2float(rn16(__fmul_rn(x, rstd_s[m]))), __half2float(rn16(__fadd_rn(g, 1.0f)))));
        else
            o = rn16(__fmul_rn(__fmul_rn(x, rstd_s[m]), g));
        dst[static_cast<int64_t>(m) * H + h] = o;
    };
    if (cached) {
#pragma unroll
        for (int i = 0; i < kNormCache; ++i) {
            const int h = tid + i * nthr;
            if (h < H) {
#pragma unroll
                for (int m = 0; m < M; ++m) put(h, m, xc[i][m]);
            }
        }
    } else {
        for (int h = tid; h < H; h += nthr) {
#pragma unroll
            for (int m = 0; m < M; ++m) put(h, m, __half2float(src[static_cast<int64_t>(m) * H + h]));
        }
    }
    __syncthreads();
}

__device__ __forceinline__ __half silu_mul1(__half gate, __half up) {
    const float g = __half2float(gate);
    const float s = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
    return rn16(__fmul_rn(s, __half2float(up)));
}

// Eight consecutive elements (one 16-byte vector of each operand).
__device__ __forceinline__ uint4 silu_mul8(uint4 g, uint4 u) {
    uint4 r;
    uint32_t* rp = &r.x;
    const uint32_t* gp = &g.x;
    const uint32_t* up = &u.x;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __half2 gg = *reinterpret_cast<const __half2*>(&gp[i]);
        const __half2 uu = *reinterpret_cast<const __half2*>(&up[i]);
        const __half2 o = __halves2half2(silu_mul1(__low2half(gg), __low2half(uu)),
                                         silu_mul1(__high2half(gg), __high2half(uu)));
        rp[i] = *reinterpret_cast<const uint32_t*>(&o);
    }
    return r;
}

}  // namespace mcv
