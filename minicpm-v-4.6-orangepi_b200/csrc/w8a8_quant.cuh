// Per-row symmetric int8 quantization of activations, shared by the W8A8
// kernels and the W8A8 lm_head so both quantize x with the same arithmetic:
// scale = max|x| / 127 (at least 1e-8), q = trunc(clamp(x / scale) +/- 0.5)
// with every float step explicitly rounded, as the reference's
// w8a8_quantize kernel (op_kernel/w8a8_quantize_custom.cpp:25-41).
#pragma once

#include "common.cuh"

namespace mcv {

__device__ __forceinline__ int8_t quant_act(float v, float inv) {
    float q = __fmul_rn(v, inv);
    q = q > 127.0f ? 127.0f : q;
    q = q < -128.0f ? -128.0f : q;
    q = q >= 0.0f ? __fadd_rn(q, 0.5f) : __fsub_rn(q, 0.5f);
    return static_cast<int8_t>(__float2int_rz(q));
}

__device__ __forceinline__ float scale_from_absmax(float max_abs) {
    float s = __fdiv_rn(max_abs, 127.0f);
    return s < 0.00000001f ? 0.00000001f : s;
}

// Quantizes the M rows of x (fp16 [M][K], 16-byte aligned) into xq8 (int8,
// row stride `stride` bytes) and their fp16-rounded scales into xscale_s
// (as float).  All rows are loaded into registers with independent 16-byte
// loads (one round trip), reduced to per-row maxima across the block (NT
// threads), then quantized from the same registers.  Block 0 also writes
// the optional copies xq_out ([M][K]) and xs_out ([M]).  VPT = 16-byte
// vectors per thread per row (K <= 8 * NT * VPT).
template <int M, int VPT, int NT>
__device__ __forceinline__ void quantize_rows_to_smem(const __half* x, int K, int8_t* xq8, int stride, float* xscale_s,
                                                      int8_t* xq_out, __half* xs_out) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // All M rows are loaded into registers with independent 16-byte loads
    // (one L2 round trip), reduced to per-row maxima, then quantized from
    // the same registers into shared memory.
    constexpr int T = NT;
    const uint4* xh4 = reinterpret_cast<const uint4*>(x);
    const int vpr = K >> 3;  // 16-byte vectors per row
    uint4 xr[M][VPT];
    float mx[M];
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
        for (int t = 0; t < VPT; ++t) {
            const int v = threadIdx.x + t * T;
            xr[m][t] = v < vpr ? xh4[m * vpr + v] : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
    for (int m = 0; m < M; ++m) {
        mx[m] = 0.0f;
#pragma unroll
        for (int t = 0; t < VPT; ++t) {
            const uint32_t wd[4] = {xr[m][t].x, xr[m][t].y, xr[m][t].z, xr[m][t].w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 f = __half22float2(u32_as_h2(wd[e]));
                mx[m] = fmaxf(mx[m], fmaxf(fabsf(f.x), fabsf(f.y)));
            }
        }
    }
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx[m] = fmaxf(mx[m], __shfl_xor_sync(0xffffffffu, mx[m], o));
    __shared__ float red_m[NT / 32][M];
    __shared__ float inv_s[M];
    if (lane == 0) {
#pragma unroll
        for (int m = 0; m < M; ++m) red_m[warp][m] = mx[m];
    }
    __syncthreads();
    if (threadIdx.x < M) {
        const int m = threadIdx.x;
        float r = 0.0f;
        for (int i = 0; i < NT / 32; ++i) r = fmaxf(r, red_m[i][m]);
        const float scale = scale_from_absmax(r);
        inv_s[m] = __fdiv_rn(1.0f, scale);
        const __half sh = __float2half_rn(scale);
        xscale_s[m] = __half2float(sh);
        if (blockIdx.x == 0 && xs_out) xs_out[m] = sh;
    }
    __syncthreads();
#pragma unroll
    for (int m = 0; m < M; ++m) {
        const float inv = inv_s[m];
#pragma unroll
        for (int t = 0; t < VPT; ++t) {
            const int v = threadIdx.x + t * T;
            if (v >= vpr) continue;
            const uint32_t wd[4] = {xr[m][t].x, xr[m][t].y, xr[m][t].z, xr[m][t].w};
            uint32_t packed[2] = {0u, 0u};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 f = __half22float2(u32_as_h2(wd[e]));
                const uint32_t q0 = static_cast<uint8_t>(quant_act(f.x, inv));
                const uint32_t q1 = static_cast<uint8_t>(quant_act(f.y, inv));
                packed[e >> 1] |= (q0 | (q1 << 8)) << (16 * (e & 1));
            }
            *reinterpret_cast<uint2*>(xq8 + m * stride + v * 8) = make_uint2(packed[0], packed[1]);
            if (blockIdx.x == 0 && xq_out)
                *reinterpret_cast<uint2*>(xq_out + static_cast<int64_t>(m) * K + v * 8) =
                    make_uint2(packed[0], packed[1]);
        }
    }
}

}  // namespace mcv
