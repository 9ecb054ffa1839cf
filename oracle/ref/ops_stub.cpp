// The reference engine's ops (src/csrc/include/minicpmv/ops.h) that its
// CPU-checked tests call, implemented on the host by this repository's CPU
// oracle (../oracle.c).  TEST INFRASTRUCTURE: linked with the reference's own
// test programs and host sources (built by ./Makefile into ../_ref/), so that
// the reference's tests - their own seeded inputs and their own checker loops
// - judge the oracle that in turn judges the CUDA kernels.  Tensors are host
// memory here (acl_stub.cpp).
#include <cstring>
#include <stdexcept>
#include <vector>

#include "minicpmv/ops.h"
#include "oracle.h"

namespace minicpmv {
namespace {

void need(bool ok, const char* what) {
    if (!ok) throw std::runtime_error(what);
}

template <class T>
T* ptr(const Tensor& t) {
    return static_cast<T*>(t.data());
}

void rn16_store(const std::vector<float>& v, Tensor& out) {
    need(out.numel() == v.size(), "output size mismatch");
    orc_f32_to_f16_rn_array(v.data(), ptr<uint16_t>(out), static_cast<int64_t>(v.size()));
}

}  // namespace

// ops.h:104-108: x fp16 [1,K], w int8 tile-packed [rows, tile_len], scales fp16 [K/128, N]
void matmul_w4a16(const Tensor& x, const Tensor& w_int8, const Tensor& scales, Tensor& out, aclrtStream) {
    need(x.shape().size() == 2 && scales.shape().size() == 2 && w_int8.shape().size() == 2, "matmul_w4a16 ranks");
    const int64_t M = x.shape()[0], K = x.shape()[1], N = scales.shape()[1], tile = w_int8.shape()[1];
    need(scales.shape()[0] * 128 == K, "matmul_w4a16 scales shape");
    need(orc_w4a16_tile_rows(K, N, tile) == w_int8.shape()[0], "matmul_w4a16 tile rows");
    std::vector<int8_t> w(static_cast<size_t>(K * N));
    orc_w4a16_unpack_tiles(ptr<int8_t>(w_int8), K, N, tile, w.data());
    std::vector<float> o(static_cast<size_t>(M * N));
    orc_w4a16_gemv(ptr<uint16_t>(x), w.data(), ptr<uint16_t>(scales), M, K, N, 128, o.data());
    rn16_store(o, out);
}

// ops.h:112-115: int8 x [M,K] . int8 w [K,N] -> int32 [M,N]
void matmul_w8a8_i32(const Tensor& x, const Tensor& w, Tensor& out, aclrtStream) {
    const int64_t M = x.shape()[0], K = x.shape()[1], N = w.shape()[1];
    need(w.shape()[0] == K, "matmul_w8a8_i32 K");
    orc_w8a8_gemm_i32(ptr<int8_t>(x), ptr<int8_t>(w), M, K, N, ptr<int32_t>(out));
}

// ops.h:117-120
void w8a8_quantize(const Tensor& x, Tensor& x_int8, Tensor& x_scale, aclrtStream) {
    const int64_t M = x.shape()[0], K = x.shape()[1];
    orc_w8a8_quantize(ptr<uint16_t>(x), M, K, ptr<int8_t>(x_int8), ptr<uint16_t>(x_scale));
}

// ops.h:122-126
void w8a8_dequant(const Tensor& acc, const Tensor& x_scale, const Tensor& w_scale, Tensor& out, aclrtStream) {
    const int64_t M = acc.shape()[0], N = acc.shape()[1];
    orc_w8a8_dequant(ptr<int32_t>(acc), ptr<uint16_t>(x_scale), ptr<uint16_t>(w_scale), M, N, ptr<uint16_t>(out));
}

// ops.h:17: fp16 a [M,K] . b [K,N]
void matmul(const Tensor& a, const Tensor& b, Tensor& out, aclrtStream) {
    const int64_t M = a.shape()[0], K = a.shape()[1], N = b.shape()[1];
    need(b.shape()[0] == K, "matmul K");
    std::vector<float> o(static_cast<size_t>(M * N));
    orc_gemv_f16(ptr<uint16_t>(a), ptr<uint16_t>(b), M, K, N, 1, o.data());
    rn16_store(o, out);
}

// ops.h:19: b is [N,K] or [K,N], told apart by a's K as ops.cpp:165-171 does
void matmul_b_transposed(const Tensor& a, const Tensor& b, Tensor& out, aclrtStream) {
    const int64_t M = a.shape()[0], K = a.shape()[1];
    int layout;
    int64_t N;
    if (b.shape()[1] == K) {
        layout = 0, N = b.shape()[0];
    } else {
        need(b.shape()[0] == K, "matmul_b_transposed K");
        layout = 1, N = b.shape()[1];
    }
    std::vector<float> o(static_cast<size_t>(M * N));
    orc_gemv_f16(ptr<uint16_t>(a), ptr<uint16_t>(b), M, K, N, layout, o.data());
    rn16_store(o, out);
}

// ops.h:21: first maximum of each fp16 row -> int64
void argmax_last_dim(const Tensor& self, Tensor& out, aclrtStream) {
    const int64_t M = self.shape()[0], V = self.shape()[1];
    const uint16_t* p = ptr<uint16_t>(self);
    int64_t* o = ptr<int64_t>(out);
    for (int64_t m = 0; m < M; ++m) {
        int64_t best = 0;
        float bv = orc_f16_to_f32(p[m * V]);
        for (int64_t v = 1; v < V; ++v) {
            const float f = orc_f16_to_f32(p[m * V + v]);
            if (f > bv) bv = f, best = v;
        }
        o[m] = best;
    }
}

// ops.h:53-55 (the fp32 custom kernel) and :56-58 (the engine's fp16 chain)
void rms_norm1024(const Tensor& x, const Tensor& gamma, Tensor& out, double epsilon, aclrtStream) {
    const int64_t H = x.shape().back(), rows = static_cast<int64_t>(x.numel()) / H;
    orc_rms_norm_fp32(ptr<uint16_t>(x), ptr<uint16_t>(gamma), rows, H, static_cast<float>(epsilon), ptr<uint16_t>(out));
}
void rms_norm(const Tensor& x, const Tensor& gamma, Tensor& out, double epsilon, aclrtStream) {
    const int64_t H = x.shape().back(), rows = static_cast<int64_t>(x.numel()) / H;
    orc_rms_norm_chain(ptr<uint16_t>(x), ptr<uint16_t>(gamma), rows, H, static_cast<float>(epsilon),
                       ptr<uint16_t>(out));
}

// ops.h:41
void silu_mul(const Tensor& gate, const Tensor& up, Tensor& out, aclrtStream) {
    orc_silu_mul(ptr<uint16_t>(gate), ptr<uint16_t>(up), static_cast<int64_t>(gate.numel()), ptr<uint16_t>(out));
}

}  // namespace minicpmv
