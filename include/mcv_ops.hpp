/* C++ shim over the mcv_matmul.h C ABI with the reference engine's op names
 * and calling convention (src/csrc/include/minicpmv/ops.h): tensors in,
 * output tensor by reference, a stream last, errors as exceptions.
 *
 * The functions are templates over the caller's tensor type; it needs
 *   void* data() const;  const std::vector<int64_t>& shape() const;
 * which the reference's minicpmv::Tensor provides (tensor.h:56-60), so the
 * engine's call sites keep their arguments.  Unlike the reference, calls do
 * not synchronise the stream unless `sync` is true (ops.cpp:359-377 syncs
 * after every op).  Quantized weights are the library's own packed formats
 * (W4A16Weight / W8A8Weight below), prepared once at load time. */
#ifndef MCV_OPS_HPP
#define MCV_OPS_HPP

#include <cuda_runtime_api.h>

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include "mcv_matmul.h"

namespace mcv_ops {

/* A failed call: the library status and its message (mcv_last_error). */
class Error : public std::runtime_error {
public:
    Error(int status, const std::string& what)
        : std::runtime_error(what + ": " + mcv_status_string(status) + ": " + mcv_last_error()), status_(status) {}
    int status() const { return status_; }

private:
    int status_;
};

inline void check(int status, const char* what) {
    if (status != MCV_OK) throw Error(status, what);
}

inline void finish(cudaStream_t stream, bool sync, const char* what) {
    if (!sync) return;
    const cudaError_t e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

/* mcv-int4 weight of one projection (mcv_w4a16_pack_*_host + one H2D copy
 * per array).  Stands in for W4A16QuantizedWeight (quantized_weight.h:11-17). */
struct W4A16Weight {
    const void* qweight = nullptr;
    const void* scales = nullptr;
    const void* zeros = nullptr;
    int zero_bias = 0;
    int64_t K = 0, N = 0;
};

/* int8 weight [N][K] + fp16 per-channel scales [N] (mcv_w8a8_quantize_weight,
 * w_layout 0).  Stands in for W8A8QuantizedWeight (quantized_weight.h:19-24). */
struct W8A8Weight {
    const void* w_int8 = nullptr;
    const void* w_scale = nullptr;
    int64_t K = 0, N = 0;
};

namespace detail {
template <class T>
void need_rank2(const T& t, const char* what) {
    if (t.shape().size() != 2) throw Error(MCV_ERR_SHAPE, std::string(what) + ": expected a 2-D tensor");
}
}  // namespace detail

/* out [M,N] = x [M,K] . W for the packed int4 weight (the GEMV up to 32 rows,
 * or 64 rows with K <= 4096; the tensor-core GEMM beyond).  ops.h:104-108. */
template <class T>
void matmul_w4a16(const T& x, const W4A16Weight& w, T& out, cudaStream_t stream, bool sync = false) {
    detail::need_rank2(x, "matmul_w4a16");
    const int64_t M = x.shape()[0], K = x.shape()[1];
    if (K != w.K) throw Error(MCV_ERR_SHAPE, "matmul_w4a16: x and weight K differ");
    const int st = (M <= 32 || (M <= 64 && K <= 4096)) ? mcv_w4a16_gemv(x.data(), w.qweight, w.scales, w.zeros, w.zero_bias, out.data(), M, K,
                                           w.N, 128, stream)
                          : mcv_w4a16_gemm(x.data(), w.qweight, w.scales, w.zeros, w.zero_bias, out.data(), M, K,
                                           w.N, 128, stream);
    check(st, "matmul_w4a16");
    finish(stream, sync, "matmul_w4a16");
}

/* The MLP's gate / up projections and their silu_mul in one launch:
 * act [M,N] = silu_mul(x . gate, x . up) (decoder_layer.cpp:1186-1203). */
template <class T>
void matmul_w4a16_gate_up_silu(const T& x, const W4A16Weight& gate, const W4A16Weight& up, T& act,
                               cudaStream_t stream, bool sync = false) {
    detail::need_rank2(x, "matmul_w4a16_gate_up_silu");
    const mcv_w4a16_problem g{nullptr, gate.qweight, gate.scales, gate.zeros, nullptr, static_cast<int32_t>(gate.K),
                              static_cast<int32_t>(gate.N), 128, gate.zero_bias};
    const mcv_w4a16_problem u{nullptr, up.qweight, up.scales, up.zeros, nullptr, static_cast<int32_t>(up.K),
                              static_cast<int32_t>(up.N), 128, up.zero_bias};
    check(mcv_w4a16_gemv_gate_up_silu(x.data(), &g, &u, act.data(), x.shape()[0], stream), "matmul_w4a16_gate_up_silu");
    finish(stream, sync, "matmul_w4a16_gate_up_silu");
}

/* out [M,N] = a [M,K] . B with b stored [N,K] or [K,N], told apart by a's K
 * as the reference does (ops.cpp:165-171): the GEMV for M <= 8, the
 * tensor-core GEMM beyond ([N,K] weights only).  ops.h:19. */
template <class T>
void matmul_b_transposed(const T& a, const T& b, T& out, cudaStream_t stream, bool sync = false) {
    detail::need_rank2(a, "matmul_b_transposed");
    detail::need_rank2(b, "matmul_b_transposed");
    const int64_t M = a.shape()[0], K = a.shape()[1];
    int layout;
    int64_t N;
    if (b.shape()[1] == K) {
        layout = 0, N = b.shape()[0];
    } else if (b.shape()[0] == K) {
        layout = 1, N = b.shape()[1];
    } else {
        throw Error(MCV_ERR_SHAPE, "matmul_b_transposed: K dim mismatch");
    }
    if (M > 8) {
        // the tensor-core GEMM takes [N,K]; a [K,N] weight needs mcv_transpose_f16 once at load time
        if (layout != 0) throw Error(MCV_ERR_SHAPE, "matmul_b_transposed: M > 8 needs the weight as [N,K]");
        check(mcv_gemm_f16(a.data(), b.data(), out.data(), M, K, N, stream), "matmul_b_transposed");
    } else {
        check(mcv_gemv_f16(a.data(), b.data(), out.data(), M, K, N, layout, stream), "matmul_b_transposed");
    }
    finish(stream, sync, "matmul_b_transposed");
}

/* int64 [M] = first-max index of fp16 [M,V] along the last dim.  ops.h:21. */
template <class T>
void argmax_last_dim(const T& self, T& out, cudaStream_t stream, bool sync = false) {
    detail::need_rank2(self, "argmax_last_dim");
    check(mcv_argmax_last_dim_f16(self.data(), out.data(), self.shape()[0], self.shape()[1], stream),
          "argmax_last_dim");
    finish(stream, sync, "argmax_last_dim");
}

/* int32 [M,N] = int8 x [M,K] . int8 w [K,N] (the reference's layout).  ops.h:112-115. */
template <class T>
void matmul_w8a8_i32(const T& x, const T& w, T& out, cudaStream_t stream, bool sync = false) {
    detail::need_rank2(x, "matmul_w8a8_i32");
    detail::need_rank2(w, "matmul_w8a8_i32");
    check(mcv_w8a8_gemm_i32(x.data(), w.data(), out.data(), x.shape()[0], x.shape()[1], w.shape()[1], 1, stream),
          "matmul_w8a8_i32");
    finish(stream, sync, "matmul_w8a8_i32");
}

/* Per-row absmax quantization to int8 + fp16 scales.  ops.h:117-120. */
template <class T>
void w8a8_quantize(const T& x, T& x_int8, T& x_scale, cudaStream_t stream, bool sync = false) {
    detail::need_rank2(x, "w8a8_quantize");
    check(mcv_w8a8_quantize(x.data(), x_int8.data(), x_scale.data(), x.shape()[0], x.shape()[1], stream),
          "w8a8_quantize");
    finish(stream, sync, "w8a8_quantize");
}

/* fp16 out = RN((acc * w_scale) * x_scale).  ops.h:122-126. */
template <class T>
void w8a8_dequant(const T& acc, const T& x_scale, const T& w_scale, T& out, cudaStream_t stream, bool sync = false) {
    detail::need_rank2(acc, "w8a8_dequant");
    check(mcv_w8a8_dequant(acc.data(), x_scale.data(), w_scale.data(), out.data(), acc.shape()[0], acc.shape()[1],
                           stream),
          "w8a8_dequant");
    finish(stream, sync, "w8a8_dequant");
}

/* matmul_decode_w8a8_prequant (decoder_layer.cpp:216-224): int8 x with its
 * fp16 scales (from w8a8_quantize) against a W8A8Weight, int32 GEMV + dequant
 * in one kernel. */
template <class T>
void matmul_decode_w8a8_prequant(const T& x_int8, const T& x_scale, const W8A8Weight& w, T& out, cudaStream_t stream,
                                 bool sync = false) {
    detail::need_rank2(x_int8, "matmul_decode_w8a8_prequant");
    if (x_int8.shape()[1] != w.K) throw Error(MCV_ERR_SHAPE, "matmul_decode_w8a8_prequant: x and weight K differ");
    check(mcv_w8a8_gemv_prequant(x_int8.data(), x_scale.data(), w.w_int8, w.w_scale, out.data(), nullptr,
                                 x_int8.shape()[0], w.K, w.N, stream),
          "matmul_decode_w8a8_prequant");
    finish(stream, sync, "matmul_decode_w8a8_prequant");
}

/* The projection's format chosen like matmul_decode_dispatch
 * (decoder_layer.cpp:226-244); absent formats are nullptr. */
template <class T>
void matmul_decode_dispatch(const T& x, const T* dense_weight, const W4A16Weight* quant_weight,
                            const W8A8Weight* w8_weight, T& out, cudaStream_t stream, bool sync = false) {
    detail::need_rank2(x, "matmul_decode_dispatch");
    detail::need_rank2(out, "matmul_decode_dispatch");
    const int64_t M = x.shape()[0], K = x.shape()[1], N = out.shape()[1];
    mcv_decode_weights f{};
    if (dense_weight) {
        detail::need_rank2(*dense_weight, "matmul_decode_dispatch");
        f.dense = dense_weight->data();
        f.dense_layout = dense_weight->shape()[1] == K ? 0 : 1;
    }
    if (quant_weight) {
        f.w4_qweight = quant_weight->qweight;
        f.w4_scales = quant_weight->scales;
        f.w4_zeros = quant_weight->zeros;
        f.w4_zero_bias = quant_weight->zero_bias;
    }
    if (w8_weight) {
        f.w8_weight = w8_weight->w_int8;
        f.w8_scale = w8_weight->w_scale;
    }
    check(mcv_matmul_decode_dispatch(x.data(), &f, out.data(), M, K, N, stream), "matmul_decode_dispatch");
    finish(stream, sync, "matmul_decode_dispatch");
}

/* Greedy lm_head over fp16 embedding rows [V,K] for one row of x: the fused
 * GEMV + first-max argmax, index read back to the host (one 8-byte copy,
 * then a stream sync) - the device part of lm_head_greedy
 * (language_model.cpp:412-482).  `workspace` holds
 * mcv_lm_head_workspace_size(1) zero-filled bytes; index_dev one int64. */
template <class T>
int64_t lm_head_greedy_index(const T& x, const T& embed, void* workspace, size_t workspace_bytes, void* index_dev,
                             cudaStream_t stream) {
    detail::need_rank2(x, "lm_head_greedy_index");
    detail::need_rank2(embed, "lm_head_greedy_index");
    check(mcv_lm_head_argmax(x.data(), embed.data(), nullptr, index_dev, 1, x.shape()[1], embed.shape()[0], 0, 0,
                             workspace, workspace_bytes, stream),
          "lm_head_greedy_index");
    int64_t idx = -1;
    cudaError_t e = cudaMemcpyAsync(&idx, index_dev, sizeof(idx), cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) throw std::runtime_error(std::string("lm_head_greedy_index: ") + cudaGetErrorString(e));
    return idx;
}

/* lm_head_greedy (language_model.cpp:412-482) as the engine calls it: the raw
 * last hidden state [1,K], the final norm weight [K] (rms_norm of :423 fused
 * into the kernel), the fp16 embedding rows [V,K]; returns the token id. */
template <class T>
int64_t lm_head_greedy(const T& last_hidden, const T& final_norm_w, const T& embed, double rms_epsilon,
                       void* workspace, size_t workspace_bytes, void* index_dev, cudaStream_t stream) {
    detail::need_rank2(last_hidden, "lm_head_greedy");
    detail::need_rank2(embed, "lm_head_greedy");
    if (final_norm_w.shape().size() != 1 || final_norm_w.shape()[0] != last_hidden.shape()[1])
        throw Error(MCV_ERR_SHAPE, "lm_head_greedy: norm weight must be [hidden]");
    check(mcv_lm_head_argmax_rmsnorm(nullptr, last_hidden.data(), final_norm_w.data(), static_cast<float>(rms_epsilon),
                                     0, embed.data(), nullptr, index_dev, 1, last_hidden.shape()[1],
                                     embed.shape()[0], 0, 0, workspace, workspace_bytes, stream),
          "lm_head_greedy");
    int64_t idx = -1;
    cudaError_t e = cudaMemcpyAsync(&idx, index_dev, sizeof(idx), cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) throw std::runtime_error(std::string("lm_head_greedy: ") + cudaGetErrorString(e));
    return idx;
}

/* rms_norm (ops.h / ops.cpp:564-737): the engine's fp16 chain with (1 + gamma). */
template <class T>
void rms_norm(const T& x, const T& gamma, T& out, double epsilon, cudaStream_t stream, bool sync = false) {
    if (x.shape().empty() || x.shape() != out.shape()) throw Error(MCV_ERR_SHAPE, "rms_norm: x/out shape mismatch");
    const int64_t H = x.shape().back();
    if (gamma.shape().size() != 1 || gamma.shape()[0] != H) throw Error(MCV_ERR_SHAPE, "rms_norm: gamma must be [H]");
    int64_t rows = 1;
    for (size_t i = 0; i + 1 < x.shape().size(); ++i) rows *= x.shape()[i];
    check(mcv_rms_norm(x.data(), gamma.data(), out.data(), rows, H, static_cast<float>(epsilon), 0, stream), "rms_norm");
    finish(stream, sync, "rms_norm");
}

/* silu_mul (ops.h:41, ops.cpp:437-456). */
template <class T>
void silu_mul(const T& gate, const T& up, T& out, cudaStream_t stream, bool sync = false) {
    if (gate.shape() != up.shape() || gate.shape() != out.shape()) throw Error(MCV_ERR_SHAPE, "silu_mul shape mismatch");
    int64_t n = 1;
    for (int64_t d : gate.shape()) n *= d;
    check(mcv_silu_mul(gate.data(), up.data(), out.data(), n, stream), "silu_mul");
    finish(stream, sync, "silu_mul");
}

/* The W8A8 branch of lm_head_greedy (language_model.cpp:430-479): int8
 * embedding rows `embed_int8` [V,K] with fp16 per-row scales `embed_scale`
 * (mcv_w8a8_quantize_weight, w_layout 2), x quantized in the kernel; index
 * read back as above. */
template <class T>
int64_t lm_head_greedy_index_w8a8(const T& x, const T& embed_int8, const T& embed_scale, void* workspace,
                                  size_t workspace_bytes, void* index_dev, cudaStream_t stream) {
    detail::need_rank2(x, "lm_head_greedy_index_w8a8");
    detail::need_rank2(embed_int8, "lm_head_greedy_index_w8a8");
    check(mcv_lm_head_argmax_w8a8(x.data(), embed_int8.data(), embed_scale.data(), nullptr, index_dev, 1,
                                  x.shape()[1], embed_int8.shape()[0], 0, workspace, workspace_bytes, stream),
          "lm_head_greedy_index_w8a8");
    int64_t idx = -1;
    cudaError_t e = cudaMemcpyAsync(&idx, index_dev, sizeof(idx), cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) throw std::runtime_error(std::string("lm_head_greedy_index_w8a8: ") + cudaGetErrorString(e));
    return idx;
}

}  // namespace mcv_ops

#endif
