/*
 * CPU oracle for the decode-matmul hot path.  TEST INFRASTRUCTURE ONLY.
 *
 * This library restates, in plain C, the CPU reference arithmetic that the
 * reference engine (lvyufeng/minicpm-v-4.6-orangepi) uses to check its own
 * device kernels, plus its host-side weight packers.  It is the checker for
 * the CUDA path and the timed CPU baseline; nothing in the shipped library
 * links or calls it.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline legs may load it.
 *
 * Parity pin: the reference cannot be built or run here (its kernels are
 * AscendC and its host code includes the CANN runtime headers).  The oracle
 * is pinned against the reference tests' own seeded inputs and checker
 * formulas (tests/golden/gen_golden.cpp regenerates them with libstdc++'s
 * std::mt19937 exactly as the reference tests do) and against analytic known
 * answers (constant inputs of bench/bench_matmul_w4a16.cpp).
 *
 * Every function cites the reference file:line whose arithmetic it restates.
 * Compile with -O3 -ffp-contract=off so fp32 operation order is as written.
 */
#ifndef MCV_ORACLE_H
#define MCV_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- fp16 <-> fp32 bit conversions ------------------------------------ */
/* Full IEEE half -> float, subnormals included
 * (src/csrc/lib/quantized_weight.cpp:162-184). */
float orc_f16_to_f32(uint16_t h);
/* Half -> float with subnormal inputs flushed to signed zero
 * (tests/test_w8a8_dequant.cpp:24-35). */
float orc_f16_to_f32_ftz(uint16_t h);
/* Float -> half, IEEE round-to-nearest-even with subnormals and overflow to
 * inf.  This is the rounding of an fp32 -> fp16 hardware cast (CAST_RINT in
 * op_kernel/w8a8_dequant_custom.cpp:58, static_cast<half> in
 * op_kernel/w8a8_quantize_custom.cpp:40). */
uint16_t orc_f32_to_f16_rn(float f);
/* Float -> half by mantissa truncation with underflow to signed zero, the
 * reference's host helper (quantized_weight.cpp:186-195, and the f2h of every
 * reference test, e.g. tests/test_matmul_w4a16.cpp:23-32). */
uint16_t orc_f32_to_f16_trunc(float f);
void orc_f16_to_f32_array(const uint16_t* src, float* dst, int64_t n);
void orc_f32_to_f16_rn_array(const float* src, uint16_t* dst, int64_t n);

/* ---- W4A16 ------------------------------------------------------------- */
/* out[m,n] = sum_g fp32( sum_{k in g} x[m,k] * w[k,n] ) * s[g,n]
 * with w = (q - z) held as int8 [K,N], scales fp16 [K/group, N].  Per group
 * the fp32 partial is summed in ascending k, then partial*scale is added to
 * the running fp32 sum in ascending g: tests/test_matmul_w4a16.cpp:217-227
 * (same formula tests/test_matmul_awq.cpp:205-215), extended to M rows. */
void orc_w4a16_gemv(const uint16_t* x, const int8_t* w_kn, const uint16_t* scales,
                    int64_t M, int64_t K, int64_t N, int64_t group, float* out);
/* Same result, rows of N split over nthreads POSIX threads (CPU baseline). */
void orc_w4a16_gemv_mt(const uint16_t* x, const int8_t* w_kn, const uint16_t* scales,
                       int64_t M, int64_t K, int64_t N, int64_t group, float* out,
                       int nthreads);
/* w[k,n] = q[k,n] - z[k/group, n] from unsigned 4-bit values held one per
 * byte (synthetic configs: q, z in 0..15). */
void orc_w4a16_fold_zeros(const uint8_t* q_kn, const uint8_t* z_gn, int64_t K, int64_t N,
                          int64_t group, int8_t* w_kn);
/* GPTQ unpack: qweight int32 [K/8, N] (nibble i of word = k%8 == i), qzeros
 * int32 [G, N/8] (nibble n%8), g_idx [K]; w = q - (zero + 1).
 * src/csrc/lib/quantized_weight.cpp:75-120.  Returns 0, or -1 when g_idx is
 * out of range (the reference throws). */
int orc_unpack_gptq(const int32_t* qweight, const int32_t* qzeros, const int32_t* g_idx,
                    int64_t K, int64_t N, int64_t groups, int8_t* w_kn);
/* AWQ unpack: qweight int32 [K, N/8], qzeros int32 [G, N/8]; slot s of a
 * word holds column j*8 + {0,2,4,6,1,3,5,7}[s]; w = q - z.
 * src/csrc/lib/quantized_weight.cpp:17, 122-160. */
void orc_unpack_awq(const int32_t* qweight, const int32_t* qzeros, int64_t K, int64_t N,
                    int64_t group, int8_t* w_kn);
/* The reference's tile-packed int8 layout for its 8-core kernel
 * (quantized_weight.cpp:41-73): tile_len choice and the pack itself.
 * packed must hold orc_w4a16_tile_rows(K,N,tile_len)*tile_len bytes. */
int64_t orc_w4a16_choose_tile_len(int64_t N);
int64_t orc_w4a16_tile_rows(int64_t K, int64_t N, int64_t tile_len);
void orc_w4a16_pack_tiles(const int8_t* w_kn, int64_t K, int64_t N, int64_t tile_len,
                          int8_t* packed);
/* The inverse: tile-packed [rows][tile_len] back to w [K,N]. */
void orc_w4a16_unpack_tiles(const int8_t* packed, int64_t K, int64_t N, int64_t tile_len, int8_t* w_kn);

/* ---- dense fp16 GEMV / lm_head ----------------------------------------- */
/* out[m,n] = fp32 sum over ascending k of x[m,k]*w(k,n); w_layout 0 = [N,K]
 * (row n contiguous, the tied-embedding layout), 1 = [K,N] natural.
 * Restates tests/test_matmul.cpp:88-92 and tests/test_lm_head_pipeline.cpp:99-101. */
void orc_gemv_f16(const uint16_t* x, const uint16_t* w, int64_t M, int64_t K, int64_t N,
                  int w_layout, float* out);
/* Greedy argmax over the logits of x[m,:] . w: fp32 dot in ascending k, then
 * strict '>' so the first maximum wins (tests/test_lm_head_pipeline.cpp:95-107).
 * fp16_logits != 0 rounds each logit to fp16 first, as the production
 * lm_head_greedy does after its D2H copy (src/csrc/lib/language_model.cpp:471-479).
 * Also returns the winning logit and the gap to the runner-up (for ambiguity
 * checks).  Rows n in [0,N) get global index n_offset + n. */
void orc_lm_head_argmax(const uint16_t* x, const uint16_t* w, int64_t M, int64_t K, int64_t N,
                        int w_layout, int fp16_logits, int64_t n_offset,
                        int64_t* out_idx, float* out_best, float* out_gap);
void orc_lm_head_argmax_mt(const uint16_t* x, const uint16_t* w, int64_t M, int64_t K,
                           int64_t N, int w_layout, int fp16_logits, int64_t n_offset,
                           int64_t* out_idx, float* out_best, float* out_gap, int nthreads);

/* ---- W8A8 ---------------------------------------------------------------- */
/* Per-row symmetric absmax quantization, the scalar loop of
 * op_kernel/w8a8_quantize_custom.cpp:25-41 applied to each of M rows:
 * scale = max|x|/127 (fp32), clamped to >= 1e-8, inv = 1/scale,
 * q = (int)(clamp(x*inv, -128, 127) +/- 0.5), x_scale stored as fp16 (RN). */
void orc_w8a8_quantize(const uint16_t* x, int64_t M, int64_t K, int8_t* xq,
                       uint16_t* x_scale_f16);
/* int32 out[m,n] = sum_k x[m,k]*w[k,n], w int8 [K,N]
 * (tests/test_matmul_w8a8_i32.cpp:39-45). */
void orc_w8a8_gemm_i32(const int8_t* xq, const int8_t* w_kn, int64_t M, int64_t K, int64_t N,
                       int32_t* acc);
/* out = fp16_rn((float(acc) * float(w_scale[n])) * float(x_scale[m]))
 * (op_kernel/w8a8_dequant_custom.cpp:52-59). */
void orc_w8a8_dequant(const int32_t* acc, const uint16_t* x_scale, const uint16_t* w_scale,
                      int64_t M, int64_t N, uint16_t* out);
/* quantize -> int32 GEMM -> dequant in one call (the dispatcher's W8A8 branch,
 * src/csrc/lib/decoder_layer.cpp:226-232 with 216-224). */
void orc_w8a8_fused(const uint16_t* x, const int8_t* w_kn, const uint16_t* w_scale,
                    int64_t M, int64_t K, int64_t N, int32_t* acc, uint16_t* out);
void orc_w8a8_fused_mt(const uint16_t* x, const int8_t* w_kn, const uint16_t* w_scale,
                       int64_t M, int64_t K, int64_t N, int32_t* acc, uint16_t* out,
                       int nthreads);
/* Per-output-channel weight quantization of an fp16 [K,N] matrix
 * (src/csrc/lib/quantized_weight.cpp:231-268): scale stored by the
 * truncating f32->f16 helper, values by round-half-away quantize_i8
 * (quantized_weight.cpp:197-202) using the fp32 reciprocal of the fp32 scale. */
void orc_quantize_dense_weight_w8a8(const uint16_t* w_kn, int64_t K, int64_t N,
                                    int8_t* wq, uint16_t* w_scale);

/* ---- misc ---------------------------------------------------------------- */
/* Order-preserving 64-bit argmax key: (ordered fp32 bits << 32) |
 * (0xFFFFFFFF - index); a larger key means a larger logit, ties going to the
 * smaller index (the first-max rule above).  -0 is canonicalised to +0. */
uint64_t orc_argmax_key(float logit, uint32_t index);


/* ---- neighbours of the GEMVs: rms_norm and silu_mul -------------------- */
/* The engine's rms_norm (src/csrc/lib/ops.cpp:564-737), which lm_head_greedy
 * applies before the lm_head (src/csrc/lib/language_model.cpp:423) and every
 * decoder layer before its projections: a chain of fp16 tensor ops, each
 * result rounded to fp16 - x_sq = x*x; mean over the row; + eps; rsqrt;
 * x * rstd; gamma + 1; (x * rstd) * (gamma + 1).  The mean's sum is taken
 * exactly (a double sum of fp16 squares, which no order changes) and then
 * rounded through fp32 to fp16: the reference's aclnnMean leaves the
 * accumulation order unspecified. */
void orc_rms_norm_chain(const uint16_t* x, const uint16_t* gamma, int64_t M, int64_t H, float eps,
                        uint16_t* out);
/* The rms_norm1024 custom kernel (op_kernel/rms_norm1024_custom.cpp:57-70):
 * fp32 throughout, inv = 1 / sqrt(sum(x^2) / H + eps), out = RN(x * inv * gamma)
 * (gamma itself, no +1); the sum of squares is taken in double. */
void orc_rms_norm_fp32(const uint16_t* x, const uint16_t* gamma, int64_t M, int64_t H, float eps,
                       uint16_t* out);
/* silu_mul (op_kernel/silu_mul_custom.cpp:63-72): fp32
 * s = g / (1 + exp(-g)), out = RN(s * u). */
void orc_silu_mul(const uint16_t* gate, const uint16_t* up, int64_t n, uint16_t* out);

#ifdef __cplusplus
}
#endif
#endif
