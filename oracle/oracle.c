/*
 * CPU oracle for the decode-matmul hot path.  TEST INFRASTRUCTURE ONLY: the
 * checker for the CUDA path and the timed CPU baseline, never shipped or
 * called by the product library.  See oracle.h for the contract and the
 * reference file:line each function restates.
 */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* fp16 <-> fp32                                                              */
/* ------------------------------------------------------------------------ */

static inline float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

float orc_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1fu;
    const uint32_t m = h & 0x3ffu;
    if (e == 0) {
        /* zero or subnormal: m * 2^-24, exact in fp32 */
        const float v = ldexpf((float)m, -24);
        return (h & 0x8000u) ? -v : v;
    }
    if (e == 31) return bits_f32(sign | 0x7f800000u | (m << 13));
    return bits_f32(sign | ((e + 112u) << 23) | (m << 13));
}

float orc_f16_to_f32_ftz(uint16_t h) {
    if (((h >> 10) & 0x1fu) == 0) return bits_f32((uint32_t)(h & 0x8000u) << 16);
    return orc_f16_to_f32(h);
}

uint16_t orc_f32_to_f16_rn(float f) {
    const uint32_t x = f32_bits(f);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t)(sign | (ax > 0x7f800000u ? 0x7e00u : 0x7c00u));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 rounds to inf */
    const uint32_t e = ax >> 23;
    if (e < 113) {
        /* result is an fp16 subnormal (or zero): round(value * 2^24) */
        if (e < 101) return sign; /* below 2^-25: rounds to zero */
        const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
        const uint32_t shift = 126u - e; /* 14..25 */
        uint32_t r = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (r & 1u))) ++r;
        return (uint16_t)(sign | r);
    }
    const uint32_t mant = ax & 0x7fffffu;
    uint32_t r = ((e - 112u) << 10) | (mant >> 13);
    const uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) ++r;
    return (uint16_t)(sign | r);
}

uint16_t orc_f32_to_f16_trunc(float f) {
    const uint32_t x = f32_bits(f);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const int32_t e = (int32_t)((x >> 23) & 0xffu) - 112;
    if (e <= 0) return sign;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    return (uint16_t)(sign | ((uint32_t)e << 10) | ((x & 0x7fffffu) >> 13));
}

static float g_h2f[65536];
static pthread_once_t g_h2f_once = PTHREAD_ONCE_INIT;
static void h2f_init(void) {
    for (uint32_t i = 0; i < 65536u; ++i) g_h2f[i] = orc_f16_to_f32((uint16_t)i);
}
static inline const float* h2f_table(void) {
    pthread_once(&g_h2f_once, h2f_init);
    return g_h2f;
}

void orc_f16_to_f32_array(const uint16_t* src, float* dst, int64_t n) {
    const float* t = h2f_table();
    for (int64_t i = 0; i < n; ++i) dst[i] = t[src[i]];
}

void orc_f32_to_f16_rn_array(const float* src, uint16_t* dst, int64_t n) {
    for (int64_t i = 0; i < n; ++i) dst[i] = orc_f32_to_f16_rn(src[i]);
}

/* ------------------------------------------------------------------------ */
/* simple POSIX-thread range splitter                                         */
/* ------------------------------------------------------------------------ */

typedef void (*range_fn)(void* ctx, int64_t begin, int64_t end, int tid);
typedef struct { range_fn fn; void* ctx; int64_t b, e; int tid; } range_job;

static void* range_tramp(void* p) {
    range_job* j = (range_job*)p;
    j->fn(j->ctx, j->b, j->e, j->tid);
    return NULL;
}

/* Splits [0,n) into nthreads contiguous, ordered ranges (range t precedes t+1). */
static void parallel_ranges(int64_t n, int nthreads, range_fn fn, void* ctx) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    if ((int64_t)nthreads > n) nthreads = n > 0 ? (int)n : 1;
    range_job jobs[256];
    pthread_t th[256];
    const int64_t chunk = (n + nthreads - 1) / nthreads;
    for (int t = 0; t < nthreads; ++t) {
        int64_t b = t * chunk, e = b + chunk;
        if (b > n) b = n;
        if (e > n) e = n;
        jobs[t] = (range_job){fn, ctx, b, e, t};
    }
    for (int t = 1; t < nthreads; ++t) pthread_create(&th[t], NULL, range_tramp, &jobs[t]);
    range_tramp(&jobs[0]);
    for (int t = 1; t < nthreads; ++t) pthread_join(th[t], NULL);
}

/* ------------------------------------------------------------------------ */
/* W4A16                                                                      */
/* ------------------------------------------------------------------------ */

/* Columns [n0,n1) of every row.  For each column the arithmetic is exactly the
 * reference checker's: per group an fp32 partial over ascending k, then
 * ref += partial * scale (tests/test_matmul_w4a16.cpp:217-227).  The loop is
 * ordered group -> k -> n so it streams rows of w; the per-column operation
 * sequence is unchanged, so results are bit-identical to the k-innermost form. */
static void w4a16_cols(const uint16_t* x, const int8_t* w, const uint16_t* s, int64_t M,
                       int64_t K, int64_t N, int64_t group, float* out, int64_t n0, int64_t n1) {
    const float* t = h2f_table();
    const int64_t G = K / group;
    const int64_t W = n1 - n0;
    if (W <= 0) return;
    float* partial = (float*)malloc(sizeof(float) * (size_t)W);
    for (int64_t m = 0; m < M; ++m) {
        float* o = out + m * N;
        for (int64_t n = n0; n < n1; ++n) o[n] = 0.0f;
        for (int64_t g = 0; g < G; ++g) {
            for (int64_t j = 0; j < W; ++j) partial[j] = 0.0f;
            for (int64_t kk = 0; kk < group; ++kk) {
                const int64_t k = g * group + kk;
                const float xk = t[x[m * K + k]];
                const int8_t* wr = w + k * N + n0;
                for (int64_t j = 0; j < W; ++j) partial[j] += xk * (float)wr[j];
            }
            const uint16_t* sr = s + g * N + n0;
            for (int64_t j = 0; j < W; ++j) o[n0 + j] += partial[j] * t[sr[j]];
        }
    }
    free(partial);
}

void orc_w4a16_gemv(const uint16_t* x, const int8_t* w_kn, const uint16_t* scales, int64_t M,
                    int64_t K, int64_t N, int64_t group, float* out) {
    w4a16_cols(x, w_kn, scales, M, K, N, group, out, 0, N);
}

typedef struct {
    const uint16_t* x; const int8_t* w; const uint16_t* s;
    int64_t M, K, N, group; float* out;
} w4a16_ctx;

static void w4a16_range(void* p, int64_t b, int64_t e, int tid) {
    (void)tid;
    w4a16_ctx* c = (w4a16_ctx*)p;
    w4a16_cols(c->x, c->w, c->s, c->M, c->K, c->N, c->group, c->out, b, e);
}

void orc_w4a16_gemv_mt(const uint16_t* x, const int8_t* w_kn, const uint16_t* scales,
                       int64_t M, int64_t K, int64_t N, int64_t group, float* out,
                       int nthreads) {
    w4a16_ctx c = {x, w_kn, scales, M, K, N, group, out};
    parallel_ranges(N, nthreads, w4a16_range, &c);
}

void orc_w4a16_fold_zeros(const uint8_t* q_kn, const uint8_t* z_gn, int64_t K, int64_t N,
                          int64_t group, int8_t* w_kn) {
    for (int64_t k = 0; k < K; ++k) {
        const int64_t g = k / group;
        for (int64_t n = 0; n < N; ++n)
            w_kn[k * N + n] = (int8_t)((int)q_kn[k * N + n] - (int)z_gn[g * N + n]);
    }
}

int orc_unpack_gptq(const int32_t* qweight, const int32_t* qzeros, const int32_t* g_idx,
                    int64_t K, int64_t N, int64_t groups, int8_t* w_kn) {
    const int64_t kpack = K / 8;
    for (int64_t kp = 0; kp < kpack; ++kp) {
        for (int64_t n = 0; n < N; ++n) {
            const uint32_t word = (uint32_t)qweight[kp * N + n];
            for (int i = 0; i < 8; ++i) {
                const int64_t k = kp * 8 + i;
                const int64_t g = g_idx[k];
                if (g < 0 || g >= groups) return -1;
                const uint32_t zw = (uint32_t)qzeros[g * (N / 8) + n / 8];
                const int zero = (int)((zw >> (4 * (n % 8))) & 0xfu) + 1;
                const int q = (int)((word >> (4 * i)) & 0xfu);
                w_kn[k * N + n] = (int8_t)(q - zero);
            }
        }
    }
    return 0;
}

void orc_unpack_awq(const int32_t* qweight, const int32_t* qzeros, int64_t K, int64_t N,
                    int64_t group, int8_t* w_kn) {
    static const int order[8] = {0, 2, 4, 6, 1, 3, 5, 7};
    const int64_t np = N / 8;
    for (int64_t k = 0; k < K; ++k) {
        const int64_t g = k / group;
        for (int64_t j = 0; j < np; ++j) {
            const uint32_t qw = (uint32_t)qweight[k * np + j];
            const uint32_t zw = (uint32_t)qzeros[g * np + j];
            for (int s = 0; s < 8; ++s) {
                const int64_t n = j * 8 + order[s];
                const int q = (int)((qw >> (4 * s)) & 0xfu);
                const int z = (int)((zw >> (4 * s)) & 0xfu);
                w_kn[k * N + n] = (int8_t)(q - z);
            }
        }
    }
}

int64_t orc_w4a16_choose_tile_len(int64_t N) {
    const int64_t block_len = (N + 7) / 8;
    const int64_t tiles = (block_len + 447) / 448;
    int64_t t = ((block_len + tiles - 1) / tiles + 15) / 16 * 16;
    return t < 16 ? 16 : t;
}

int64_t orc_w4a16_tile_rows(int64_t K, int64_t N, int64_t tile_len) {
    const int64_t block_len = (N + 7) / 8;
    const int64_t tiles_per_block = (block_len + tile_len - 1) / tile_len;
    return (K / 128) * 8 * tiles_per_block * 128;
}

void orc_w4a16_pack_tiles(const int8_t* w_kn, int64_t K, int64_t N, int64_t tile_len,
                          int8_t* packed) {
    const int64_t G = 128, groups = K / G;
    const int64_t block_len = (N + 7) / 8;
    const int64_t tpb = (block_len + tile_len - 1) / tile_len;
    memset(packed, 0, (size_t)(orc_w4a16_tile_rows(K, N, tile_len) * tile_len));
    for (int64_t g = 0; g < groups; ++g)
        for (int64_t b = 0; b < 8; ++b) {
            const int64_t bstart = b * block_len;
            int64_t bvalid = N - bstart;
            if (bvalid > block_len) bvalid = block_len;
            if (bvalid < 0) bvalid = 0;
            for (int64_t t = 0; t < tpb; ++t) {
                const int64_t tstart = t * tile_len;
                int64_t tvalid = bvalid - tstart;
                if (tvalid > tile_len) tvalid = tile_len;
                if (tvalid < 0) tvalid = 0;
                const int64_t base = (((g * 8 + b) * tpb + t) * G) * tile_len;
                for (int64_t kk = 0; kk < G; ++kk)
                    for (int64_t i = 0; i < tvalid; ++i)
                        packed[base + kk * tile_len + i] =
                            w_kn[(g * G + kk) * N + bstart + tstart + i];
            }
        }
}

void orc_w4a16_unpack_tiles(const int8_t* packed, int64_t K, int64_t N, int64_t tile_len, int8_t* w_kn) {
    const int64_t G = 128, groups = K / G;
    const int64_t block_len = (N + 7) / 8;
    const int64_t tpb = (block_len + tile_len - 1) / tile_len;
    for (int64_t g = 0; g < groups; ++g)
        for (int64_t b = 0; b < 8; ++b) {
            const int64_t bstart = b * block_len;
            int64_t bvalid = N - bstart;
            if (bvalid > block_len) bvalid = block_len;
            if (bvalid < 0) bvalid = 0;
            for (int64_t t = 0; t < tpb; ++t) {
                const int64_t tstart = t * tile_len;
                int64_t tvalid = bvalid - tstart;
                if (tvalid > tile_len) tvalid = tile_len;
                if (tvalid < 0) tvalid = 0;
                const int64_t base = (((g * 8 + b) * tpb + t) * G) * tile_len;
                for (int64_t kk = 0; kk < G; ++kk)
                    for (int64_t i = 0; i < tvalid; ++i)
                        w_kn[(g * G + kk) * N + bstart + tstart + i] = packed[base + kk * tile_len + i];
            }
        }
}

/* ------------------------------------------------------------------------ */
/* dense fp16 GEMV and the lm_head argmax                                     */
/* ------------------------------------------------------------------------ */

static inline float w_at(const float* t, const uint16_t* w, int64_t K, int64_t N, int layout,
                         int64_t k, int64_t n) {
    return layout == 0 ? t[w[n * K + k]] : t[w[k * N + n]];
}

void orc_gemv_f16(const uint16_t* x, const uint16_t* w, int64_t M, int64_t K, int64_t N,
                  int w_layout, float* out) {
    const float* t = h2f_table();
    for (int64_t m = 0; m < M; ++m)
        for (int64_t n = 0; n < N; ++n) {
            float acc = 0.0f;
            for (int64_t k = 0; k < K; ++k) acc += t[x[m * K + k]] * w_at(t, w, K, N, w_layout, k, n);
            out[m * N + n] = acc;
        }
}

uint64_t orc_argmax_key(float logit, uint32_t index) {
    uint32_t u = f32_bits(logit + 0.0f);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    if (logit != logit) u = 0u; /* NaN never wins a strict '>' scan */
    return ((uint64_t)u << 32) | (uint64_t)(0xffffffffu - index);
}

typedef struct { float best, second; int64_t idx; } top2;

/* Rows [n0,n1) for output row m, keeping the first maximum (strict '>') and
 * the runner-up value.  Eight rows are evaluated together, each with its own
 * accumulator summed over ascending k, so every logit is bit-identical to
 * the one-row-at-a-time checker loop. */
static top2 lm_rows(const float* t, const uint16_t* x, const uint16_t* w, int64_t K, int64_t N,
                    int layout, int fp16_logits, int64_t m, int64_t n0, int64_t n1) {
    top2 r = {-INFINITY, -INFINITY, -1};
    float* xf = (float*)malloc(sizeof(float) * (size_t)K);
    for (int64_t k = 0; k < K; ++k) xf[k] = t[x[m * K + k]];
    int64_t n = n0;
    for (; n < n1; n += 8) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        const int64_t cnt = (n1 - n) < 8 ? (n1 - n) : 8;
        if (layout == 0) {
            for (int64_t j = 0; j < cnt; ++j) {
                const uint16_t* wr = w + (n + j) * K;
                float a = 0.0f;
                for (int64_t k = 0; k < K; ++k) a += xf[k] * t[wr[k]];
                acc[j] = a;
            }
        } else {
            for (int64_t k = 0; k < K; ++k)
                for (int64_t j = 0; j < cnt; ++j) acc[j] += xf[k] * t[w[k * N + n + j]];
        }
        for (int64_t j = 0; j < cnt; ++j) {
            float v = acc[j];
            if (fp16_logits) v = t[orc_f32_to_f16_rn(v)];
            if (v > r.best) {
                r.second = r.best;
                r.best = v;
                r.idx = n + j;
            } else if (v > r.second) {
                r.second = v;
            }
        }
    }
    free(xf);
    return r;
}

static void finish_top2(top2 r, int64_t n_offset, int64_t* idx, float* best, float* gap) {
    if (idx) *idx = r.idx < 0 ? -1 : r.idx + n_offset;
    if (best) *best = r.best;
    if (gap) *gap = r.best - r.second;
}

void orc_lm_head_argmax(const uint16_t* x, const uint16_t* w, int64_t M, int64_t K, int64_t N,
                        int w_layout, int fp16_logits, int64_t n_offset, int64_t* out_idx,
                        float* out_best, float* out_gap) {
    const float* t = h2f_table();
    for (int64_t m = 0; m < M; ++m) {
        top2 r = lm_rows(t, x, w, K, N, w_layout, fp16_logits, m, 0, N);
        finish_top2(r, n_offset, out_idx ? out_idx + m : NULL, out_best ? out_best + m : NULL,
                    out_gap ? out_gap + m : NULL);
    }
}

typedef struct {
    const uint16_t* x; const uint16_t* w; int64_t K, N; int layout, fp16; int64_t m;
    top2 part[256];
} lm_ctx;

static void lm_range(void* p, int64_t b, int64_t e, int tid) {
    lm_ctx* c = (lm_ctx*)p;
    c->part[tid] = lm_rows(h2f_table(), c->x, c->w, c->K, c->N, c->layout, c->fp16, c->m, b, e);
}

void orc_lm_head_argmax_mt(const uint16_t* x, const uint16_t* w, int64_t M, int64_t K,
                           int64_t N, int w_layout, int fp16_logits, int64_t n_offset,
                           int64_t* out_idx, float* out_best, float* out_gap, int nthreads) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    lm_ctx* c = (lm_ctx*)calloc(1, sizeof(lm_ctx));
    c->x = x; c->w = w; c->K = K; c->N = N; c->layout = w_layout; c->fp16 = fp16_logits;
    for (int64_t m = 0; m < M; ++m) {
        for (int i = 0; i < 256; ++i) c->part[i] = (top2){-INFINITY, -INFINITY, -1};
        c->m = m;
        parallel_ranges(N, nthreads, lm_range, c);
        /* merge in range order; strict '>' keeps the earliest maximum */
        top2 r = {-INFINITY, -INFINITY, -1};
        for (int i = 0; i < 256; ++i) {
            const top2 q = c->part[i];
            if (q.idx < 0) continue;
            if (q.best > r.best) {
                r.second = r.best > q.second ? r.best : q.second;
                r.best = q.best;
                r.idx = q.idx;
            } else {
                const float cand = q.best;
                if (cand > r.second) r.second = cand;
            }
        }
        finish_top2(r, n_offset, out_idx ? out_idx + m : NULL, out_best ? out_best + m : NULL,
                    out_gap ? out_gap + m : NULL);
    }
    free(c);
}

/* ------------------------------------------------------------------------ */
/* W8A8                                                                       */
/* ------------------------------------------------------------------------ */

void orc_w8a8_quantize(const uint16_t* x, int64_t M, int64_t K, int8_t* xq,
                       uint16_t* x_scale_f16) {
    const float* t = h2f_table();
    for (int64_t m = 0; m < M; ++m) {
        const uint16_t* xr = x + m * K;
        float max_abs = 0.0f;
        for (int64_t i = 0; i < K; ++i) {
            float v = t[xr[i]];
            if (v < 0.0f) v = -v;
            if (v > max_abs) max_abs = v;
        }
        float scale = max_abs / 127.0f;
        if (scale < 0.00000001f) scale = 0.00000001f;
        const float inv = 1.0f / scale;
        for (int64_t i = 0; i < K; ++i) {
            float v = t[xr[i]] * inv;
            if (v > 127.0f) v = 127.0f;
            if (v < -128.0f) v = -128.0f;
            const int32_t q = (int32_t)(v >= 0.0f ? v + 0.5f : v - 0.5f);
            xq[m * K + i] = (int8_t)q;
        }
        x_scale_f16[m] = orc_f32_to_f16_rn(scale);
    }
}

static void w8a8_gemm_cols(const int8_t* xq, const int8_t* w, int64_t M, int64_t K, int64_t N,
                           int32_t* acc, int64_t n0, int64_t n1) {
    for (int64_t m = 0; m < M; ++m) {
        int32_t* a = acc + m * N;
        for (int64_t n = n0; n < n1; ++n) a[n] = 0;
        for (int64_t k = 0; k < K; ++k) {
            const int32_t xv = xq[m * K + k];
            const int8_t* wr = w + k * N;
            for (int64_t n = n0; n < n1; ++n) a[n] += xv * (int32_t)wr[n];
        }
    }
}

void orc_w8a8_gemm_i32(const int8_t* xq, const int8_t* w_kn, int64_t M, int64_t K, int64_t N,
                       int32_t* acc) {
    w8a8_gemm_cols(xq, w_kn, M, K, N, acc, 0, N);
}

static void w8a8_dequant_cols(const int32_t* acc, const uint16_t* xs, const uint16_t* ws,
                              int64_t M, int64_t N, uint16_t* out, int64_t n0, int64_t n1) {
    const float* t = h2f_table();
    for (int64_t m = 0; m < M; ++m) {
        const float x_scale = t[xs[m]];
        for (int64_t n = n0; n < n1; ++n) {
            float v = (float)acc[m * N + n] * t[ws[n]];
            v = v * x_scale;
            out[m * N + n] = orc_f32_to_f16_rn(v);
        }
    }
}

void orc_w8a8_dequant(const int32_t* acc, const uint16_t* x_scale, const uint16_t* w_scale,
                      int64_t M, int64_t N, uint16_t* out) {
    w8a8_dequant_cols(acc, x_scale, w_scale, M, N, out, 0, N);
}

void orc_w8a8_fused(const uint16_t* x, const int8_t* w_kn, const uint16_t* w_scale, int64_t M,
                    int64_t K, int64_t N, int32_t* acc, uint16_t* out) {
    int8_t* xq = (int8_t*)malloc((size_t)(M * K));
    uint16_t* xs = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)M);
    orc_w8a8_quantize(x, M, K, xq, xs);
    orc_w8a8_gemm_i32(xq, w_kn, M, K, N, acc);
    orc_w8a8_dequant(acc, xs, w_scale, M, N, out);
    free(xq);
    free(xs);
}

typedef struct {
    const int8_t* xq; const uint16_t* xs; const int8_t* w; const uint16_t* ws;
    int64_t M, K, N; int32_t* acc; uint16_t* out;
} w8_ctx;

static void w8_range(void* p, int64_t b, int64_t e, int tid) {
    (void)tid;
    w8_ctx* c = (w8_ctx*)p;
    w8a8_gemm_cols(c->xq, c->w, c->M, c->K, c->N, c->acc, b, e);
    w8a8_dequant_cols(c->acc, c->xs, c->ws, c->M, c->N, c->out, b, e);
}

void orc_w8a8_fused_mt(const uint16_t* x, const int8_t* w_kn, const uint16_t* w_scale,
                       int64_t M, int64_t K, int64_t N, int32_t* acc, uint16_t* out,
                       int nthreads) {
    int8_t* xq = (int8_t*)malloc((size_t)(M * K));
    uint16_t* xs = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)M);
    orc_w8a8_quantize(x, M, K, xq, xs);
    w8_ctx c = {xq, xs, w_kn, w_scale, M, K, N, acc, out};
    parallel_ranges(N, nthreads, w8_range, &c);
    free(xq);
    free(xs);
}

static int8_t quantize_i8(float value, float inv_scale) {
    float q = value * inv_scale;
    if (q > 127.0f) q = 127.0f;
    if (q < -128.0f) q = -128.0f;
    return (int8_t)(q >= 0.0f ? q + 0.5f : q - 0.5f);
}

void orc_quantize_dense_weight_w8a8(const uint16_t* w_kn, int64_t K, int64_t N, int8_t* wq,
                                    uint16_t* w_scale) {
    const float* t = h2f_table();
    for (int64_t n = 0; n < N; ++n) {
        float max_abs = 0.0f;
        for (int64_t k = 0; k < K; ++k) {
            const float v = fabsf(t[w_kn[k * N + n]]);
            if (v > max_abs) max_abs = v;
        }
        float scale = max_abs / 127.0f;
        if (scale < 0.00000001f) scale = 0.00000001f;
        const float inv = 1.0f / scale;
        w_scale[n] = orc_f32_to_f16_trunc(scale);
        for (int64_t k = 0; k < K; ++k) wq[k * N + n] = quantize_i8(t[w_kn[k * N + n]], inv);
    }
}

/* ------------------------------------------------------------------------ */
/* rms_norm (engine chain and the fp32 custom kernel) and silu_mul           */
/* ------------------------------------------------------------------------ */

static inline uint16_t rn16(float f) { return orc_f32_to_f16_rn(f); }

void orc_rms_norm_chain(const uint16_t* x, const uint16_t* gamma, int64_t M, int64_t H, float eps,
                        uint16_t* out) {
    const float* t = h2f_table();
    for (int64_t m = 0; m < M; ++m) {
        const uint16_t* xr = x + m * H;
        double sum = 0.0; /* exact: fp16 squares span < 53 bits */
        for (int64_t h = 0; h < H; ++h) sum += (double)t[rn16(t[xr[h]] * t[xr[h]])];
        const uint16_t mean = rn16((float)sum / (float)H);
        const uint16_t ms = rn16(t[mean] + eps);
        const uint16_t rstd = rn16(1.0f / sqrtf(t[ms]));
        for (int64_t h = 0; h < H; ++h) {
            const uint16_t scaled = rn16(t[xr[h]] * t[rstd]);
            const uint16_t gp1 = rn16(t[gamma[h]] + 1.0f);
            out[m * H + h] = rn16(t[scaled] * t[gp1]);
        }
    }
}

void orc_rms_norm_fp32(const uint16_t* x, const uint16_t* gamma, int64_t M, int64_t H, float eps,
                       uint16_t* out) {
    const float* t = h2f_table();
    for (int64_t m = 0; m < M; ++m) {
        const uint16_t* xr = x + m * H;
        double sum = 0.0;
        for (int64_t h = 0; h < H; ++h) sum += (double)t[xr[h]] * (double)t[xr[h]];
        const float inv = 1.0f / sqrtf((float)sum * (1.0f / (float)H) + eps);
        for (int64_t h = 0; h < H; ++h) out[m * H + h] = rn16((t[xr[h]] * inv) * t[gamma[h]]);
    }
}

void orc_silu_mul(const uint16_t* gate, const uint16_t* up, int64_t n, uint16_t* out) {
    const float* t = h2f_table();
    for (int64_t i = 0; i < n; ++i) {
        const float g = t[gate[i]];
        const float s = g / (1.0f + expf(-g));
        out[i] = rn16(s * t[up[i]]);
    }
}
