// Per-projection decode dispatch and the W8A8 decode policy: which of a
// projection's weight formats a decode-time matmul runs on.
//
// Reference: matmul_decode_dispatch / w8a8_weight_ready
// (src/csrc/lib/decoder_layer.cpp:212-244) and the MINICPM_W8A8_DECODE
// policy (src/csrc/lib/language_model.cpp:19-41, decoder_layer.cpp:19-25).
// The policy string is read from the environment once per process, as the
// reference's function-local statics do; mcv_set_w8a8_decode_mode replaces it
// for callers that configure the engine programmatically.
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"

namespace mcv {
namespace {

std::mutex g_policy_mu;
bool g_policy_loaded = false;
bool g_policy_set = false;  // the variable exists (possibly empty)
std::string g_policy_mode;

void load_policy_locked() {
    if (!g_policy_loaded) {
        const char* v = std::getenv("MINICPM_W8A8_DECODE");
        g_policy_mode = v ? v : "";
        g_policy_set = v != nullptr;
        g_policy_loaded = true;
    }
}

std::string policy_mode() {
    std::lock_guard<std::mutex> lock(g_policy_mu);
    load_policy_locked();
    return g_policy_mode;
}

// decoder_layer.cpp:19-25: the per-layer decode gate is "set, and neither
// "0" nor "false"", so a set-but-empty variable turns W8A8 decode on there,
// while language_model.cpp:27-30 (the lm_head policy) treats it as off.
bool decode_gate_enabled() {
    std::lock_guard<std::mutex> lock(g_policy_mu);
    load_policy_locked();
    return g_policy_set && g_policy_mode != "0" && g_policy_mode != "false";
}

// language_model.cpp:27-30
bool mode_enabled(const std::string& mode) { return !mode.empty() && mode != "0" && mode != "false"; }

// language_model.cpp:32-41
bool mode_allows(const std::string& mode, const char* token) {
    if (!mode_enabled(mode)) return false;
    if (mode == "all") return true;
    const std::string t(token);
    if (mode == "1" || mode == "selective") return t == "lm_head";
    return mode.find(t) != std::string::npos;
}

}  // namespace
}  // namespace mcv

using namespace mcv;

extern "C" {

int mcv_set_w8a8_decode_mode(const char* mode) {
    std::lock_guard<std::mutex> lock(g_policy_mu);
    if (mode) {
        g_policy_mode = mode;
        g_policy_set = true;
        g_policy_loaded = true;
    } else {
        g_policy_loaded = false;  // back to the environment on the next query
    }
    return MCV_OK;
}

int mcv_w8a8_decode_enabled(void) { return mode_enabled(policy_mode()) ? 1 : 0; }

int mcv_w8a8_decode_gate_enabled(void) { return decode_gate_enabled() ? 1 : 0; }

int mcv_w8a8_policy_allows(const char* token) {
    if (!token) return 0;
    return mode_allows(policy_mode(), token) ? 1 : 0;
}

int mcv_w8a8_policy_allows_mode(const char* mode, const char* token) {
    if (!token) return 0;
    return mode_allows(mode ? std::string(mode) : std::string(), token) ? 1 : 0;
}

int mcv_matmul_decode_dispatch(const void* x, const mcv_decode_weights* w, void* out, int64_t M, int64_t K,
                               int64_t N, mcv_stream_t stream) {
    if (!x || !w || !out) return fail(MCV_ERR_NULL, "matmul_decode_dispatch: null pointer");
    if (M < 1) return fail(MCV_ERR_SHAPE, "matmul_decode_dispatch: M must be >= 1");
    // decoder_layer.cpp:212-214, 232: W8A8 when the decode gate is on, the
    // weight exists and the input is one row
    const bool w8_ready = decode_gate_enabled() && w->w8_weight != nullptr && w->w8_scale != nullptr;
    if (w8_ready && M == 1)
        return mcv_w8a8_fused(x, w->w8_weight, w->w8_scale, out, nullptr, nullptr, nullptr, M, K, N, 0, stream);
    // decoder_layer.cpp:239-242: W4A16 for one row; more rows go to the
    // dense weight, or - where there is none - stay on the int4 weights
    // (the GEMV up to 32 rows, or 64 with K <= 4096 - B200, K = 1024, N = 3584:
    // 3.9 / 5.0 us at M = 48 / 64 against 7.0 / 7.2 on the tensor-core GEMM,
    // which wins at K = 8192 - the GEMM beyond)
    const bool have_w4 = w->w4_qweight != nullptr && w->w4_scales != nullptr && w->w4_zeros != nullptr;
    if (have_w4 && (M == 1 || w->dense == nullptr)) {
        if (M <= 32 || (M <= 64 && K <= 4096))
            return mcv_w4a16_gemv(x, w->w4_qweight, w->w4_scales, w->w4_zeros, w->w4_zero_bias, out, M, K, N, 128,
                                  stream);
        return mcv_w4a16_gemm(x, w->w4_qweight, w->w4_scales, w->w4_zeros, w->w4_zero_bias, out, M, K, N, 128,
                              stream);
    }
    if (!w->dense) return fail(MCV_ERR_NULL, "matmul_decode_dispatch: no weight usable for this call");
    // decoder_layer.cpp:243: the dense fp16 weight - GEMV up to 8 rows, the
    // tensor-core GEMM beyond (which takes the [N][K] layout)
    if (M <= 8) return mcv_gemv_f16(x, w->dense, out, M, K, N, w->dense_layout, stream);
    if (w->dense_layout != 0)
        return fail(MCV_ERR_SHAPE, "matmul_decode_dispatch: M > 8 on a dense weight needs the [N][K] layout "
                                   "(mcv_transpose_f16 at load time)");
    return mcv_gemm_f16(x, w->dense, out, M, K, N, stream);
}

}  // extern "C"
