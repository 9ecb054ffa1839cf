// Regenerates the reference tests' seeded inputs and evaluates their CPU
// checker formulas, writing raw little-endian arrays to <outdir>/<case>.<name>.bin.
//
// The reference's hot-path tests (tests/test_matmul_w4a16.cpp,
// test_matmul_w8a8_i32.cpp, test_w8a8_dequant.cpp, test_lm_head_pipeline.cpp,
// test_matmul_cube.cpp, test_matmul.cpp, bench/bench_matmul_w4a16.cpp) need an
// Ascend NPU, so they cannot run here.  Their inputs, however, come from
// std::mt19937 and the <random> distributions of libstdc++ (or from fixed
// modular fills) and are reproducible bit for bit with g++.  This program
// rebuilds those inputs with the same engines, distributions and draw order,
// converts them to fp16 with the tests' own truncating conversion, and runs
// each test's CPU checker formula on them.  make_golden.py commits the checker
// outputs (and input hashes) as fixtures that pin the oracle.
//
// Build: g++ -O2 -std=c++17 -ffp-contract=off gen_golden.cpp -o gen_golden
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <random>
#include <string>
#include <vector>

namespace {

std::string g_out;

template <typename T>
void dump(const std::string& name, const std::vector<T>& v) {
    const std::string path = g_out + "/" + name + ".bin";
    FILE* f = std::fopen(path.c_str(), "wb");
    if (!f) { std::perror(path.c_str()); std::exit(2); }
    if (!v.empty()) std::fwrite(v.data(), sizeof(T), v.size(), f);
    std::fclose(f);
}

// fp32 -> fp16 by truncating the mantissa, underflow to signed zero: the f2h
// helper every reference test uses (e.g. tests/test_matmul_w4a16.cpp:23-32).
uint16_t to_half_trunc(float f) {
    uint32_t b;
    std::memcpy(&b, &f, 4);
    const uint16_t sign = static_cast<uint16_t>((b >> 16) & 0x8000u);
    const int e = static_cast<int>((b >> 23) & 0xffu) - 112;
    if (e <= 0) return sign;
    if (e >= 31) return static_cast<uint16_t>(sign | 0x7c00u);
    return static_cast<uint16_t>(sign | (e << 10) | ((b & 0x7fffffu) >> 13));
}

// fp16 -> fp32 with subnormals (tests/test_matmul_w4a16.cpp:33-53).
float from_half(uint16_t h) {
    const int e = (h >> 10) & 0x1f;
    const int m = h & 0x3ff;
    float v;
    if (e == 0) v = std::ldexp(static_cast<float>(m), -24);
    else if (e == 31) v = m ? NAN : INFINITY;
    else v = std::ldexp(static_cast<float>(m | 0x400), e - 25);
    return (h & 0x8000u) ? -v : v;
}

// fp16 -> fp32 with subnormals flushed (tests/test_w8a8_dequant.cpp:24-35).
float from_half_ftz(uint16_t h) {
    if (((h >> 10) & 0x1f) == 0) return (h & 0x8000u) ? -0.0f : 0.0f;
    return from_half(h);
}

// tests/test_matmul_w4a16.cpp:172-241 (random path, no --gptq).
void case_w4a16() {
    const int K = 1024, N = 3584, G = 128, NG = K / G;
    std::mt19937 rng(0);
    std::uniform_real_distribution<float> xd(-0.3f, 0.3f);
    std::uniform_int_distribution<int> wd(-8, 7);
    std::uniform_real_distribution<float> sd(0.001f, 0.02f);
    std::vector<uint16_t> x(K);
    for (auto& v : x) v = to_half_trunc(xd(rng));
    std::vector<int8_t> w(static_cast<size_t>(K) * N);
    for (auto& v : w) v = static_cast<int8_t>(wd(rng));
    std::vector<uint16_t> s(static_cast<size_t>(NG) * N);
    for (auto& v : s) v = to_half_trunc(sd(rng));
    std::vector<float> ref(N, 0.0f);
    for (int g = 0; g < NG; ++g)
        for (int n = 0; n < N; ++n) {
            float partial = 0.0f;
            for (int kk = 0; kk < G; ++kk) {
                const int k = g * G + kk;
                partial += from_half(x[k]) * static_cast<float>(w[static_cast<size_t>(k) * N + n]);
            }
            ref[n] += partial * from_half(s[static_cast<size_t>(g) * N + n]);
        }
    dump("w4a16.x", x);
    dump("w4a16.w", w);
    dump("w4a16.s", s);
    dump("w4a16.ref", ref);
}

// bench/bench_matmul_w4a16.cpp:75-79: x = 1.0, w = 1, s = 1.0, so every
// output is exactly K.
void case_w4a16_const() {
    const int K = 1024, N = 3584, NG = K / 128;
    std::vector<uint16_t> x(K, 0x3c00);
    std::vector<int8_t> w(static_cast<size_t>(K) * N, 1);
    std::vector<uint16_t> s(static_cast<size_t>(NG) * N, 0x3c00);
    std::vector<float> ref(N, static_cast<float>(K));
    dump("w4a16_const.x", x);
    dump("w4a16_const.w", w);
    dump("w4a16_const.s", s);
    dump("w4a16_const.ref", ref);
}

// tests/test_matmul_w8a8_i32.cpp:12-56.
void case_w8a8_i32() {
    const int K = 1024, N = 3584;
    std::mt19937 rng(0);
    std::uniform_int_distribution<int> xd(-8, 7);
    std::uniform_int_distribution<int> wd(-8, 7);
    std::vector<int8_t> x(K), w(static_cast<size_t>(K) * N);
    for (auto& v : x) v = static_cast<int8_t>(xd(rng));
    for (auto& v : w) v = static_cast<int8_t>(wd(rng));
    std::vector<int32_t> ref(N);
    for (int n = 0; n < N; ++n) {
        int32_t acc = 0;
        for (int k = 0; k < K; ++k) acc += static_cast<int32_t>(x[k]) * w[static_cast<size_t>(k) * N + n];
        ref[n] = acc;
    }
    dump("w8a8_i32.x", x);
    dump("w8a8_i32.w", w);
    dump("w8a8_i32.ref", ref);
}

// tests/test_w8a8_dequant.cpp:38-64: deterministic acc / scales; the
// checker value is float(acc) * xs * ws with the ftz conversion, pass
// criterion max-abs < 0.02.
void case_w8a8_dequant() {
    const int N = 3584;
    std::vector<int32_t> acc(N);
    std::vector<uint16_t> ws(N), xs(1, to_half_trunc(0.02f));
    for (int i = 0; i < N; ++i) {
        acc[i] = i - 1024;
        ws[i] = to_half_trunc(0.01f + static_cast<float>(i % 7) * 0.001f);
    }
    std::vector<float> ref(N);
    for (int i = 0; i < N; ++i)
        ref[i] = static_cast<float>(acc[i]) * from_half_ftz(xs[0]) * from_half_ftz(ws[i]);
    dump("w8a8_dequant.acc", acc);
    dump("w8a8_dequant.ws", ws);
    dump("w8a8_dequant.xs", xs);
    dump("w8a8_dequant.ref", ref);
}

// tests/test_lm_head_pipeline.cpp:50-120: hidden [4,64], weight [64,128]
// (natural [K,N]), fp32 dot in ascending k, strict '>' argmax.
void case_lm_head() {
    const int64_t Nr = 4, H = 64, V = 128;
    std::vector<uint16_t> hidden(Nr * H), weight(H * V);
    for (int64_t i = 0; i < Nr * H; ++i) {
        const float v = static_cast<float>((i * 13 + 7) % 31) / 31.0f - 0.5f;
        hidden[i] = to_half_trunc(v * 0.25f);
    }
    for (int64_t i = 0; i < H * V; ++i) {
        const float v = static_cast<float>((i * 17 + 3) % 29) / 29.0f - 0.5f;
        weight[i] = to_half_trunc(v * 0.5f);
    }
    std::vector<int64_t> tokens(Nr);
    for (int64_t n = 0; n < Nr; ++n) {
        float best = -INFINITY;
        int64_t arg = -1;
        for (int64_t v = 0; v < V; ++v) {
            float acc = 0.0f;
            for (int64_t h = 0; h < H; ++h) acc += from_half(hidden[n * H + h]) * from_half(weight[h * V + v]);
            if (acc > best) { best = acc; arg = v; }
        }
        tokens[n] = arg;
    }
    dump("lm_head.x", hidden);
    dump("lm_head.w", weight);
    dump("lm_head.ref", tokens);
}

// tests/test_matmul_cube.cpp:42-51: mt19937(42), U(-0.5,0.5), x [1,1024]
// then w [N,1024]; that test diffs against the stock library matmul, so
// the checker here is the fp32 ascending-k dot of tests/test_matmul.cpp:88-92.
void case_cube() {
    const int N = 3584, K = 1024;
    std::mt19937 rng(42);
    std::uniform_real_distribution<float> dist(-0.5f, 0.5f);
    std::vector<uint16_t> x(K), w(static_cast<size_t>(N) * K);
    for (auto& v : x) v = to_half_trunc(dist(rng));
    for (auto& v : w) v = to_half_trunc(dist(rng));
    std::vector<float> ref(N);
    for (int n = 0; n < N; ++n) {
        float acc = 0.0f;
        for (int k = 0; k < K; ++k) acc += from_half(x[k]) * from_half(w[static_cast<size_t>(n) * K + k]);
        ref[n] = acc;
    }
    dump("cube.x", x);
    dump("cube.w_nk", w);
    dump("cube.ref", ref);
}

// tests/test_matmul.cpp:53-110 cases (M,K,N) = (4,128,64) and (1,1024,4096):
// modular fills, B natural [K,N], checker fp32 ascending k.
void case_matmul(int64_t M, int64_t K, int64_t N) {
    std::vector<uint16_t> a(M * K), b(K * N);
    for (int64_t i = 0; i < M * K; ++i) a[i] = to_half_trunc(static_cast<float>((i % 7) - 3) * 0.125f);
    for (int64_t i = 0; i < K * N; ++i) b[i] = to_half_trunc(static_cast<float>((i % 5) - 2) * 0.0625f);
    std::vector<float> ref(M * N);
    for (int64_t m = 0; m < M; ++m)
        for (int64_t n = 0; n < N; ++n) {
            float acc = 0.0f;
            for (int64_t k = 0; k < K; ++k) acc += from_half(a[m * K + k]) * from_half(b[k * N + n]);
            ref[m * N + n] = acc;
        }
    const std::string tag = "matmul_" + std::to_string(M) + "x" + std::to_string(K) + "x" + std::to_string(N);
    dump(tag + ".x", a);
    dump(tag + ".w_kn", b);
    dump(tag + ".ref", ref);
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 2) {
        std::fprintf(stderr, "usage: %s <outdir>\n", argv[0]);
        return 2;
    }
    g_out = argv[1];
    case_w4a16();
    case_w4a16_const();
    case_w8a8_i32();
    case_w8a8_dequant();
    case_lm_head();
    case_cube();
    case_matmul(4, 128, 64);
    case_matmul(1, 1024, 4096);
    return 0;
}
