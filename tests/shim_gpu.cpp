// Compiled and run by tests/test_cpp_shim.py (GPU part): the C++ shim
// (include/mcv_ops.hpp) driving real kernels through the reference's op
// names on a tensor type shaped like minicpmv::Tensor.  Reads its inputs from
// the directory given as argv[1] (written by the test), runs
//   matmul_w4a16 (M = 1), matmul_b_transposed (M = 3), lm_head_greedy (with
//   its final rms_norm), rms_norm, silu_mul and w8a8 quantize + i32 matmul +
//   dequant,
// and writes each result next to the inputs for the test to check against
// the CPU oracle.
#include <cuda_runtime_api.h>

#include <cstdio>
#include <fstream>
#include <string>
#include <vector>

#include "mcv_ops.hpp"

struct DevTensor {  // data() / shape() as minicpmv::Tensor (tensor.h:56-60), device memory
    void* p = nullptr;
    std::vector<int64_t> s;
    void* data() const { return p; }
    const std::vector<int64_t>& shape() const { return s; }
};

static std::string dir;

static std::vector<char> read_file(const std::string& name) {
    std::ifstream f(dir + "/" + name, std::ios::binary);
    return std::vector<char>((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
}

static DevTensor upload(const std::string& name, std::vector<int64_t> shape) {
    const auto h = read_file(name);
    DevTensor t;
    t.s = std::move(shape);
    cudaMalloc(&t.p, h.size());
    cudaMemcpy(t.p, h.data(), h.size(), cudaMemcpyHostToDevice);
    return t;
}

static DevTensor alloc(size_t bytes, std::vector<int64_t> shape) {
    DevTensor t;
    t.s = std::move(shape);
    cudaMalloc(&t.p, bytes);
    cudaMemset(t.p, 0, bytes);
    return t;
}

static void save(const std::string& name, const DevTensor& t, size_t bytes) {
    std::vector<char> h(bytes);
    cudaMemcpy(h.data(), t.p, bytes, cudaMemcpyDeviceToHost);
    std::ofstream(dir + "/" + name, std::ios::binary).write(h.data(), static_cast<std::streamsize>(bytes));
}

int main(int argc, char** argv) {
    if (argc < 2) return 2;
    dir = argv[1];
    cudaStream_t s = nullptr;
    try {
        // W4A16, K=1024, N=3584, mcv-int4 arrays packed by the test
        mcv_ops::W4A16Weight w4;
        DevTensor qw = upload("w4.qw", {}), sc = upload("w4.sc", {}), zw = upload("w4.zw", {});
        w4.qweight = qw.p, w4.scales = sc.p, w4.zeros = zw.p, w4.zero_bias = 0, w4.K = 1024, w4.N = 3584;
        DevTensor x = upload("w4.x", {1, 1024}), out = alloc(3584 * 2, {1, 3584});
        mcv_ops::matmul_w4a16(x, w4, out, s, true);
        save("w4.out", out, 3584 * 2);

        // dense fp16, weight [N,K]
        DevTensor a = upload("mm.a", {3, 1024}), b = upload("mm.b", {512, 1024}), o = alloc(3 * 512 * 2, {3, 512});
        mcv_ops::matmul_b_transposed(a, b, o, s, true);
        save("mm.out", o, 3 * 512 * 2);

        // lm_head_greedy: raw hidden, final norm weight, embedding rows
        DevTensor h = upload("lm.h", {1, 1024}), g = upload("lm.g", {1024}), e = upload("lm.e", {20000, 1024});
        DevTensor ws = alloc(mcv_lm_head_workspace_size(1), {}), idx = alloc(8, {1});
        const int64_t tok = mcv_ops::lm_head_greedy(h, g, e, 1e-6, ws.p, mcv_lm_head_workspace_size(1), idx.p, s);
        std::ofstream(dir + "/lm.tok") << tok << "\n";

        // rms_norm and silu_mul
        DevTensor n_out = alloc(1024 * 2, {1, 1024});
        mcv_ops::rms_norm(h, g, n_out, 1e-6, s, true);
        save("norm.out", n_out, 1024 * 2);
        DevTensor gt = upload("silu.g", {1, 3584}), up = upload("silu.u", {1, 3584}), so = alloc(3584 * 2, {1, 3584});
        mcv_ops::silu_mul(gt, up, so, s, true);
        save("silu.out", so, 3584 * 2);

        // W8A8: quantize x, int8 matmul on [K,N] weights, dequant
        DevTensor x8 = upload("w8.x", {1, 1024}), w8 = upload("w8.w", {1024, 1024}), ws8 = upload("w8.ws", {1024});
        DevTensor xq = alloc(1024, {1, 1024}), xs = alloc(2, {1}), acc = alloc(1024 * 4, {1, 1024}),
                  o8 = alloc(1024 * 2, {1, 1024});
        mcv_ops::w8a8_quantize(x8, xq, xs, s);
        mcv_ops::matmul_w8a8_i32(xq, w8, acc, s);
        mcv_ops::w8a8_dequant(acc, xs, ws8, o8, s, true);
        save("w8.acc", acc, 1024 * 4);
        save("w8.out", o8, 1024 * 2);
    } catch (const std::exception& ex) {
        std::printf("shim gpu error: %s\n", ex.what());
        return 1;
    }
    std::printf("shim gpu ok\n");
    return 0;
}
