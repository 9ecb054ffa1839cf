// Compiled and run by tests/test_cpp_shim.py: the C++ shim (include/mcv_ops.hpp)
// binds to a tensor type shaped like the reference's minicpmv::Tensor and turns
// statuses into exceptions.  Every call here is refused on the host before any
// device work, so it needs no GPU.
#include <cstdio>
#include <vector>

#include "mcv_ops.hpp"

struct FakeTensor {  // data() / shape() as minicpmv::Tensor (tensor.h:56-60)
    void* p = nullptr;
    std::vector<int64_t> s;
    void* data() const { return p; }
    const std::vector<int64_t>& shape() const { return s; }
};

template <class F>
int expect_status(F f, int want, const char* what) {
    try {
        f();
    } catch (const mcv_ops::Error& e) {
        if (e.status() == want) return 0;
        std::printf("%s: status %d, want %d (%s)\n", what, e.status(), want, e.what());
        return 1;
    }
    std::printf("%s: no exception\n", what);
    return 1;
}

int main() {
    cudaStream_t s = nullptr;
    FakeTensor x{nullptr, {1, 1024}}, b{nullptr, {512, 300}}, out{nullptr, {1, 512}};
    int bad = 0;
    bad += expect_status([&] { mcv_ops::matmul_b_transposed(x, b, out, s); }, MCV_ERR_SHAPE, "K mismatch");
    FakeTensor b_nk{nullptr, {512, 1024}};
    bad += expect_status([&] { mcv_ops::matmul_b_transposed(x, b_nk, out, s); }, MCV_ERR_NULL, "null dense");
    mcv_ops::W4A16Weight w4;
    w4.K = 1024, w4.N = 512;
    bad += expect_status([&] { mcv_ops::matmul_w4a16(x, w4, out, s); }, MCV_ERR_NULL, "null int4 weight");
    w4.K = 2048;
    bad += expect_status([&] { mcv_ops::matmul_w4a16(x, w4, out, s); }, MCV_ERR_SHAPE, "int4 K mismatch");
    bad += expect_status([&] { mcv_ops::argmax_last_dim(x, out, s); }, MCV_ERR_NULL, "null logits");
    FakeTensor flat{nullptr, {1024}};
    bad += expect_status([&] { mcv_ops::w8a8_quantize(flat, out, out, s); }, MCV_ERR_SHAPE, "1-D input");
    bad += expect_status([&] { mcv_ops::matmul_decode_dispatch<FakeTensor>(x, nullptr, nullptr, nullptr, out, s); },
                         MCV_ERR_NULL, "no formats");
    FakeTensor emb8{nullptr, {1000, 1024}}, emb_scale{nullptr, {1000}};
    bad += expect_status([&] { mcv_ops::lm_head_greedy_index_w8a8(x, emb8, emb_scale, nullptr, 0, nullptr, s); },
                         MCV_ERR_NULL, "w8a8 lm_head, null scales");
    if (bad == 0) std::printf("shim ok\n");
    return bad;
}
