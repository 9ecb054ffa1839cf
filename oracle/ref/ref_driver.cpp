// Runs the reference engine's own host code on this machine's CPU - its
// safetensors reader (src/csrc/lib/weights.cpp), W4A16 checkpoint loader and
// W8A8 weight quantizer (src/csrc/lib/quantized_weight.cpp) - and writes
// what it produces to files, so tests can compare this repository's loader,
// packers and quantizer with the reference's actual output.  TEST
// INFRASTRUCTURE, built by ./Makefile into ../_ref/ from the reference's
// sources where they lie; never part of the shipped library.
//
//   ref_driver names <file.safetensors>
//   ref_driver load_w4a16 <file.safetensors> <base> <out_prefix>
//       -> <out>.tiles (int8 [rows][tile_len]), <out>.scales (fp16 [G][N]),
//          <out>.meta ("K N tile_len rows")
//   ref_driver load_f16 <file.safetensors> <name> <out>      (load_to_device_as F16)
//   ref_driver quantize_w8a8 <w_kn.f16> <K> <N> <out_prefix> -> <out>.wq, <out>.ws
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <iostream>
#include <string>
#include <vector>

#include "minicpmv/quantized_weight.h"
#include "minicpmv/weights.h"

using namespace minicpmv;

static void write_file(const std::string& path, const void* p, size_t n) {
    std::ofstream f(path, std::ios::binary);
    f.write(static_cast<const char*>(p), static_cast<std::streamsize>(n));
    if (!f) throw std::runtime_error("cannot write " + path);
}

static std::vector<char> host_bytes(const Tensor& t) {
    std::vector<char> v(t.size_bytes());
    if (!v.empty()) t.copy_to_host(v.data(), v.size());
    return v;
}

int main(int argc, char** argv) {
    try {
        if (argc < 3) throw std::runtime_error("usage: ref_driver <command> ...");
        const std::string cmd = argv[1];
        if (cmd == "names") {
            WeightsIndex idx(argv[2]);
            for (const auto& n : idx.names()) std::cout << n << "\n";
            return 0;
        }
        if (cmd == "load_w4a16" && argc == 5) {
            WeightsIndex idx(argv[2]);
            const std::string base = argv[3], out = argv[4];
            if (!has_w4a16_quantized_weight(idx, base)) throw std::runtime_error("no quantized weight " + base);
            W4A16QuantizedWeight w = load_w4a16_quantized_weight(idx, base);
            const auto tiles = host_bytes(w.w_int8), scales = host_bytes(w.scales);
            write_file(out + ".tiles", tiles.data(), tiles.size());
            write_file(out + ".scales", scales.data(), scales.size());
            std::ofstream(out + ".meta") << w.K << " " << w.N << " " << w.w_int8.shape()[1] << " "
                                         << w.w_int8.shape()[0] << "\n";
            return 0;
        }
        if (cmd == "load_f16" && argc == 5) {
            WeightsIndex idx(argv[2]);
            Tensor t = idx.load_to_device_as(argv[3], DType::Float16);
            const auto b = host_bytes(t);
            write_file(argv[4], b.data(), b.size());
            return 0;
        }
        if (cmd == "quantize_w8a8" && argc == 6) {
            const int64_t K = std::atoll(argv[3]), N = std::atoll(argv[4]);
            std::vector<uint16_t> h(static_cast<size_t>(K * N));
            std::ifstream f(argv[2], std::ios::binary);
            f.read(reinterpret_cast<char*>(h.data()), static_cast<std::streamsize>(h.size() * 2));
            if (!f) throw std::runtime_error("short input");
            Tensor w({K, N}, DType::Float16);
            w.copy_from_host(h.data(), h.size() * 2);
            W8A8QuantizedWeight q = quantize_dense_weight_w8a8(w);
            const auto wq = host_bytes(q.w_int8), ws = host_bytes(q.w_scale);
            write_file(std::string(argv[5]) + ".wq", wq.data(), wq.size());
            write_file(std::string(argv[5]) + ".ws", ws.data(), ws.size());
            return 0;
        }
        throw std::runtime_error("bad command line");
    } catch (const std::exception& e) {
        std::cerr << "ref_driver: " << e.what() << "\n";
        return 2;
    }
}
