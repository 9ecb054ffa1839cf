// Checkpoint side of the W4A16 path: a safetensors reader and the GPTQ / AWQ
// loader that turns a checkpoint's quantized projection into the mcv-int4
// device layout in one call.  Host code only.
//
// Reference behaviour replaced:
//  * WeightsIndex (src/csrc/lib/weights.cpp:197-333): the safetensors file
//    (8-byte little-endian header length, a JSON header mapping tensor names
//    to {dtype, shape, data_offsets}, then the raw data), read into memory;
//    load_to_device_as's BF16 -> F16 conversion (weights.cpp:239-262, with
//    the truncating bf16_bits_to_f16_bits of :25-33);
//  * has_w4a16_quantized_weight / load_w4a16_quantized_weight
//    (src/csrc/lib/quantized_weight.cpp:204-229): `base.qweight`,
//    `base.qzeros`, `base.scales`, and `base.g_idx` for GPTQ (absent: AWQ),
//    with the dtype and shape checks of unpack_gptq_weight / unpack_awq_weight
//    (:75-160).
// Here the file is memory-mapped instead of read whole, the header is parsed
// by a small JSON reader of its own, every tensor's byte range is checked
// against its dtype and shape and against the file size, and the quantized
// projection is repacked straight from the mapping into the caller's device
// buffers (no allocation on the device; sizes from mcv_w4a16_layout_bytes).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cctype>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "common.cuh"

namespace mcv {
namespace {

struct StTensor {
    int dtype = 0;
    std::vector<int64_t> shape;
    uint64_t begin = 0, end = 0;  // absolute file offsets
};

struct StFile {
    int fd = -1;
    const unsigned char* map = nullptr;
    size_t size = 0;
    std::map<std::string, StTensor> tensors;  // sorted by name
    std::vector<std::string> names;
};

int dtype_code(const std::string& s) {
    if (s == "F16") return MCV_DT_F16;
    if (s == "BF16") return MCV_DT_BF16;
    if (s == "F32") return MCV_DT_F32;
    if (s == "F64") return MCV_DT_F64;
    if (s == "I8") return MCV_DT_I8;
    if (s == "U8") return MCV_DT_U8;
    if (s == "I16") return MCV_DT_I16;
    if (s == "I32") return MCV_DT_I32;
    if (s == "I64") return MCV_DT_I64;
    if (s == "BOOL") return MCV_DT_BOOL;
    return 0;
}

int dtype_bytes(int dt) {
    switch (dt) {
        case MCV_DT_F16: case MCV_DT_BF16: case MCV_DT_I16: return 2;
        case MCV_DT_F32: case MCV_DT_I32: return 4;
        case MCV_DT_F64: case MCV_DT_I64: return 8;
        case MCV_DT_I8: case MCV_DT_U8: case MCV_DT_BOOL: return 1;
        default: return 0;
    }
}

// A JSON reader over the header text, just large enough for safetensors:
// objects, arrays, strings (with escapes), numbers, true/false/null.
class Json {
public:
    explicit Json(const std::string& t) : t_(t) {}
    const std::string& error() const { return err_; }

    void ws() {
        while (i_ < t_.size() && std::isspace(static_cast<unsigned char>(t_[i_]))) ++i_;
    }
    bool peek(char c) {
        ws();
        return i_ < t_.size() && t_[i_] == c;
    }
    bool eat(char c) {
        if (!peek(c)) return bad(std::string("expected '") + c + "'");
        ++i_;
        return true;
    }
    bool str(std::string& out) {
        out.clear();
        if (!eat('"')) return false;
        while (i_ < t_.size() && t_[i_] != '"') {
            char c = t_[i_++];
            if (c == '\\') {
                if (i_ >= t_.size()) return bad("bad escape");
                const char e = t_[i_++];
                switch (e) {
                    case '"': case '\\': case '/': out += e; break;
                    case 'b': out += '\b'; break;
                    case 'f': out += '\f'; break;
                    case 'n': out += '\n'; break;
                    case 'r': out += '\r'; break;
                    case 't': out += '\t'; break;
                    case 'u': {
                        if (i_ + 4 > t_.size()) return bad("bad \\u escape");
                        unsigned v = 0;
                        for (int k = 0; k < 4; ++k) {
                            const char h = t_[i_++];
                            v <<= 4;
                            if (h >= '0' && h <= '9') v |= static_cast<unsigned>(h - '0');
                            else if (h >= 'a' && h <= 'f') v |= static_cast<unsigned>(h - 'a' + 10);
                            else if (h >= 'A' && h <= 'F') v |= static_cast<unsigned>(h - 'A' + 10);
                            else return bad("bad \\u escape");
                        }
                        // UTF-8 of the BMP code point (names are ASCII in practice)
                        if (v < 0x80) {
                            out += static_cast<char>(v);
                        } else if (v < 0x800) {
                            out += static_cast<char>(0xc0 | (v >> 6));
                            out += static_cast<char>(0x80 | (v & 0x3f));
                        } else {
                            out += static_cast<char>(0xe0 | (v >> 12));
                            out += static_cast<char>(0x80 | ((v >> 6) & 0x3f));
                            out += static_cast<char>(0x80 | (v & 0x3f));
                        }
                        break;
                    }
                    default: return bad("bad escape");
                }
            } else {
                out += c;
            }
        }
        if (i_ >= t_.size()) return bad("unterminated string");
        ++i_;
        return true;
    }
    bool uint(uint64_t& v) {
        ws();
        const size_t s = i_;
        v = 0;
        while (i_ < t_.size() && std::isdigit(static_cast<unsigned char>(t_[i_]))) {
            const uint64_t d = static_cast<uint64_t>(t_[i_++] - '0');
            if (v > (~0ull - d) / 10) return bad("integer overflow");
            v = v * 10 + d;
        }
        return i_ > s ? true : bad("expected an unsigned integer");
    }
    bool uint_array(std::vector<uint64_t>& out) {
        out.clear();
        if (!eat('[')) return false;
        if (peek(']')) return eat(']');
        for (;;) {
            uint64_t v;
            if (!uint(v)) return false;
            out.push_back(v);
            if (peek(',')) {
                ++i_;
                continue;
            }
            return eat(']');
        }
    }
    // Skips any value (used for __metadata__ and unknown keys).
    bool skip(int depth = 0) {
        if (depth > 64) return bad("nesting too deep");
        ws();
        if (i_ >= t_.size()) return bad("unexpected end");
        const char c = t_[i_];
        if (c == '"') {
            std::string s;
            return str(s);
        }
        if (c == '{' || c == '[') {
            const char close = c == '{' ? '}' : ']';
            ++i_;
            if (peek(close)) return eat(close);
            for (;;) {
                if (c == '{') {
                    std::string k;
                    if (!str(k) || !eat(':')) return false;
                }
                if (!skip(depth + 1)) return false;
                if (peek(',')) {
                    ++i_;
                    continue;
                }
                return eat(close);
            }
        }
        const size_t s = i_;
        while (i_ < t_.size() && (std::isalnum(static_cast<unsigned char>(t_[i_])) || t_[i_] == '-' || t_[i_] == '+' ||
                                  t_[i_] == '.'))
            ++i_;
        return i_ > s ? true : bad("unexpected character");
    }
    bool bad(const std::string& m) {
        if (err_.empty()) err_ = m + " at header byte " + std::to_string(i_);
        return false;
    }

private:
    const std::string& t_;
    size_t i_ = 0;
    std::string err_;
};

int parse_header(StFile& f) {
    if (f.size < 8) return fail(MCV_ERR_FORMAT, "safetensors: file shorter than its 8-byte header length");
    uint64_t hlen = 0;
    for (int b = 7; b >= 0; --b) hlen = (hlen << 8) | f.map[b];  // little-endian
    if (hlen > f.size - 8) return fail(MCV_ERR_FORMAT, "safetensors: header length runs past the end of the file");
    const std::string text(reinterpret_cast<const char*>(f.map + 8), static_cast<size_t>(hlen));
    const uint64_t data0 = 8 + hlen;
    Json j(text);
    auto bad = [&]() { return fail(MCV_ERR_FORMAT, "safetensors header: " + j.error()); };
    if (!j.eat('{')) return bad();
    if (j.peek('}')) {
        j.eat('}');
        return MCV_OK;
    }
    for (;;) {
        std::string name;
        if (!j.str(name) || !j.eat(':')) return bad();
        if (name == "__metadata__") {
            if (!j.skip()) return bad();
        } else {
            StTensor t;
            bool has_dt = false, has_shape = false, has_off = false;
            if (!j.eat('{')) return bad();
            if (!j.peek('}')) {
                for (;;) {
                    std::string key;
                    if (!j.str(key) || !j.eat(':')) return bad();
                    if (key == "dtype") {
                        std::string d;
                        if (!j.str(d)) return bad();
                        t.dtype = dtype_code(d);
                        if (!t.dtype) return fail(MCV_ERR_FORMAT, "safetensors: unsupported dtype " + d + " of " + name);
                        has_dt = true;
                    } else if (key == "shape") {
                        std::vector<uint64_t> v;
                        if (!j.uint_array(v)) return bad();
                        for (uint64_t d : v) {
                            if (d > (1ull << 40)) return fail(MCV_ERR_FORMAT, "safetensors: dimension too large in " + name);
                            t.shape.push_back(static_cast<int64_t>(d));
                        }
                        has_shape = true;
                    } else if (key == "data_offsets") {
                        std::vector<uint64_t> v;
                        if (!j.uint_array(v)) return bad();
                        if (v.size() != 2 || v[0] > v[1])
                            return fail(MCV_ERR_FORMAT, "safetensors: bad data_offsets of " + name);
                        t.begin = data0 + v[0];
                        t.end = data0 + v[1];
                        has_off = true;
                    } else if (!j.skip()) {
                        return bad();
                    }
                    if (j.peek(',')) {
                        j.eat(',');
                        continue;
                    }
                    break;
                }
            }
            if (!j.eat('}')) return bad();
            if (!has_dt || !has_shape || !has_off)
                return fail(MCV_ERR_FORMAT, "safetensors: entry " + name + " lacks dtype, shape or data_offsets");
            uint64_t numel = 1;
            for (int64_t d : t.shape) {
                if (d != 0 && numel > (1ull << 62) / static_cast<uint64_t>(d))
                    return fail(MCV_ERR_FORMAT, "safetensors: element count overflows in " + name);
                numel *= static_cast<uint64_t>(d);
            }
            if (t.end > f.size) return fail(MCV_ERR_FORMAT, "safetensors: data of " + name + " runs past the end of the file");
            if (t.end - t.begin != numel * static_cast<uint64_t>(dtype_bytes(t.dtype)))
                return fail(MCV_ERR_FORMAT, "safetensors: byte size of " + name + " disagrees with its dtype and shape");
            if (f.tensors.count(name)) return fail(MCV_ERR_FORMAT, "safetensors: duplicate tensor " + name);
            f.tensors.emplace(name, std::move(t));
        }
        if (j.peek(',')) {
            j.eat(',');
            continue;
        }
        break;
    }
    if (!j.eat('}')) return bad();
    for (const auto& kv : f.tensors) f.names.push_back(kv.first);
    return MCV_OK;
}

const StTensor* find(const StFile* f, const std::string& name) {
    auto it = f->tensors.find(name);
    return it == f->tensors.end() ? nullptr : &it->second;
}

// bf16 -> fp16 bits the way the reference's loader converts
// (weights.cpp:25-33): mantissa truncated, out-of-range exponents to signed
// zero or infinity.
uint16_t bf16_to_f16_trunc(uint16_t bf) {
    const uint32_t bits = static_cast<uint32_t>(bf) << 16;
    const uint16_t sign = static_cast<uint16_t>((bits >> 16) & 0x8000u);
    const int e = static_cast<int>((bits >> 23) & 0xffu) - 112;
    if (e <= 0) return sign;
    if (e >= 31) return static_cast<uint16_t>(sign | 0x7c00u);
    return static_cast<uint16_t>(sign | (e << 10) | ((bits & 0x7fffffu) >> 13));
}

// Copy of a tensor's elements into an aligned host vector.
template <class T>
std::vector<T> elements(const StFile* f, const StTensor* t) {
    std::vector<T> v((t->end - t->begin) / sizeof(T));
    if (!v.empty()) std::memcpy(v.data(), f->map + t->begin, v.size() * sizeof(T));
    return v;
}

// fp16 scales from an F16 or BF16 tensor.
std::vector<uint16_t> f16_elements(const StFile* f, const StTensor* t) {
    std::vector<uint16_t> v = elements<uint16_t>(f, t);
    if (t->dtype == MCV_DT_BF16)
        for (auto& x : v) x = bf16_to_f16_trunc(x);
    return v;
}

struct QuantTensors {
    const StTensor *q, *z, *s, *g;
    bool gptq;
    int64_t K, N;
};

int quant_tensors(const StFile* f, const char* base_c, QuantTensors& o) {
    const std::string base(base_c);
    o.q = find(f, base + ".qweight");
    o.z = find(f, base + ".qzeros");
    o.s = find(f, base + ".scales");
    o.g = find(f, base + ".g_idx");
    if (!o.q || !o.z || !o.s) return fail(MCV_ERR_VALUE, "w4a16 load: " + base + " has no .qweight/.qzeros/.scales");
    o.gptq = o.g != nullptr;
    const bool f16s = o.s->dtype == MCV_DT_F16 || o.s->dtype == MCV_DT_BF16;
    if (o.q->dtype != MCV_DT_I32 || o.z->dtype != MCV_DT_I32 || !f16s || (o.gptq && o.g->dtype != MCV_DT_I32))
        return fail(MCV_ERR_VALUE, "w4a16 load: unexpected tensor dtypes for " + base);
    if (o.q->shape.size() != 2 || o.z->shape.size() != 2 || o.s->shape.size() != 2 || (o.gptq && o.g->shape.size() != 1))
        return fail(MCV_ERR_SHAPE, "w4a16 load: unexpected tensor ranks for " + base);
    const int64_t G = o.s->shape[0];
    if (o.gptq) {
        // quantized_weight.cpp:87-95: qweight [K/8, N], qzeros [G, N/8], scales [G, N], g_idx [K]
        o.K = o.q->shape[0] * 8;
        o.N = o.q->shape[1];
        if (o.g->shape[0] != o.K || G * 128 != o.K || o.s->shape[1] != o.N || o.z->shape[0] != G || o.z->shape[1] * 8 != o.N)
            return fail(MCV_ERR_SHAPE, "w4a16 load: unexpected GPTQ tensor shapes for " + base);
    } else {
        // quantized_weight.cpp:136-143: qweight [K, N/8], qzeros [G, N/8], scales [G, N]
        o.K = o.q->shape[0];
        o.N = o.q->shape[1] * 8;
        if (o.z->shape[0] != G || o.z->shape[1] != o.q->shape[1] || o.s->shape[1] != o.N || G * 128 != o.K)
            return fail(MCV_ERR_SHAPE, "w4a16 load: unexpected AWQ tensor shapes for " + base);
    }
    return MCV_OK;
}

}  // namespace
}  // namespace mcv

using namespace mcv;

extern "C" {

int mcv_safetensors_open(const char* path, void** st_out) {
    if (!path || !st_out) return fail(MCV_ERR_NULL, "safetensors_open: null argument");
    *st_out = nullptr;
    auto* f = new StFile();
    f->fd = ::open(path, O_RDONLY | O_CLOEXEC);
    if (f->fd < 0) {
        delete f;
        return fail(MCV_ERR_FORMAT, std::string("safetensors_open: cannot open ") + path + ": " + std::strerror(errno));
    }
    struct stat sb{};
    if (fstat(f->fd, &sb) != 0 || sb.st_size < 0) {
        ::close(f->fd);
        delete f;
        return fail(MCV_ERR_FORMAT, std::string("safetensors_open: cannot stat ") + path);
    }
    f->size = static_cast<size_t>(sb.st_size);
    if (f->size > 0) {
        void* m = mmap(nullptr, f->size, PROT_READ, MAP_PRIVATE, f->fd, 0);
        if (m == MAP_FAILED) {
            ::close(f->fd);
            delete f;
            return fail(MCV_ERR_FORMAT, std::string("safetensors_open: cannot map ") + path);
        }
        f->map = static_cast<const unsigned char*>(m);
    }
    const int st = parse_header(*f);
    if (st) {
        mcv_safetensors_close(f);
        return st;
    }
    *st_out = f;
    return MCV_OK;
}

int mcv_safetensors_close(void* st) {
    auto* f = static_cast<StFile*>(st);
    if (!f) return MCV_OK;
    if (f->map) munmap(const_cast<unsigned char*>(f->map), f->size);
    if (f->fd >= 0) ::close(f->fd);
    delete f;
    return MCV_OK;
}

int64_t mcv_safetensors_count(const void* st) {
    const auto* f = static_cast<const StFile*>(st);
    return f ? static_cast<int64_t>(f->names.size()) : 0;
}

const char* mcv_safetensors_name(const void* st, int64_t i) {
    const auto* f = static_cast<const StFile*>(st);
    if (!f || i < 0 || i >= static_cast<int64_t>(f->names.size())) return nullptr;
    return f->names[static_cast<size_t>(i)].c_str();
}

int mcv_safetensors_info(const void* st, const char* name, int* dtype, int* rank, int64_t* shape,
                         const void** data, uint64_t* nbytes) {
    const auto* f = static_cast<const StFile*>(st);
    if (!f || !name) return fail(MCV_ERR_NULL, "safetensors_info: null argument");
    const StTensor* t = find(f, name);
    if (!t) return fail(MCV_ERR_VALUE, std::string("safetensors_info: no tensor ") + name);
    if (t->shape.size() > 8) return fail(MCV_ERR_SHAPE, std::string("safetensors_info: rank above 8 for ") + name);
    if (dtype) *dtype = t->dtype;
    if (rank) *rank = static_cast<int>(t->shape.size());
    if (shape)
        for (size_t d = 0; d < t->shape.size(); ++d) shape[d] = t->shape[d];
    if (data) *data = f->map + t->begin;
    if (nbytes) *nbytes = t->end - t->begin;
    return MCV_OK;
}

int mcv_safetensors_copy_f16(const void* st, const char* name, void* dst_dev, uint64_t dst_bytes, mcv_stream_t stream) {
    const auto* f = static_cast<const StFile*>(st);
    if (!f || !name || !dst_dev) return fail(MCV_ERR_NULL, "safetensors_copy_f16: null argument");
    const StTensor* t = find(f, name);
    if (!t) return fail(MCV_ERR_VALUE, std::string("safetensors_copy_f16: no tensor ") + name);
    if (t->dtype != MCV_DT_F16 && t->dtype != MCV_DT_BF16)
        return fail(MCV_ERR_VALUE, std::string("safetensors_copy_f16: ") + name + " is neither F16 nor BF16");
    const uint64_t n = t->end - t->begin;
    if (dst_bytes < n) return fail(MCV_ERR_WORKSPACE, "safetensors_copy_f16: destination too small");
    auto s = static_cast<cudaStream_t>(stream);
    if (t->dtype == MCV_DT_F16) {
        MCV_CHECK_CUDA(cudaMemcpyAsync(dst_dev, f->map + t->begin, n, cudaMemcpyHostToDevice, s));
    } else {
        const std::vector<uint16_t> v = f16_elements(f, t);
        MCV_CHECK_CUDA(cudaMemcpyAsync(dst_dev, v.data(), n, cudaMemcpyHostToDevice, s));
        MCV_CHECK_CUDA(cudaStreamSynchronize(s));  // v is freed on return
    }
    return MCV_OK;
}

int mcv_w4a16_safetensors_dims(const void* st, const char* base, int64_t* K, int64_t* N, int* is_gptq) {
    const auto* f = static_cast<const StFile*>(st);
    if (!f || !base) return fail(MCV_ERR_NULL, "w4a16_safetensors_dims: null argument");
    QuantTensors q{};
    int rc = quant_tensors(f, base, q);
    if (rc) return rc;
    if (K) *K = q.K;
    if (N) *N = q.N;
    if (is_gptq) *is_gptq = q.gptq ? 1 : 0;
    return MCV_OK;
}

int mcv_w4a16_load_safetensors_host(const void* st, const char* base, uint32_t* qw, uint16_t* sc, uint32_t* zw,
                                    int* zero_bias_out) {
    const auto* f = static_cast<const StFile*>(st);
    if (!f || !base || !qw || !sc || !zw) return fail(MCV_ERR_NULL, "w4a16_load_safetensors: null argument");
    QuantTensors q{};
    int rc = quant_tensors(f, base, q);
    if (rc) return rc;
    const std::vector<int32_t> qweight = elements<int32_t>(f, q.q);
    const std::vector<int32_t> qzeros = elements<int32_t>(f, q.z);
    const std::vector<uint16_t> scales = f16_elements(f, q.s);
    if (q.gptq) {
        const std::vector<int32_t> g_idx = elements<int32_t>(f, q.g);
        return mcv_w4a16_pack_gptq_host(qweight.data(), qzeros.data(), g_idx.data(), scales.data(), q.K, q.N, 128, qw,
                                        sc, zw, zero_bias_out);
    }
    return mcv_w4a16_pack_awq_host(qweight.data(), qzeros.data(), scales.data(), q.K, q.N, 128, qw, sc, zw,
                                   zero_bias_out);
}

int mcv_w4a16_load_safetensors(const void* st, const char* base, void* qweight_dev, void* scales_dev, void* zeros_dev,
                               int* zero_bias_out, mcv_stream_t stream) {
    const auto* f = static_cast<const StFile*>(st);
    if (!f || !base || !qweight_dev || !scales_dev || !zeros_dev)
        return fail(MCV_ERR_NULL, "w4a16_load_safetensors: null argument");
    QuantTensors q{};
    int rc = quant_tensors(f, base, q);
    if (rc) return rc;
    size_t qb = 0, sb = 0, zb = 0;
    rc = mcv_w4a16_layout_bytes(q.K, q.N, 128, &qb, &sb, &zb);
    if (rc) return rc;
    std::vector<uint32_t> hq(qb / 4), hz(zb / 4);
    std::vector<uint16_t> hs(sb / 2);
    int bias = 0;
    rc = mcv_w4a16_load_safetensors_host(st, base, hq.data(), hs.data(), hz.data(), &bias);
    if (rc) return rc;
    auto s = static_cast<cudaStream_t>(stream);
    MCV_CHECK_CUDA(cudaMemcpyAsync(qweight_dev, hq.data(), qb, cudaMemcpyHostToDevice, s));
    MCV_CHECK_CUDA(cudaMemcpyAsync(scales_dev, hs.data(), sb, cudaMemcpyHostToDevice, s));
    MCV_CHECK_CUDA(cudaMemcpyAsync(zeros_dev, hz.data(), zb, cudaMemcpyHostToDevice, s));
    MCV_CHECK_CUDA(cudaStreamSynchronize(s));  // the host staging is freed on return
    if (zero_bias_out) *zero_bias_out = bias;
    return MCV_OK;
}

}  // extern "C"
