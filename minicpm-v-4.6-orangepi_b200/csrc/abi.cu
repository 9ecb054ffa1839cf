// Status strings, per-thread error messages and global launch settings of
// the C ABI (include/mcv_matmul.h).
#include <atomic>
#include <string>

#include "common.cuh"

namespace mcv {

unsigned take_w4a16_device_error();
unsigned take_dense_device_error();
unsigned take_gemm_device_error();
unsigned take_dense_gemm_device_error();

namespace {
thread_local std::string g_last_error;
std::atomic<int> g_pdl{1};
std::atomic<int> g_tuning[MCV_TUNE_COUNT];
}  // namespace

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int status, const std::string& msg) {
    g_last_error = msg;
    return status;
}

int cuda_fail(cudaError_t e, const char* what) {
    g_last_error = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
    return MCV_ERR_CUDA;
}

int tuning(int key) {
    return (key > 0 && key < MCV_TUNE_COUNT) ? g_tuning[key].load(std::memory_order_relaxed) : 0;
}

bool pdl_enabled() { return g_pdl.load(std::memory_order_relaxed) != 0; }

int sm_count() {
    // Cached per device (up to 64 devices per process).
    static std::atomic<int> cache[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    int v = cache[dev].load(std::memory_order_relaxed);
    if (v == 0) {
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
            v = 148;
        cache[dev].store(v, std::memory_order_relaxed);
    }
    return v;
}

}  // namespace mcv

extern "C" {

const char* mcv_status_string(int status) {
    switch (status) {
        case MCV_OK: return "ok";
        case MCV_ERR_NULL: return "null pointer";
        case MCV_ERR_SHAPE: return "unsupported shape";
        case MCV_ERR_ALIGN: return "misaligned pointer";
        case MCV_ERR_CUDA: return "CUDA error";
        case MCV_ERR_NCCL: return "NCCL error";
        case MCV_ERR_WORKSPACE: return "workspace missing or too small";
        case MCV_ERR_VALUE: return "bad argument value";
        case MCV_ERR_TIMEOUT: return "device wait timed out";
        case MCV_ERR_FORMAT: return "unreadable or malformed file";
        default: return "unknown status";
    }
}

const char* mcv_last_error(void) { return mcv::g_last_error.c_str(); }

int mcv_version(void) { return (1 << 16) | 0; }

void mcv_set_pdl(int enabled) { mcv::g_pdl.store(enabled ? 1 : 0); }

int mcv_set_tuning(int key, int value) {
    if (key <= 0 || key >= MCV_TUNE_COUNT) return mcv::fail(MCV_ERR_VALUE, "set_tuning: unknown key");
    mcv::g_tuning[key].store(value);
    return MCV_OK;
}

int mcv_get_tuning(int key) { return mcv::tuning(key); }

unsigned mcv_device_errors(void) {
    cudaDeviceSynchronize();
    return mcv::take_w4a16_device_error() | mcv::take_dense_device_error() | mcv::take_gemm_device_error() |
           mcv::take_dense_gemm_device_error();
}

}  // extern "C"
