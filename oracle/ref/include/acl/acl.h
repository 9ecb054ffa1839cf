/* Host-only stand-in for the parts of the CANN runtime API that the
 * reference engine's host sources (tensor.cpp, acl_context.cpp, weights.cpp,
 * quantized_weight.cpp) and its CPU-checked tests use.  TEST INFRASTRUCTURE:
 * it lets those reference sources compile and run on this machine's CPU, with
 * "device" memory being ordinary host memory.  Only names and signatures are
 * given here; the definitions are in acl_stub.cpp. */
#ifndef MCV_REF_ACL_STUB_H
#define MCV_REF_ACL_STUB_H

#include <stddef.h>
#include <stdint.h>

typedef int aclError;
typedef void* aclrtStream;
#define ACL_SUCCESS 0
#define ACL_ERROR_INVALID_PARAM 100000

typedef enum {
    ACL_DT_UNDEFINED = -1,
    ACL_FLOAT = 0,
    ACL_FLOAT16 = 1,
    ACL_INT8 = 2,
    ACL_INT32 = 3,
    ACL_UINT8 = 4,
    ACL_INT16 = 6,
    ACL_UINT16 = 7,
    ACL_UINT32 = 8,
    ACL_INT64 = 9,
    ACL_UINT64 = 10,
    ACL_DOUBLE = 11,
    ACL_BOOL = 12,
    ACL_BF16 = 27
} aclDataType;

typedef enum { ACL_MEM_MALLOC_HUGE_FIRST = 0, ACL_MEM_MALLOC_HUGE_ONLY = 1, ACL_MEM_MALLOC_NORMAL_ONLY = 2 } aclrtMemMallocPolicy;
typedef enum {
    ACL_MEMCPY_HOST_TO_HOST = 0,
    ACL_MEMCPY_HOST_TO_DEVICE = 1,
    ACL_MEMCPY_DEVICE_TO_HOST = 2,
    ACL_MEMCPY_DEVICE_TO_DEVICE = 3
} aclrtMemcpyKind;

#ifdef __cplusplus
extern "C" {
#endif
aclError aclInit(const char* config);
aclError aclFinalize(void);
aclError aclrtSetDevice(int32_t device);
aclError aclrtResetDevice(int32_t device);
aclError aclrtCreateStream(aclrtStream* stream);
aclError aclrtDestroyStream(aclrtStream stream);
aclError aclrtSynchronizeStream(aclrtStream stream);
aclError aclrtMalloc(void** ptr, size_t size, aclrtMemMallocPolicy policy);
aclError aclrtFree(void* ptr);
aclError aclrtMemcpy(void* dst, size_t dst_max, const void* src, size_t count, aclrtMemcpyKind kind);
aclError aclrtMemset(void* ptr, size_t max, int32_t value, size_t count);
const char* aclGetRecentErrMsg(void);
#ifdef __cplusplus
}
#endif

#endif
