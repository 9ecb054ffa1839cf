// Definitions of the host-only CANN stand-in (include/acl/acl.h): memory is
// host memory, streams are null handles, copies are memcpy.  TEST
// INFRASTRUCTURE for running the reference's host code on the CPU.
#include <cstdlib>
#include <cstring>

#include "acl/acl.h"

extern "C" {
aclError aclInit(const char*) { return ACL_SUCCESS; }
aclError aclFinalize(void) { return ACL_SUCCESS; }
aclError aclrtSetDevice(int32_t) { return ACL_SUCCESS; }
aclError aclrtResetDevice(int32_t) { return ACL_SUCCESS; }
aclError aclrtCreateStream(aclrtStream* s) {
    if (s) *s = nullptr;
    return ACL_SUCCESS;
}
aclError aclrtDestroyStream(aclrtStream) { return ACL_SUCCESS; }
aclError aclrtSynchronizeStream(aclrtStream) { return ACL_SUCCESS; }
aclError aclrtMalloc(void** p, size_t n, aclrtMemMallocPolicy) {
    if (!p) return ACL_ERROR_INVALID_PARAM;
    *p = std::calloc(n ? n : 1, 1);
    return *p ? ACL_SUCCESS : ACL_ERROR_INVALID_PARAM;
}
aclError aclrtFree(void* p) {
    std::free(p);
    return ACL_SUCCESS;
}
aclError aclrtMemcpy(void* dst, size_t dst_max, const void* src, size_t count, aclrtMemcpyKind) {
    if (count > dst_max || (!dst && count) || (!src && count)) return ACL_ERROR_INVALID_PARAM;
    if (count) std::memmove(dst, src, count);
    return ACL_SUCCESS;
}
aclError aclrtMemset(void* p, size_t max, int32_t v, size_t count) {
    if (count > max) return ACL_ERROR_INVALID_PARAM;
    std::memset(p, v, count);
    return ACL_SUCCESS;
}
const char* aclGetRecentErrMsg(void) { return ""; }
}
