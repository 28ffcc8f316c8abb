// Thread-local last-error storage behind dn_last_error().
#include "status.h"

#include <string>

namespace dnb {
namespace {
thread_local std::string g_last_error;
}

const char* g_last_error_ptr() { return g_last_error.c_str(); }

int dn_fail(int code, const char* msg) {
    g_last_error = msg ? msg : "";
    return code;
}

int dn_fail_str(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

int dn_cuda_fail(cudaError_t e, const char* where) {
    g_last_error = std::string(where) + ": " + cudaGetErrorString(e);
    return DN_ERR_CUDA;
}

}  // namespace dnb

extern "C" const char* dn_last_error(void) { return dnb::g_last_error_ptr(); }

extern "C" int dn_abi_version(void) { return 100; }
