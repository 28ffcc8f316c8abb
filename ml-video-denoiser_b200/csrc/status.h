// Status codes and the thread-local "last error" message of the C-ABI.
// Every extern "C" entry point returns DN_OK (0) or a negative DN_ERR_* code
// and never lets a C++ exception cross the boundary.
#pragma once

#include <cuda_runtime.h>

#include <string>

#include "denoiser_b200.h"

namespace dnb {

// Records `msg` as the calling thread's last error and returns `code`.
int dn_fail(int code, const char* msg);
int dn_fail_str(int code, const std::string& msg);
// Records a CUDA error with context and returns DN_ERR_CUDA.
int dn_cuda_fail(cudaError_t e, const char* where);

// Returns the status of `x` from the enclosing function unless it is DN_OK.
#define DN_TRY(x)                     \
    do {                              \
        const int _rc = (x);          \
        if (_rc != DN_OK) return _rc; \
    } while (0)

}  // namespace dnb
