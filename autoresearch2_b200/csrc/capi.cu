// Library-level C ABI: version, error strings, last CUDA error.
#include <stdio.h>

#include "common.cuh"

namespace sffn {
namespace {
thread_local char g_last_cuda_error[256] = "";
}
void set_cuda_error(cudaError_t e) {
    snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "%s: %s", cudaGetErrorName(e),
             cudaGetErrorString(e));
}
void set_error_text(const char* msg) { snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "%s", msg); }
}  // namespace sffn

extern "C" int sffn_version(void) { return 100; }

extern "C" const char* sffn_error_string(int code) {
    switch (code) {
        case SFFN_OK: return "ok";
        case SFFN_ERR_ARG: return "invalid argument";
        case SFFN_ERR_DTYPE: return "unsupported dtype";
        case SFFN_ERR_ALIGN: return "misaligned pointer or stride";
        case SFFN_ERR_WORKSPACE: return "workspace too small";
        case SFFN_ERR_CUDA: return "CUDA error";
        case SFFN_ERR_UNSUPPORTED: return "unsupported shape or layout";
        case SFFN_ERR_DEVICE: return "device is not sm_100";
        case SFFN_ERR_TOO_LARGE: return "size exceeds the entry point's fixed capacity";
        default: return "unknown error";
    }
}

extern "C" const char* sffn_last_cuda_error(void) { return sffn::g_last_cuda_error; }
