// Library-level C ABI: version, error strings, last CUDA error; the device
// scope every entry point binds its device with.
#include <cuda.h>
#include <stdio.h>

#include "common.cuh"

namespace sffn {
namespace {
thread_local char g_last_cuda_error[256] = "";

// Driver entry points for the caller's current context, found through the
// runtime (the library links no driver library, so it also loads on hosts
// without one).
using CtxGetFn = CUresult (*)(CUcontext*);
using CtxSetFn = CUresult (*)(CUcontext);
using CtxIdFn = CUresult (*)(CUcontext, unsigned long long*);
struct CtxFns {
    CtxGetFn get = nullptr;
    CtxSetFn set = nullptr;
    CtxIdFn id = nullptr;
};
const CtxFns& ctx_fns() {
    static const CtxFns fns = [] {
        CtxFns f;
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            f.get = reinterpret_cast<CtxGetFn>(p);
        p = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxSetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            f.set = reinterpret_cast<CtxSetFn>(p);
        p = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            f.id = reinterpret_cast<CtxIdFn>(p);
        cudaGetLastError();
        return f;
    }();
    return fns;
}
}  // namespace

void set_cuda_error(cudaError_t e) {
    snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "%s: %s", cudaGetErrorName(e),
             cudaGetErrorString(e));
}
void set_error_text(const char* msg) { snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "%s", msg); }

int device_of(const void* p) {
    cudaPointerAttributes a;
    if (p && cudaPointerGetAttributes(&a, p) == cudaSuccess &&
        (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged))
        return a.device;
    cudaGetLastError();  // clear a failed pointer query
    return -1;
}

unsigned long long current_context_id() {
    const CtxFns& f = ctx_fns();
    CUcontext c = nullptr;
    unsigned long long id = 0;
    if (!f.get || !f.id || f.get(&c) != CUDA_SUCCESS || !c || f.id(c, &id) != CUDA_SUCCESS) return 0;
    return id;
}

int DeviceScope::bind(const void* p) {
    const int d = device_of(p);
    if (d < 0) return SFFN_ERR_ARG;
    const CtxFns& f = ctx_fns();
    CUcontext before = nullptr;
    const bool have_before = f.get && f.set && f.get(&before) == CUDA_SUCCESS;
    // cudaSetDevice initialises the device's primary context and makes it
    // current on this thread, also when the device is current already.
    if (cudaSetDevice(d) != cudaSuccess) {
        cudaGetLastError();
        set_error_text("cudaSetDevice failed for the device of an argument");
        return SFFN_ERR_CUDA;
    }
    CUcontext now = nullptr;
    if (have_before && f.get(&now) == CUDA_SUCCESS && now != before) {
        saved_ = before;
        restore_ = true;
    }
    dev_ = d;
    return SFFN_OK;
}

int DeviceScope::bind_same(const void* p, std::initializer_list<const void*> others) {
    if (int rc = bind(p)) return rc;
    for (const void* q : others)
        if (q && device_of(q) != dev_) {
            set_error_text("arguments live on different devices");
            return SFFN_ERR_ARG;
        }
    return SFFN_OK;
}

DeviceScope::~DeviceScope() {
    if (restore_) ctx_fns().set(static_cast<CUcontext>(saved_));
}
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
