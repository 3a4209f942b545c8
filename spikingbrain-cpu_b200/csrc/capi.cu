// Library-level C ABI: version, status strings and the thread-local error message.
#include <stdarg.h>
#include <stdio.h>

#include "common.cuh"

namespace sbq {

static thread_local char g_last_error[512] = "";

int set_error(int status, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return status;
}

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(SBQ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return SBQ_OK;
}

}  // namespace sbq

extern "C" int sbq_version(void) { return 1 * 10000 + 0 * 100 + 0; }

extern "C" const char* sbq_last_error(void) { return sbq::g_last_error; }

extern "C" const char* sbq_status_string(int status) {
    switch (status) {
        case SBQ_OK: return "SBQ_OK";
        case SBQ_ERR_INVALID_ARGUMENT: return "SBQ_ERR_INVALID_ARGUMENT";
        case SBQ_ERR_ALIGNMENT: return "SBQ_ERR_ALIGNMENT";
        case SBQ_ERR_UNSUPPORTED: return "SBQ_ERR_UNSUPPORTED";
        case SBQ_ERR_CUDA: return "SBQ_ERR_CUDA";
        case SBQ_ERR_TIMEOUT: return "SBQ_ERR_TIMEOUT";
        case SBQ_ERR_DEVICE: return "SBQ_ERR_DEVICE";
        case SBQ_ERR_WORKSPACE: return "SBQ_ERR_WORKSPACE";
        default: return "SBQ_ERR_UNKNOWN";
    }
}
