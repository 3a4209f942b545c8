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

// ---- device error word and TMA tensor-map encoding -----------------------------------------------
#include <cuda.h>
#include <mutex>

#include "tc.cuh"

namespace sbq {

int poll_error_dyn();
int poll_error_w8a16();
int poll_error_gemv();

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

int encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
                const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return set_error(SBQ_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    cuuint64_t gd[5], gs[4];
    cuuint32_t bx[5], es[5];
    for (int i = 0; i < rank; ++i) {
        gd[i] = dims[i];
        bx[i] = box[i];
        es[i] = 1;
        if (i + 1 < rank) gs[i] = strides_bytes[i];
    }
    CUresult r = fn(map, dtype, (cuuint32_t)rank, const_cast<void*>(base), gd, gs, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(SBQ_ERR_INVALID_ARGUMENT, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return SBQ_OK;
}

}  // namespace sbq

extern "C" int sbq_check_device_error(void) {
    if (cudaDeviceSynchronize() != cudaSuccess) return sbq::check_launch("device synchronise");
    int h = sbq::poll_error_dyn();
    if (h == 0) h = sbq::poll_error_w8a16();
    if (h == 0) h = sbq::poll_error_gemv();
    if (h != 0)
        return sbq::set_error(h, "a kernel reported %s (bounded device-side wait expired)", sbq_status_string(h));
    return SBQ_OK;
}
