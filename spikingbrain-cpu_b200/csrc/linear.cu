// Format-level entry point of the int8 weight-only format: Int8Linear.forward (GEMV / GEMM dispatch).
#include "common.cuh"

namespace sbq {
int check_linear_args(const void* x, int x_dtype, int64_t ldx, const void* packed, const float* scale, int64_t m,
                      int64_t n, int64_t k, const void* y, int y_dtype, int64_t ldy);
}

using namespace sbq;

extern "C" int sbq_linear_w8(const void* x, int x_dtype, int64_t ldx, const void* packed, const float* scale,
                             const float* bias, int64_t m, int64_t n, int64_t k, void* y, int y_dtype, int64_t ldy,
                             void* stream) {
    return sbq_gemv_w8(x, x_dtype, ldx, packed, scale, bias, m, n, k, y, y_dtype, ldy, stream);
}

extern "C" int sbq_gemm_w8a16(const void*, int, int64_t, const void*, const float*, const float*, int64_t, int64_t,
                              int64_t, void*, int, int64_t, void*) {
    return set_error(SBQ_ERR_UNSUPPORTED, "sbq_gemm_w8a16 not built yet");
}
