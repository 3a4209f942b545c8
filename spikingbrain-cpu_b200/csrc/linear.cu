// Format-level entry point of the int8 weight-only format: Int8Linear.forward (GEMV / GEMM dispatch).
#include "common.cuh"

namespace sbq {
int check_linear_args(const void* x, int x_dtype, int64_t ldx, const void* packed, const float* scale, int64_t m,
                      int64_t n, int64_t k, const void* y, int y_dtype, int64_t ldy);
}

using namespace sbq;

// Rows of x above which the tensor-memory GEMM (64-token tiles up to 128 rows, 256-token tiles
// beyond) replaces the weight-streaming GEMV, which re-reads the weight once per 16 rows.
constexpr int64_t kGemmMinRows = 32;

extern "C" int sbq_linear_w8(const void* x, int x_dtype, int64_t ldx, const void* packed, const float* scale,
                             const float* bias, int64_t m, int64_t n, int64_t k, void* y, int y_dtype, int64_t ldy,
                             void* stream) {
    if (m > kGemmMinRows && x_dtype == SBQ_F16)
        return sbq_gemm_w8a16(x, x_dtype, ldx, packed, scale, bias, m, n, k, y, y_dtype, ldy, stream);
    return sbq_gemv_w8(x, x_dtype, ldx, packed, scale, bias, m, n, k, y, y_dtype, ldy, stream);
}

