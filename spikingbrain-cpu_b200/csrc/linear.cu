// Format-level entry points of the int8 weight-only format: Int8Linear.forward (GEMV / GEMM dispatch).
#include "common.cuh"

namespace sbq {
int check_linear_args(const void* x, int x_dtype, int64_t ldx, const void* packed, const float* scale, int64_t m,
                      int64_t n, int64_t k, const void* y, int y_dtype, int64_t ldy);
int gemm_w8a16_run_x2(const void* hi, const void* lo, int64_t ldx, const void* packed, const float* scale,
                      const float* bias, int64_t m, int64_t n, int64_t k, void* y, int y_dtype, int64_t ldy, void* stream,
                      int gated);
size_t split_workspace_bytes(int64_t m, int64_t k);
int split_into_workspace(const void* x, int64_t ldx, int64_t m, int64_t k, void* workspace, size_t workspace_bytes,
                         void** hi, void** lo, void* stream);
}  // namespace sbq

using namespace sbq;

extern "C" size_t sbq_linear_w8_workspace_bytes(int64_t m, int64_t k, int x_dtype) {
    if (m <= kGemmMinRows || k <= 0 || x_dtype != SBQ_F32) return 0;
    return split_workspace_bytes(m, k);
}

extern "C" int sbq_linear_w8(const void* x, int x_dtype, int64_t ldx, const void* packed, const float* scale,
                             const float* bias, int64_t m, int64_t n, int64_t k, void* y, int y_dtype, int64_t ldy,
                             void* stream) {
    if (m > kGemmMinRows && (x_dtype == SBQ_F16 || x_dtype == SBQ_BF16))
        return sbq_gemm_w8a16(x, x_dtype, ldx, packed, scale, bias, m, n, k, y, y_dtype, ldy, stream);
    return sbq_gemv_w8(x, x_dtype, ldx, packed, scale, bias, m, n, k, y, y_dtype, ldy, stream);
}

extern "C" int sbq_linear_w8_ws(const void* x, int x_dtype, int64_t ldx, const void* packed, const float* scale,
                                const float* bias, int64_t m, int64_t n, int64_t k, void* y, int y_dtype, int64_t ldy,
                                void* workspace, size_t workspace_bytes, void* stream) {
    if (m > kGemmMinRows && x_dtype == SBQ_F32) {
        int st = check_linear_args(x, x_dtype, ldx, packed, scale, m, n, k, y, y_dtype, ldy);
        if (st) return st;
        void *hi = nullptr, *lo = nullptr;
        st = split_into_workspace(x, ldx, m, k, workspace, workspace_bytes, &hi, &lo, stream);
        if (st) return st;
        return gemm_w8a16_run_x2(hi, lo, k, packed, scale, bias, m, n, k, y, y_dtype, ldy, stream, 0);
    }
    return sbq_linear_w8(x, x_dtype, ldx, packed, scale, bias, m, n, k, y, y_dtype, ldy, stream);
}
