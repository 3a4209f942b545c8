/*
 * CPU oracle for the integer stages of the int8 / int8-dyn quantised-linear path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product path links or calls this
 * file; only tests/, __graft_entry__.smoke() and bench.py's CPU baseline leg use
 * it, as the checker.
 *
 * It restates, in plain C, the arithmetic the reference runs on the CPU:
 *
 *   quantize_per_channel       spikingbrain_cpu/quant.py:25-29
 *   DynamicInt8Linear.forward  spikingbrain_cpu/quant.py:63-66, i.e. torch's
 *                              quantized::linear_dynamic on the fbgemm / x86
 *                              engine (fbgemm is a torch-wheel dependency, not
 *                              vendored in the reference).  The steps restated:
 *     1. min/max over the whole [M, K] fp32 activation, widened to include 0;
 *     2. torch's ChooseQuantizationParams (qmin 0, qmax 255, no range
 *        reduction): scale in double, the zero point chosen from whichever
 *        end (min or max) has the smaller rounding error, nudged by
 *        round-half-even and clamped to [0, 255]; the scale is stored as fp32;
 *     3. fbgemm's quantiser: xq = clamp(rint(fma(x, 1/s, zp)), 0, 255) with
 *        1/s an fp32 reciprocal, one rounding for the fused multiply-add, and
 *        ties to even;
 *     4. acc[m,n] = sum_k (xq[m,k] - zp) * q[n,k] in int32;
 *     5. y[m,n] = float(acc) * (s * scale[n]) in fp32; with a bias the last
 *        multiply and the bias add are one fused multiply-add.
 *   Steps 3 and 5 were pinned against linear_dynamic bit for bit (see
 *   tests/golden/make_golden.py); plain rint(x / s) + zp is NOT equivalent.
 *
 *   The per-token symmetric mode (an addition with no reference counterpart)
 *   is restated the same way: s_t = max(max|x_t|, 1e-8) / 127 in fp32,
 *   xq = clamp(rint(x / s_t), -127, 127), y = float(acc) * (s_t * scale[n]).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define EXPORT __attribute__((visibility("default")))

/* quant.py:25-29: scale = max(amax_k |w|, 1e-8) / 127 (fp32); q = clamp(rint(w / scale)). */
EXPORT void orc_quantize_per_channel(const float* w, int64_t n, int64_t k, int8_t* q, float* scale) {
    for (int64_t r = 0; r < n; ++r) {
        const float* row = w + r * k;
        float amax = 0.0f;
        for (int64_t c = 0; c < k; ++c) {
            float a = fabsf(row[c]);
            if (a > amax) amax = a;
        }
        if (amax < 1e-8f) amax = 1e-8f;
        volatile float s = amax / 127.0f;
        scale[r] = s;
        for (int64_t c = 0; c < k; ++c) {
            volatile float t = row[c] / s;
            float v = rintf(t);
            if (v > 127.0f) v = 127.0f;
            if (v < -127.0f) v = -127.0f;
            q[r * k + c] = (int8_t)v;
        }
    }
}

/* torch ChooseQuantizationParams for quint8, reduce_range = false, preserve_sparsity = false. */
EXPORT void orc_choose_qparams(float mn, float mx, float* scale_out, int32_t* zp_out) {
    const int qmin = 0, qmax = 255;
    const float small_scale = 6.1e-5f;
    if (mn > 0.0f) mn = 0.0f;
    if (mx < 0.0f) mx = 0.0f;
    double scale = ((double)mx - (double)mn) / (double)(qmax - qmin);
    if ((float)scale == 0.0f || isinf(1.0f / (float)scale)) scale = 0.1;
    if (scale < (double)small_scale) {
        float org_scale = (float)scale;
        scale = small_scale;
        if (mn == 0.0f) {
            mx = small_scale * (float)(qmax - qmin);
        } else if (mx == 0.0f) {
            mn = -small_scale * (float)(qmax - qmin);
        } else {
            float amplifier = small_scale / org_scale;
            mn *= amplifier;
            mx *= amplifier;
        }
    }
    double zp_from_min = qmin - mn / scale;
    double zp_from_max = qmax - mx / scale;
    double err_min = fabs((double)qmin) - fabs(mn / scale);
    double err_max = fabs((double)qmax) - fabs(mx / scale);
    double zp0 = err_min < err_max ? zp_from_min : zp_from_max;
    int32_t zp;
    if (zp0 < qmin) zp = qmin;
    else if (zp0 > qmax) zp = qmax;
    else zp = (int32_t)nearbyint(zp0);
    *scale_out = (float)scale;
    *zp_out = zp;
}

/* Steps 1-2: per-tensor parameters of a [count] fp32 activation. */
EXPORT void orc_act_qparams_per_tensor(const float* x, int64_t count, float* scale_out, int32_t* zp_out) {
    float mn = 0.0f, mx = 0.0f;
    if (count > 0) { mn = x[0]; mx = x[0]; }
    for (int64_t i = 1; i < count; ++i) {
        if (x[i] < mn) mn = x[i];
        if (x[i] > mx) mx = x[i];
    }
    orc_choose_qparams(mn, mx, scale_out, zp_out);
}

/* Step 3: fbgemm quantiser, fused multiply-add with the fp32 reciprocal of the scale. */
EXPORT void orc_quantize_per_tensor(const float* x, int64_t count, float scale, int32_t zp, uint8_t* xq) {
    volatile float inv = 1.0f / scale;
    const float fzp = (float)zp;
    for (int64_t i = 0; i < count; ++i) {
        float t = rintf(fmaf(x[i], inv, fzp));
        if (t < 0.0f) t = 0.0f;
        if (t > 255.0f) t = 255.0f;
        xq[i] = (uint8_t)t;
    }
}

/* Per-token symmetric mode: one fp32 scale per row, int8 in [-127, 127]. */
EXPORT void orc_quantize_per_token(const float* x, int64_t m, int64_t k, int8_t* xq, float* s_tok) {
    for (int64_t r = 0; r < m; ++r) {
        const float* row = x + r * k;
        float amax = 0.0f;
        for (int64_t c = 0; c < k; ++c) {
            float a = fabsf(row[c]);
            if (a > amax) amax = a;
        }
        if (amax < 1e-8f) amax = 1e-8f;
        volatile float s = amax / 127.0f;
        s_tok[r] = s;
        for (int64_t c = 0; c < k; ++c) {
            volatile float t = row[c] / s;
            float v = rintf(t);
            if (v > 127.0f) v = 127.0f;
            if (v < -127.0f) v = -127.0f;
            xq[r * k + c] = (int8_t)v;
        }
    }
}

/* Step 4 for any integer activation: a[m,k] (already offset by its zero point, as int16) times q[n,k]. */
static void gemm_i16_i8(const int16_t* a, const int8_t* q, int64_t m, int64_t n, int64_t k, int32_t* acc) {
    int16_t* qrow = (int16_t*)malloc((size_t)k * sizeof(int16_t));
    for (int64_t j = 0; j < n; ++j) {
        for (int64_t c = 0; c < k; ++c) qrow[c] = q[j * k + c];
        for (int64_t i = 0; i < m; ++i) {
            const int16_t* ar = a + i * k;
            int32_t s = 0;
            for (int64_t c = 0; c < k; ++c) s += (int32_t)ar[c] * (int32_t)qrow[c];
            acc[i * n + j] = s;
        }
    }
    free(qrow);
}

/* acc[m,n] = sum_k (xq[m,k] - zp) * q[n,k] for the per-tensor (uint8 + zero point) mode. */
EXPORT void orc_gemm_u8s8(const uint8_t* xq, int32_t zp, const int8_t* q, int64_t m, int64_t n, int64_t k, int32_t* acc) {
    int16_t* a = (int16_t*)malloc((size_t)(m * k) * sizeof(int16_t));
    for (int64_t i = 0; i < m * k; ++i) a[i] = (int16_t)((int32_t)xq[i] - zp);
    gemm_i16_i8(a, q, m, n, k, acc);
    free(a);
}

/* acc[m,n] = sum_k xq[m,k] * q[n,k] for the per-token (int8, symmetric) mode. */
EXPORT void orc_gemm_s8s8(const int8_t* xq, const int8_t* q, int64_t m, int64_t n, int64_t k, int32_t* acc) {
    int16_t* a = (int16_t*)malloc((size_t)(m * k) * sizeof(int16_t));
    for (int64_t i = 0; i < m * k; ++i) a[i] = xq[i];
    gemm_i16_i8(a, q, m, n, k, acc);
    free(a);
}

/* Step 5: y = float(acc) * (s_x[row] * scale[n]), or fma(float(acc), s_x[row] * scale[n], bias[n]).  s_rows holds one
 * scale per row (per-token mode) or a single scale when s_stride == 0. */
EXPORT void orc_dyn_epilogue(const int32_t* acc, int64_t m, int64_t n, const float* s_rows, int64_t s_stride,
                             const float* scale, const float* bias, float* y) {
    for (int64_t i = 0; i < m; ++i) {
        const float sx = s_rows[i * s_stride];
        for (int64_t j = 0; j < n; ++j) {
            volatile float f = sx * scale[j];
            float a = (float)acc[i * n + j];
            y[i * n + j] = bias ? fmaf(a, f, bias[j]) : a * f;
        }
    }
}
