// Decode GEMV for the int8 weight-only format (and the fused gate/up SwiGLU half of the MLP).
//
// Reference: Int8Linear.forward (spikingbrain_cpu/quant.py:41-53) at decode shapes (one token per
// call, engine.py:104-106) and GatedMLP.forward (model.py:239-240).  The reference dequantises
// each 128-row block of the weight to fp32 and runs an fp32 sgemm, then multiplies by the
// per-row scale.  Here the weight is streamed from HBM exactly once per launch:
//
//   * one CTA per 16-row tile of the weight, 8 warps splitting K; each warp streams its 1 KiB
//     tiles with two contiguous 512-byte, 128-bit loads per tile (no L1 allocation);
//   * int8 -> fp16 (or bf16) conversion in registers (exact), m16n8k16 tensor-core MMAs with
//     fp32 accumulation; the activation rows form the n dimension (8 or 16 tokens per pass), so
//     the k-permutation of the packed layout is applied to x on load;
//   * partial sums of the 8 warps are reduced in shared memory, then the fp32 per-row scale (and
//     bias, or the SiLU(gate) * up product) is applied before the single store.
//
// fp32 activations are split into a bf16 high and low part (two MMAs, ~16 mantissa bits kept);
// the dot product of int8 weights and fp16/bf16 activations is exact up to fp32 accumulation.
#include "common.cuh"

namespace sbq {

enum XKind { kXF16 = 0, kXBF16 = 1, kXF32 = 2 };

struct GemvParams {
    const void* x;
    int64_t ldx;
    const int8_t* w0;  // packed weight (gate for the MLP variant)
    const float* s0;
    const int8_t* w1;  // packed up weight (MLP variant only)
    const float* s1;
    const float* bias;
    void* y;
    int64_t ldy;
    int m;  // rows of x handled by this launch (<= 8 * MT)
    int n;
    int k;
    int kt_total;
    int kt_per_warp;
};

constexpr int kGemvWarps = 8;
constexpr int kGemvUnroll = 4;

// Loads the 16 activation values lane (g, c) needs for span kt, row `row`, as MMA B fragments:
// b[s][0..1] for the four k16 steps s.  Rows beyond m (or spans beyond k) read as zero.
template <int XK>
struct XFrag {
    uint32_t b[4][2];      // fp16 / bf16 main part
    uint32_t blo[4][2];    // bf16 low part (fp32 input only)
};

template <int XK>
__device__ __forceinline__ void load_x(XFrag<XK>& f, const void* x, int64_t ldx, int row, int m, int64_t k0, int k) {
    const bool ok = row < m && k0 < k;
    if (XK == kXF16 || XK == kXBF16) {
        uint4 v0 = make_uint4(0, 0, 0, 0), v1 = v0;
        if (ok) {
            const uint16_t* p = static_cast<const uint16_t*>(x) + (int64_t)row * ldx + k0;
            v0 = ld_act(p);
            v1 = ld_act(p + 8);
        }
        f.b[0][0] = v0.x; f.b[0][1] = v0.y; f.b[1][0] = v0.z; f.b[1][1] = v0.w;
        f.b[2][0] = v1.x; f.b[2][1] = v1.y; f.b[3][0] = v1.z; f.b[3][1] = v1.w;
    } else {
        float v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = 0.0f;
        if (ok) {
            const float* p = static_cast<const float*>(x) + (int64_t)row * ldx + k0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                uint4 t = ld_act(p + 4 * i);
                v[4 * i + 0] = __uint_as_float(t.x);
                v[4 * i + 1] = __uint_as_float(t.y);
                v[4 * i + 2] = __uint_as_float(t.z);
                v[4 * i + 3] = __uint_as_float(t.w);
            }
        }
#pragma unroll
        for (int s = 0; s < 4; ++s) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const float a = v[4 * s + 2 * h], b = v[4 * s + 2 * h + 1];
                __nv_bfloat162 hi = __floats2bfloat162_rn(a, b);
                float2 hf = __bfloat1622float2(hi);
                __nv_bfloat162 lo = __floats2bfloat162_rn(a - hf.x, b - hf.y);
                f.b[s][h] = *reinterpret_cast<uint32_t*>(&hi);
                f.blo[s][h] = *reinterpret_cast<uint32_t*>(&lo);
            }
        }
    }
}

// acc += W_tile(span) . X(span) for one 1 KiB tile (the lane's two 16-byte pieces wa, wb).
template <int XK, int MT>
__device__ __forceinline__ void tile_mma(float (&acc)[MT][4], const uint4& wa, const uint4& wb,
                                         const XFrag<XK> (&xf)[MT]) {
    const uint32_t wa_[4] = {wa.x, wa.y, wa.z, wa.w};
    const uint32_t wb_[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
    for (int s = 0; s < 4; ++s) {
        uint32_t a0, a1, a2, a3;
        if (XK == kXF16) {
            i8x4_to_half2x2(wa_[s], a0, a2);
            i8x4_to_half2x2(wb_[s], a1, a3);
        } else {
            i8x4_to_bf162x2(wa_[s], a0, a2);
            i8x4_to_bf162x2(wb_[s], a1, a3);
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            if (XK == kXF16) {
                mma_f16(acc[mt], a0, a1, a2, a3, xf[mt].b[s][0], xf[mt].b[s][1]);
            } else {
                mma_bf16(acc[mt], a0, a1, a2, a3, xf[mt].b[s][0], xf[mt].b[s][1]);
                if (XK == kXF32) mma_bf16(acc[mt], a0, a1, a2, a3, xf[mt].blo[s][0], xf[mt].blo[s][1]);
            }
        }
    }
}

template <typename T>
__device__ __forceinline__ void store_out(void* y, int64_t idx, float v);
template <>
__device__ __forceinline__ void store_out<float>(void* y, int64_t idx, float v) { static_cast<float*>(y)[idx] = v; }
template <>
__device__ __forceinline__ void store_out<__half>(void* y, int64_t idx, float v) {
    static_cast<__half*>(y)[idx] = __float2half_rn(v);
}

// NMAT = 1: y = x . W^T * scale (+ bias).   NMAT = 2: y = silu(x . Wg^T * sg) * (x . Wu^T * su).
template <int XK, int MT, int NMAT, typename OutT>
__global__ void __launch_bounds__(kGemvWarps * 32) gemv_w8_kernel(const GemvParams p) {
    __shared__ float red[kGemvWarps][NMAT][MT][16][9];  // +1 column against bank conflicts

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, c = lane & 3;
    const int nt = blockIdx.x;
    const int kt_begin = warp * p.kt_per_warp;
    const int kt_end = min(kt_begin + p.kt_per_warp, p.kt_total);

    float acc[NMAT][MT][4];
#pragma unroll
    for (int i = 0; i < NMAT; ++i)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][mt][j] = 0.0f;

    const int64_t tile0 = (int64_t)nt * p.kt_total;
    const int8_t* wp0 = p.w0 + tile0 * kTileBytes + lane * 16;
    const int8_t* wp1 = NMAT == 2 ? p.w1 + tile0 * kTileBytes + lane * 16 : nullptr;

    for (int kt = kt_begin; kt < kt_end; kt += kGemvUnroll) {
        uint4 wa[NMAT][kGemvUnroll], wb[NMAT][kGemvUnroll];
#pragma unroll
        for (int u = 0; u < kGemvUnroll; ++u) {
            const bool live = kt + u < kt_end;
#pragma unroll
            for (int i = 0; i < NMAT; ++i) {
                const int8_t* wp = (i == 0 ? wp0 : wp1) + (int64_t)(kt + u) * kTileBytes;
                wa[i][u] = live ? ld_stream(wp) : make_uint4(0, 0, 0, 0);
                wb[i][u] = live ? ld_stream(wp + 512) : make_uint4(0, 0, 0, 0);
            }
        }
#pragma unroll
        for (int u = 0; u < kGemvUnroll; ++u) {
            if (kt + u >= kt_end) break;
            XFrag<XK> xf[MT];
            const int64_t k0 = (int64_t)(kt + u) * kTileCols + 16 * c;
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) load_x<XK>(xf[mt], p.x, p.ldx, 8 * mt + g, p.m, k0, p.k);
#pragma unroll
            for (int i = 0; i < NMAT; ++i) tile_mma<XK, MT>(acc[i], wa[i][u], wb[i][u], xf);
        }
    }

    // Fragment (row g / g+8, token 2c / 2c+1) -> shared memory.
#pragma unroll
    for (int i = 0; i < NMAT; ++i)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            red[warp][i][mt][g][2 * c] = acc[i][mt][0];
            red[warp][i][mt][g][2 * c + 1] = acc[i][mt][1];
            red[warp][i][mt][g + 8][2 * c] = acc[i][mt][2];
            red[warp][i][mt][g + 8][2 * c + 1] = acc[i][mt][3];
        }
    __syncthreads();

    for (int t = threadIdx.x; t < MT * 8 * 16; t += blockDim.x) {
        const int r = t & 15, tok = t >> 4, mt = tok >> 3, col = tok & 7;
        const int n = nt * 16 + r;
        if (n >= p.n || tok >= p.m) continue;
        float v[NMAT];
#pragma unroll
        for (int i = 0; i < NMAT; ++i) {
            float s = 0.0f;
#pragma unroll
            for (int w = 0; w < kGemvWarps; ++w) s += red[w][i][mt][r][col];
            v[i] = s;
        }
        float out;
        if (NMAT == 1) {
            out = v[0] * p.s0[n];
            if (p.bias) out += p.bias[n];
        } else {
            const float gv = v[0] * p.s0[n];
            const float uv = v[1] * p.s1[n];
            out = gv / (1.0f + expf(-gv)) * uv;
        }
        store_out<OutT>(p.y, (int64_t)tok * p.ldy + n, out);
    }
}

template <int XK, int MT, int NMAT>
static void launch_gemv(const GemvParams& p, int out_dtype, cudaStream_t s) {
    const dim3 grid((unsigned)ceil_div(p.n, 16)), block(kGemvWarps * 32);
    if (out_dtype == SBQ_F16)
        gemv_w8_kernel<XK, MT, NMAT, __half><<<grid, block, 0, s>>>(p);
    else
        gemv_w8_kernel<XK, MT, NMAT, float><<<grid, block, 0, s>>>(p);
}

template <int NMAT>
static void dispatch_gemv(const GemvParams& p, int xk, int out_dtype, cudaStream_t s) {
    const bool two = p.m > 8;
    switch (xk) {
        case kXF16: two ? launch_gemv<kXF16, 2, NMAT>(p, out_dtype, s) : launch_gemv<kXF16, 1, NMAT>(p, out_dtype, s); break;
        case kXBF16: two ? launch_gemv<kXBF16, 2, NMAT>(p, out_dtype, s) : launch_gemv<kXBF16, 1, NMAT>(p, out_dtype, s); break;
        default: two ? launch_gemv<kXF32, 2, NMAT>(p, out_dtype, s) : launch_gemv<kXF32, 1, NMAT>(p, out_dtype, s); break;
    }
}

static int x_kind(int dtype) {
    switch (dtype) {
        case SBQ_F16: return kXF16;
        case SBQ_BF16: return kXBF16;
        case SBQ_F32: return kXF32;
        default: return -1;
    }
}

static int elem_size(int dtype) { return dtype == SBQ_F32 ? 4 : 2; }

// Host-side validation shared by the GEMV / MLP entry points.
int check_linear_args(const void* x, int x_dtype, int64_t ldx, const void* packed, const float* scale, int64_t m,
                      int64_t n, int64_t k, const void* y, int y_dtype, int64_t ldy) {
    if (!x || !packed || !scale || !y) return set_error(SBQ_ERR_INVALID_ARGUMENT, "null pointer");
    if (m <= 0 || n <= 0 || k <= 0)
        return set_error(SBQ_ERR_INVALID_ARGUMENT, "m, n, k must be positive (m=%lld n=%lld k=%lld)", (long long)m,
                         (long long)n, (long long)k);
    if (x_kind(x_dtype) < 0) return set_error(SBQ_ERR_UNSUPPORTED, "activation dtype %d (f16, bf16, f32)", x_dtype);
    if (y_dtype != SBQ_F32 && y_dtype != SBQ_F16)
        return set_error(SBQ_ERR_UNSUPPORTED, "output dtype %d (f32, f16)", y_dtype);
    if (ldx < k || ldy < n) return set_error(SBQ_ERR_INVALID_ARGUMENT, "row stride smaller than the row");
    if (k % 16) return set_error(SBQ_ERR_UNSUPPORTED, "k must be a multiple of 16 (k=%lld)", (long long)k);
    if (reinterpret_cast<uintptr_t>(x) % 16 || (ldx * elem_size(x_dtype)) % 16)
        return set_error(SBQ_ERR_ALIGNMENT, "activation rows must be 16-byte aligned");
    if (reinterpret_cast<uintptr_t>(packed) % 256) return set_error(SBQ_ERR_ALIGNMENT, "packed weight must be 256-byte aligned");
    if (n >= (int64_t(1) << 31) || k >= (int64_t(1) << 30) || m >= (int64_t(1) << 31))
        return set_error(SBQ_ERR_UNSUPPORTED, "shape too large");
    return SBQ_OK;
}

static GemvParams make_params(const void* x, int64_t ldx, const void* w0, const float* s0, const void* w1,
                              const float* s1, const float* bias, int64_t n, int64_t k, void* y, int64_t ldy) {
    GemvParams p{};
    p.x = x;
    p.ldx = ldx;
    p.w0 = static_cast<const int8_t*>(w0);
    p.s0 = s0;
    p.w1 = static_cast<const int8_t*>(w1);
    p.s1 = s1;
    p.bias = bias;
    p.y = y;
    p.ldy = ldy;
    p.n = (int)n;
    p.k = (int)k;
    p.kt_total = (int)ceil_div(k, kTileCols);
    p.kt_per_warp = (int)ceil_div(p.kt_total, kGemvWarps);
    return p;
}

// Runs the GEMV over x in chunks of 16 rows (each chunk streams the weight once).
template <int NMAT>
static int run_gemv(GemvParams p, int64_t m, int x_dtype, int y_dtype, cudaStream_t s, const char* what) {
    const int xs = elem_size(x_dtype), ys = y_dtype == SBQ_F32 ? 4 : 2;
    for (int64_t m0 = 0; m0 < m; m0 += 16) {
        GemvParams q = p;
        q.m = (int)(m - m0 < 16 ? m - m0 : 16);
        q.x = static_cast<const char*>(p.x) + m0 * p.ldx * xs;
        q.y = static_cast<char*>(p.y) + m0 * p.ldy * ys;
        dispatch_gemv<NMAT>(q, x_kind(x_dtype), y_dtype, s);
    }
    return check_launch(what);
}

}  // namespace sbq

using namespace sbq;

extern "C" int sbq_gemv_w8(const void* x, int x_dtype, int64_t ldx, const void* packed, const float* scale,
                           const float* bias, int64_t m, int64_t n, int64_t k, void* y, int y_dtype, int64_t ldy,
                           void* stream) {
    int st = check_linear_args(x, x_dtype, ldx, packed, scale, m, n, k, y, y_dtype, ldy);
    if (st) return st;
    GemvParams p = make_params(x, ldx, packed, scale, nullptr, nullptr, bias, n, k, y, ldy);
    return run_gemv<1>(p, m, x_dtype, y_dtype, static_cast<cudaStream_t>(stream), "gemv_w8");
}

extern "C" int sbq_mlp_gateup_w8(const void* x, int x_dtype, int64_t ldx, const void* packed_gate,
                                 const float* scale_gate, const void* packed_up, const float* scale_up, int64_t m,
                                 int64_t n, int64_t k, void* h, int h_dtype, int64_t ldh, void* stream) {
    int st = check_linear_args(x, x_dtype, ldx, packed_gate, scale_gate, m, n, k, h, h_dtype, ldh);
    if (st) return st;
    if (!packed_up || !scale_up) return set_error(SBQ_ERR_INVALID_ARGUMENT, "null up-projection pointer");
    if (reinterpret_cast<uintptr_t>(packed_up) % 256) return set_error(SBQ_ERR_ALIGNMENT, "packed weight must be 256-byte aligned");
    GemvParams p = make_params(x, ldx, packed_gate, scale_gate, packed_up, scale_up, nullptr, n, k, h, ldh);
    return run_gemv<2>(p, m, x_dtype, h_dtype, static_cast<cudaStream_t>(stream), "mlp_gateup_w8");
}
