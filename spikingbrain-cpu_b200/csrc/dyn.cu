// Format "int8-dyn": dynamic activation quantisation and the int8 x int8 -> int32 tensor-memory GEMM.
//
// Reference: DynamicInt8Linear.forward (spikingbrain_cpu/quant.py:63-66), i.e. torch's
// quantized::linear_dynamic on the fbgemm/x86 engine.  Restated bit for bit:
//   1. min / max over the whole activation, widened to include 0;
//   2. torch's ChooseQuantizationParams (uint8, qmin 0, qmax 255, no range reduction): double scale,
//      zero point from whichever end rounds better, nudged with round-half-even; fp32 scale;
//   3. xq = clamp(rint(fma(x, 1/s, zp)), 0, 255), 1/s an fp32 reciprocal, one rounding;
//   4. acc = sum_k (xq - zp) * q  (int32);  5. y = float(acc) * (s * scale[n]) (fma with a bias).
// The GEMM multiplies uint8 xq by the int8 weight on the tensor cores (tcgen05 kind::i8, int32
// accumulators in tensor memory) and applies the zero-point correction acc - zp * rowsum[n] in the
// epilogue, which is exact integer arithmetic.  The per-token mode (symmetric int8, one scale per
// row, no reference counterpart) shares the GEMM with a signed A operand.
#include <atomic>
#include <cstring>

#include "tc.cuh"

namespace sbq {

// ============================================================================ quantisation ====

template <typename T>
struct Vec;
template <>
struct Vec<float> {
    static constexpr int kN = 4;
    __device__ static void load(const float* p, float (&v)[4]) {
        float4 t = __ldg(reinterpret_cast<const float4*>(p));
        v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    }
    __device__ static void cvt(const uint4& t, float (&v)[4]) {
        v[0] = __uint_as_float(t.x); v[1] = __uint_as_float(t.y); v[2] = __uint_as_float(t.z); v[3] = __uint_as_float(t.w);
    }
};
template <>
struct Vec<__half> {
    static constexpr int kN = 8;
    __device__ static void load(const __half* p, float (&v)[8]) { cvt(__ldg(reinterpret_cast<const uint4*>(p)), v); }
    __device__ static void cvt(const uint4& t, float (&v)[8]) {
        const __half2* h = reinterpret_cast<const __half2*>(&t);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float2 f = __half22float2(h[i]);
            v[2 * i] = f.x; v[2 * i + 1] = f.y;
        }
    }
};
template <>
struct Vec<__nv_bfloat16> {
    static constexpr int kN = 8;
    __device__ static void load(const __nv_bfloat16* p, float (&v)[8]) { cvt(__ldg(reinterpret_cast<const uint4*>(p)), v); }
    __device__ static void cvt(const uint4& t, float (&v)[8]) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&t);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float2 f = __bfloat1622float2(h[i]);
            v[2 * i] = f.x; v[2 * i + 1] = f.y;
        }
    }
};

constexpr int kQuantThreads = 256;
constexpr int kQuantVecs = 4;  // vectors a thread loads at once (kept in registers across a wait)
constexpr int kMaxPartials = 1024;

// Element offset of vector v (V elements) of x [m, k] with row stride ldx.
__device__ __forceinline__ int64_t vec_offset(int64_t v, int64_t per_row, int V, int64_t ldx) {
    if (ldx == per_row * V) return v * V;
    const int64_t row = v / per_row;
    return row * ldx + (v - row * per_row) * V;
}

// Two-kernel per-tensor quantisation (x up to kFusedMinBytes), step 1: per-CTA (min, max) of x [m, k] (row stride ldx; k a multiple of the vector width).  Each
// thread requests kQuantVecs vectors before folding any, so one memory latency covers them.
template <typename T>
__global__ void __launch_bounds__(kQuantThreads) minmax_partial_kernel(const T* __restrict__ x, int64_t ldx, int m,
                                                                      int k, float2* __restrict__ partials) {
    // the quantisation kernel may start now: it loads x (complete before this grid started) and
    // waits for this grid before reading the partials
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    constexpr int V = Vec<T>::kN;
    const int64_t per_row = k / V, total = (int64_t)m * per_row;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    float mn = INFINITY, mx = -INFINITY;
    for (int64_t v0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v0 < total; v0 += kQuantVecs * stride) {
        float e[kQuantVecs][V];
#pragma unroll
        for (int j = 0; j < kQuantVecs; ++j)
            if (v0 + j * stride < total) Vec<T>::load(x + vec_offset(v0 + j * stride, per_row, V, ldx), e[j]);
#pragma unroll
        for (int j = 0; j < kQuantVecs; ++j) {
            if (v0 + j * stride >= total) continue;
#pragma unroll
            for (int i = 0; i < V; ++i) {
                mn = fminf(mn, e[j][i]);
                mx = fmaxf(mx, e[j][i]);
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    __shared__ float2 red[kQuantThreads / 32];
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = make_float2(mn, mx);
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kQuantThreads / 32; ++w) {
            mn = fminf(mn, red[w].x);
            mx = fmaxf(mx, red[w].y);
        }
        partials[blockIdx.x] = make_float2(mn, mx);
    }
}


// Step 2: torch ChooseQuantizationParams (quint8, reduce_range = false, preserve_sparsity = false).
__device__ void choose_qparams(float mn, float mx, float* scale_out, int* zp_out) {
    const int qmin = 0, qmax = 255;
    const float small_scale = 6.1e-5f;
    if (mn > 0.0f) mn = 0.0f;
    if (mx < 0.0f) mx = 0.0f;
    double scale = ((double)mx - (double)mn) / (double)(qmax - qmin);
    if ((float)scale == 0.0f || isinf(__fdiv_rn(1.0f, (float)scale))) scale = 0.1;
    if (scale < (double)small_scale) {
        const float org_scale = (float)scale;
        scale = small_scale;
        if (mn == 0.0f) {
            mx = __fmul_rn(small_scale, (float)(qmax - qmin));
        } else if (mx == 0.0f) {
            mn = -__fmul_rn(small_scale, (float)(qmax - qmin));
        } else {
            const float amplifier = __fdiv_rn(small_scale, org_scale);
            mn = __fmul_rn(mn, amplifier);
            mx = __fmul_rn(mx, amplifier);
        }
    }
    const double zp_from_min = qmin - (double)mn / scale;
    const double zp_from_max = qmax - (double)mx / scale;
    const double err_min = fabs((double)qmin) - fabs((double)mn / scale);
    const double err_max = fabs((double)qmax) - fabs((double)mx / scale);
    const double zp0 = err_min < err_max ? zp_from_min : zp_from_max;
    int zp;
    if (zp0 < qmin) zp = qmin;
    else if (zp0 > qmax) zp = qmax;
    else zp = (int)rint(zp0);
    *scale_out = (float)scale;
    *zp_out = zp;
}

// Quantise V elements to V/4 packed bytes: clamp(rint(fma(x, inv, zp)), 0, 255), computed as
// rint(clamp(y, 0, 255)) - the same value, since rounding is monotonic and both bounds are integers
// (NaN: fmaxf gives 0 either way) - with the rounding done by adding 1.5 * 2^23: every float in
// [2^23, 2^24) is an integer, so the sum is y rounded to nearest even and its low mantissa byte is
// that integer (0..255).  No float -> int conversion instructions.
template <int V>
__device__ __forceinline__ void quant_u8(const float (&e)[V], float inv, float fzp, uint8_t* dst) {
    uint32_t packed[V / 4];
#pragma unroll
    for (int w = 0; w < V / 4; ++w) {
        uint32_t u[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float t = fminf(fmaxf(__fmaf_rn(e[4 * w + i], inv, fzp), 0.0f), 255.0f);
            u[i] = __float_as_uint(__fadd_rn(t, 12582912.0f));
        }
        packed[w] = __byte_perm(__byte_perm(u[0], u[1], 0x0040), __byte_perm(u[2], u[3], 0x0040), 0x5410);
    }
    if (V == 4) {
        *reinterpret_cast<uint32_t*>(dst) = packed[0];
    } else {
        *reinterpret_cast<uint2*>(dst) = make_uint2(packed[0], packed[V / 4 - 1]);
    }
}

// Step 3 of the two-kernel path, launched as a programmatic dependent of step 1.  Every CTA loads its first vectors of x
// while step 1 still runs, then waits for it, folds the partials and derives the parameters itself
// (identical result, no grid-wide synchronisation or counters); CTA 0 publishes them.
template <typename T>
__global__ void __launch_bounds__(kQuantThreads) quantize_per_tensor_kernel(const T* __restrict__ x, int64_t ldx, int m,
                                                                           int k, const float2* __restrict__ partials,
                                                                           int nparts, uint8_t* __restrict__ xq,
                                                                           float* __restrict__ s_out,
                                                                           int32_t* __restrict__ zp_out) {
    // the GEMM launched next prepares its pipeline and streams its first weight tiles meanwhile; it
    // waits for this grid before reading xq and the parameters
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    constexpr int V = Vec<T>::kN;
    const int64_t per_row = k / V, total = (int64_t)m * per_row;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t first = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    float e[kQuantVecs][V];
#pragma unroll
    for (int j = 0; j < kQuantVecs; ++j)
        if (first + j * stride < total) Vec<T>::load(x + vec_offset(first + j * stride, per_row, V, ldx), e[j]);
    asm volatile("griddepcontrol.wait;" ::: "memory");  // the partials are step 1's output

    __shared__ float2 red[kQuantThreads / 32];
    __shared__ float s_inv, s_zp;
    float mn = INFINITY, mx = -INFINITY;
    for (int i = threadIdx.x; i < nparts; i += blockDim.x) {
        const float2 p = partials[i];
        mn = fminf(mn, p.x);
        mx = fmaxf(mx, p.y);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = make_float2(mn, mx);
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kQuantThreads / 32; ++w) {
            mn = fminf(mn, red[w].x);
            mx = fmaxf(mx, red[w].y);
        }
        float s;
        int zp;
        choose_qparams(mn, mx, &s, &zp);
        s_inv = __fdiv_rn(1.0f, s);
        s_zp = (float)zp;
        if (blockIdx.x == 0) {
            *s_out = s;
            *zp_out = zp;
        }
    }
    __syncthreads();
    const float inv = s_inv, fzp = s_zp;
    for (int64_t v0 = first; v0 < total; v0 += kQuantVecs * stride) {
        if (v0 != first) {
#pragma unroll
            for (int j = 0; j < kQuantVecs; ++j)
                if (v0 + j * stride < total) Vec<T>::load(x + vec_offset(v0 + j * stride, per_row, V, ldx), e[j]);
        }
#pragma unroll
        for (int j = 0; j < kQuantVecs; ++j) {
            const int64_t v = v0 + j * stride;
            if (v >= total) continue;
            const int64_t row = v / per_row;
            quant_u8<V>(e[j], inv, fzp, xq + row * (int64_t)k + (v - row * per_row) * V);
        }
    }
}

// Grid barrier of the per-tensor quantiser (one per stream lane).  Every CTA reads the generation
// before it arrives; arrivals count modulo the grid size (atomicInc wraps the count to zero on the
// last one), and the last CTA to arrive bumps the generation while the others wait (bounded) for the
// bump.  The counters start at zero with the library and are left at zero for the next launch, so no
// memset precedes a launch and CUDA graphs replay it as captured.  The grid is a cooperative launch:
// all of its CTAs are resident together.
__device__ unsigned g_qbar_count[kStreamLanes];
__device__ unsigned g_qbar_gen[kStreamLanes];

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_gpu(unsigned* p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// atomicInc with acquire-release semantics at GPU scope
__device__ __forceinline__ unsigned atom_inc_acq_rel_gpu(unsigned* p, unsigned limit) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.inc.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(limit) : "memory");
    return old;
}

// Returns false (error word set) if the other CTAs did not arrive within the wait limit.  `gen` is
// the generation thread 0 read (acquire) before this CTA's arrival, e.g. at the start of the kernel.
// Arrivals are acquire-release atomics (each publishes its CTA's partial and the last one acquires
// all of them); the last CTA's release store of the new generation publishes them to the waiters.
__device__ bool quant_grid_barrier(int lane, unsigned gen, int* s_flag) {
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned old = atom_inc_acq_rel_gpu(&g_qbar_count[lane], gridDim.x - 1);
        int ok = 1;
        if (old >= gridDim.x - 1) {
            st_release_gpu(&g_qbar_gen[lane], gen + 1);
        } else {
            const uint64_t t0 = tc::now_ns();
            for (uint32_t i = 1; ld_acquire_gpu(&g_qbar_gen[lane]) == gen; ++i) {
                if (i > 64) __nanosleep(32);
                if ((i & 255) == 0 && tc::now_ns() - t0 > tc::kWaitLimitNs) {
                    tc::raise_error(SBQ_ERR_TIMEOUT);
                    ok = 0;
                    break;
                }
            }
        }
        *s_flag = ok;
    }
    __syncthreads();
    return *s_flag != 0;
}

// Per-tensor quantisation of larger x (at least kFusedMinBytes; fbgemm / torch quint8, the
// reference's DynamicInt8Linear step) in one cooperative launch, which reads x from memory once: (1) each thread loads up to kFusedVecs vectors of x into registers (128 bytes)
// and the CTA folds their (min, max) into partials[blockIdx.x]; (2) grid barrier; (3) every CTA folds
// all partials, derives the parameters itself (ChooseQuantizationParams: identical in every CTA) and
// quantises the vectors it holds; CTA 0 publishes s and zp.  When x is larger than the registers
// of the grid hold, step 1 walks all of its vectors and step 3 reads them again.
constexpr int kFusedThreads = 512;
// x of at least this many bytes takes the one-launch quantiser.  Measured on B200 (CUDA graphs, m x
// 4096 fp32): the grid barrier costs more than the two-kernel path's programmatic launch boundary,
// so small x (1-3 MB) ran ~2 us slower in one launch, 8 MB (m = 512) the same, and 64 MB 12 us
// faster (x read once instead of twice).
constexpr int64_t kFusedMinBytes = int64_t(8) << 20;
#ifndef SBQ_QUANT_COOP
#define SBQ_QUANT_COOP 1
#endif
template <typename T>
struct FusedVecs {
    static constexpr int kN = 8;  // 16-byte vectors per thread: 128 bytes of x held in registers
};

template <typename T>
__global__ void __launch_bounds__(kFusedThreads, 1)
    quantize_per_tensor_fused_kernel(const T* __restrict__ x, int64_t ldx, int m, int k,
                                     float2* __restrict__ partials, uint8_t* __restrict__ xq,
                                     float* __restrict__ s_out, int32_t* __restrict__ zp_out, int lane) {
    // the GEMM launched next prepares its pipeline and streams its first weight tiles meanwhile; it
    // waits for this grid before reading xq and the parameters
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // the barrier generation before this launch's arrivals (read now: its latency overlaps the loads)
    const unsigned gen = threadIdx.x == 0 && gridDim.x > 1 ? ld_acquire_gpu(&g_qbar_gen[lane]) : 0u;
    constexpr int V = Vec<T>::kN, NV = FusedVecs<T>::kN;
    const int64_t per_row = k / V, total = (int64_t)m * per_row;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t first = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const bool cached = total <= stride * NV;
    const bool dense = ldx == k;  // rows back to back: vector v of x and of xq at v * V

    uint4 raw[NV];  // 16 bytes of x per vector, as loaded (converted to fp32 where used)
    float mn = INFINITY, mx = -INFINITY;
    for (int64_t v0 = first; v0 < total; v0 += NV * stride) {
#pragma unroll
        for (int j = 0; j < NV; ++j)
            if (v0 + j * stride < total)
                raw[j] = __ldg(reinterpret_cast<const uint4*>(
                    x + (dense ? (v0 + j * stride) * V : vec_offset(v0 + j * stride, per_row, V, ldx))));
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            if (v0 + j * stride >= total) continue;
            float e[V];
            Vec<T>::cvt(raw[j], e);
#pragma unroll
            for (int i = 0; i < V; ++i) {
                mn = fminf(mn, e[i]);
                mx = fmaxf(mx, e[i]);
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    __shared__ float2 red[kFusedThreads / 32];
    __shared__ float s_inv, s_zp;
    __shared__ int s_flag;
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = make_float2(mn, mx);
    __syncthreads();
    if (gridDim.x > 1) {  // (a one-CTA grid, for small x, has the whole reduction in red[] already)
        if (threadIdx.x == 0) {
            for (int w = 1; w < kFusedThreads / 32; ++w) {
                mn = fminf(mn, red[w].x);
                mx = fmaxf(mx, red[w].y);
            }
            partials[blockIdx.x] = make_float2(mn, mx);
        }
        if (!quant_grid_barrier(lane, gen, &s_flag)) return;

        mn = INFINITY;
        mx = -INFINITY;
        for (int i = threadIdx.x; i < (int)gridDim.x; i += blockDim.x) {
            const float2 q = __ldcg(partials + i);  // written by other SMs in this launch: read through L2
            mn = fminf(mn, q.x);
            mx = fmaxf(mx, q.y);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        }
        __syncthreads();  // red[] is reused
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = make_float2(mn, mx);
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        for (int w = 1; w < kFusedThreads / 32; ++w) {
            mn = fminf(mn, red[w].x);
            mx = fmaxf(mx, red[w].y);
        }
        float s;
        int zp;
        choose_qparams(mn, mx, &s, &zp);
        s_inv = __fdiv_rn(1.0f, s);
        s_zp = (float)zp;
        if (blockIdx.x == 0) {
            *s_out = s;
            *zp_out = zp;
        }
    }
    __syncthreads();
    const float inv = s_inv, fzp = s_zp;
    for (int64_t v0 = first; v0 < total; v0 += NV * stride) {
        if (!cached) {
#pragma unroll
            for (int j = 0; j < NV; ++j)
                if (v0 + j * stride < total)
                    raw[j] = __ldg(reinterpret_cast<const uint4*>(
                        x + (dense ? (v0 + j * stride) * V : vec_offset(v0 + j * stride, per_row, V, ldx))));
        }
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int64_t v = v0 + j * stride;
            if (v >= total) continue;
            int64_t off = v * V;
            if (!dense) {
                const int64_t row = v / per_row;
                off = row * (int64_t)k + (v - row * per_row) * V;
            }
            float e[V];
            Vec<T>::cvt(raw[j], e);
            quant_u8<V>(e, inv, fzp, xq + off);
        }
    }
}

// Per-token symmetric mode: one CTA per row, s_t = max(max|x_t|, 1e-8) / 127, xq = clamp(rint(x / s_t)).
// Rows of up to kQuantVecs * kTokThreads vectors stay in registers between the two passes.
constexpr int kTokThreads = 128;

template <typename T>
__global__ void __launch_bounds__(kTokThreads) quantize_per_token_kernel(const T* __restrict__ x, int64_t ldx, int m,
                                                                        int k, int8_t* __restrict__ xq,
                                                                        float* __restrict__ s_tok) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // as in the per-tensor step 3
    constexpr int V = Vec<T>::kN;
    const int row = blockIdx.x;
    const int per_row = k / V;
    const bool cached = per_row <= kQuantVecs * kTokThreads;
    const T* xr = x + (int64_t)row * ldx;
    float e[kQuantVecs][V];
    float amax = 0.0f;
    if (cached) {
#pragma unroll
        for (int j = 0; j < kQuantVecs; ++j)
            if (threadIdx.x + j * kTokThreads < per_row) Vec<T>::load(xr + (threadIdx.x + j * kTokThreads) * V, e[j]);
#pragma unroll
        for (int j = 0; j < kQuantVecs; ++j) {
            if (threadIdx.x + j * kTokThreads >= per_row) continue;
#pragma unroll
            for (int i = 0; i < V; ++i) amax = fmaxf(amax, fabsf(e[j][i]));
        }
    } else {
        for (int c = threadIdx.x; c < per_row; c += kTokThreads) {
            Vec<T>::load(xr + c * V, e[0]);
#pragma unroll
            for (int i = 0; i < V; ++i) amax = fmaxf(amax, fabsf(e[0][i]));
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    __shared__ float red[kTokThreads / 32];
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
#pragma unroll
    for (int w = 0; w < kTokThreads / 32; ++w) amax = fmaxf(amax, red[w]);
    const float s = __fdiv_rn(fmaxf(amax, 1e-8f), 127.0f);
    int8_t* dst = xq + (int64_t)row * k;
    auto put = [&](const float (&v)[V], int c) {
        uint32_t packed[V / 4];
#pragma unroll
        for (int w = 0; w < V / 4; ++w) {
            uint32_t word = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float t = rintf(__fdiv_rn(v[4 * w + i], s));
                t = fminf(fmaxf(t, -127.0f), 127.0f);
                word |= ((uint32_t)(int32_t)t & 0xFFu) << (8 * i);
            }
            packed[w] = word;
        }
        if (V == 4) {
            *reinterpret_cast<uint32_t*>(dst + c * V) = packed[0];
        } else {
            *reinterpret_cast<uint2*>(dst + c * V) = make_uint2(packed[0], packed[V / 4 - 1]);
        }
    };
    if (cached) {
#pragma unroll
        for (int j = 0; j < kQuantVecs; ++j)
            if (threadIdx.x + j * kTokThreads < per_row) put(e[j], threadIdx.x + j * kTokThreads);
    } else {
        for (int c = threadIdx.x; c < per_row; c += kTokThreads) {
            Vec<T>::load(xr + c * V, e[0]);
            put(e[0], c);
        }
    }
    if (threadIdx.x == 0) s_tok[row] = s;
}

// ============================================================================ int8 GEMM ======
//
// One CTA computes a 128 (xq rows) x BN (weight rows) output tile, BN = 256 or 128: 4-stage TMA ring
// (xq 128 x 128 B with 128-byte swizzle, weight two BN x 64 B halves with 64-byte swizzle), one
// thread issues tcgen05.mma.cta_group::1.kind::i8 (M = 128, N = BN, K = 32) into int32 accumulators
// in tensor memory.  A per-k-block trace showed the issuing thread held about as long per MMA at
// N = 128 as at N = 256 (~150 cycles), so the 256-wide tile does twice the work per k-block; it is
// used when its tiles still cover the GPU.  When they would leave SMs idle (configuration 3: 64 such
// tiles for 148 SMs) the 128-wide tile, at twice the tile count, is as fast in total; splitting the
// K range of 256-wide tiles over a CTA pair and exchanging int32 partials (through distributed shared
// memory, or through L2) measured slower than either, the exchange being latency-bound.
// The per-channel factors are loaded by otherwise idle warps while the first tiles stream in;
// epilogue (8 warps; warps w and w + 4 share tensor-memory lanes and split the column blocks):
// acc - zp * rowsum[n], float(acc) * (s * scale[n]) (fma with a bias), staged in the freed ring and
// written with TMA stores.

struct GemmI8Params {
    int m, n, k, num_kb;
    const int32_t* rowsum;  // per-tensor zero-point correction (may be null in per-token mode)
    const float* s_x;       // one scale (per-tensor) or one per row (per-token)
    int s_stride;           // 0 or 1
    const int32_t* zp;      // per-tensor zero point (null in per-token mode)
    const float* scale;
    const float* bias;
    float* y;
    int64_t ldy;
    int32_t* acc_out;       // optional int32 accumulators (zero-point corrected), row stride n
    int tma_y;              // y is written by TMA stores through tmap_y (no acc_out, aligned rows)
    int vec_y;              // y (and acc_out) rows take 16-byte vector stores: both base pointers 16-byte
                            // aligned, ldy and n multiples of 4; otherwise the epilogue stores element-wise
    int parts;              // K parts of the single-CTA kernel (a cluster along z; 1 = no split)
    int a_rows;             // xq rows the single-CTA kernel loads per tile (up to 128; the MMA reads 128,
                            // rows past them hold stale bytes whose products land in unused output rows)
};

constexpr int kI8BM = 128;         // rows of xq per tile (MMA M)
constexpr int kI8BK = 128;         // k per pipeline stage (bytes of an int8 row = one 128-byte swizzle row)
#ifndef SBQ_I8_STAGES
#define SBQ_I8_STAGES 4
#endif
constexpr int kI8Stages = SBQ_I8_STAGES;
#ifndef SBQ_I8_STAGES_128
#define SBQ_I8_STAGES_128 6
#endif
constexpr int kI8Threads = 256;                // 8 warps
constexpr int kI8SlotBytes = kI8BM * 32 * 4;   // staging of one 32-column block: 128 rows x 128 B

template <int BN>
struct I8Smem {
    static constexpr int kA = kI8BM * kI8BK;  // 16 KiB
    static constexpr int kB = BN * kI8BK;     // two 64-wide halves of BN rows
    static constexpr int kStage = kA + kB;
    // stages: as many as the build sets for the tile width (the 128-wide tile's are smaller)
    static constexpr int kStages = BN == 128 ? SBQ_I8_STAGES_128 : kI8Stages;
    static constexpr int kRing = kStages * kStage;
    static constexpr int kTail = 256 /* barriers */ + BN * 5 * 4;  // scale, bias, rowsum, s*scale, zp*rowsum
    static constexpr int kBytes = kRing + 1024 /* alignment */ + kTail;
    static_assert((BN / 32) * kI8SlotBytes <= kRing, "epilogue staging fits in the ring");
    static_assert(BN * kI8BM * 4 <= kRing, "split-K receive buffer fits in the ring");
    static_assert(kBytes <= 227 * 1024, "shared memory per CTA");
};

// Per-channel epilogue factors of the tile's BN weight rows from n0, loaded by warps 2 and 3 while the
// main loop runs: scale, bias, row sums and, per tensor, s_x * scale[n] and zp * rowsum[n] (s_x and
// zp are the previous kernel's output: read after griddepcontrol.wait, which these otherwise idle
// warps can afford to block on).  Each thread computes the products of the entries it loaded.
template <int BN>
__device__ __forceinline__ void i8_load_factors(const GemmI8Params& p, int n0, float* s_scale, float* s_bias,
                                                int32_t* s_rowsum, float* s_f, int32_t* s_zr) {
    for (int i = threadIdx.x - 64; i < BN; i += 64) {
        const int n = n0 + i;
        s_scale[i] = n < p.n ? p.scale[n] : 0.0f;
        s_bias[i] = (p.bias && n < p.n) ? p.bias[n] : 0.0f;
        s_rowsum[i] = (p.rowsum && n < p.n) ? p.rowsum[n] : 0;
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (p.s_stride == 0) {
        const float sx0 = p.s_x[0];
        const int32_t zp = p.zp ? *p.zp : 0;
        for (int i = threadIdx.x - 64; i < BN; i += 64) {
            s_f[i] = __fmul_rn(sx0, s_scale[i]);
            s_zr[i] = zp * s_rowsum[i];
        }
    }
}

// Epilogue of the int8 GEMMs, run by all 8 warps of a CTA after its accumulators (128 xq rows x BN
// weight rows from row m0 / column n0, int32 in tensor memory from column 0) are complete: one lane
// per warp polls `done` (with back-off) so idle threads do not compete with the producer and MMA
// threads; the decision is warp-uniform (tcgen05.ld is warp-collective).  Warps w and w + 4 share
// lane quarter w % 4 and split the 32-column blocks.
template <int BN>
__device__ __forceinline__ void i8_epilogue(const GemmI8Params& p, const CUtensorMap* tmap_y, uint8_t* smem,
                                            uint64_t* done, int* abort_flag, const float* s_scale,
                                            const float* s_bias, const int32_t* s_rowsum, float* s_f, int32_t* s_zr,
                                            uint32_t tmem, int m0, int n0) {
    constexpr int kBlocks = BN / 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool per_tensor = p.s_stride == 0;
    const int g = warp & 3, h = warp >> 2;  // lane group, column-block half
    const uint32_t lane_base = tmem + ((uint32_t)(g * 32) << 16);
    const int row = m0 + g * 32 + lane;
    // the per-token scale of this thread's row comes from the previous kernel; it is read before the
    // accumulators are complete (the producer's griddepcontrol.wait has long returned by then)
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const float sx = per_tensor ? 0.0f : p.s_x[row < p.m ? row : 0];
    int waited = 1;
    if (lane == 0) waited = tc::mbar_wait_backoff(done, 0) && !*(volatile int*)abort_flag;
    const bool ok = __shfl_sync(0xffffffffu, waited, 0) != 0;
    tc::fence_after_sync();
    __syncthreads();  // the factors of warps 2, 3 (i8_load_factors) are in shared memory
    if (ok) {
#pragma unroll 1
        for (int b = h; b < kBlocks; b += 2) {
            const int nb = n0 + b * 32;
            uint32_t r[32];
            tc::tmem_ld_32x32b_x32(lane_base + b * 32, r);
            tc::tmem_wait_ld();
            float v[32];
            int32_t a[32];
#pragma unroll
            for (int j4 = 0; j4 < 8; ++j4) {
                const int i = b * 32 + 4 * j4;
                const float4 f4 = per_tensor ? *reinterpret_cast<const float4*>(s_f + i)
                                             : make_float4(__fmul_rn(sx, s_scale[i]), __fmul_rn(sx, s_scale[i + 1]),
                                                           __fmul_rn(sx, s_scale[i + 2]), __fmul_rn(sx, s_scale[i + 3]));
                const int4 z4 = per_tensor ? *reinterpret_cast<const int4*>(s_zr + i) : make_int4(0, 0, 0, 0);
                const float4 b4 = *reinterpret_cast<const float4*>(s_bias + i);
                const float fs[4] = {f4.x, f4.y, f4.z, f4.w}, bs[4] = {b4.x, b4.y, b4.z, b4.w};
                const int zs[4] = {z4.x, z4.y, z4.z, z4.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int jj = 4 * j4 + e;
                    a[jj] = (int32_t)r[jj] - zs[e];
                    const float af = __int2float_rn(a[jj]);
                    v[jj] = p.bias ? __fmaf_rn(af, fs[e], bs[e]) : __fmul_rn(af, fs[e]);
                }
            }
            if (p.tma_y) {
                // the lane group's 32 x 32 fp32 block: 32 rows of 128 bytes, 16-byte unit j of row r at
                // j ^ (r % 8) (128-byte swizzle), staged in slot b of the freed ring
                uint8_t* reg = smem + b * kI8SlotBytes + g * 4096;
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    *reinterpret_cast<float4*>(reg + lane * 128 + ((j ^ (lane & 7)) * 16)) =
                        make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                tc::fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0 && m0 + g * 32 < p.m && nb < p.n) {
                    tc::tma_store_2d(tmap_y, reg, nb, m0 + g * 32);
                    tc::bulk_commit_group();
                }
                continue;
            }
            if (row >= p.m) continue;
            float* yrow = p.y + (int64_t)row * p.ldy;
            int32_t* arow = p.acc_out ? p.acc_out + (int64_t)row * p.n : nullptr;
            if (nb + 32 <= p.n && p.vec_y) {
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                    *reinterpret_cast<float4*>(yrow + nb + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                    if (arow) *reinterpret_cast<int4*>(arow + nb + j) = make_int4(a[j], a[j + 1], a[j + 2], a[j + 3]);
                }
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    if (nb + j < p.n) {
                        yrow[nb + j] = v[j];
                        if (arow) arow[nb + j] = a[j];
                    }
                }
            }
        }
    }
    if (p.tma_y && lane == 0) tc::bulk_wait_all_read();  // the staged blocks stay in use until read
}

// Split-K epilogue of the single-CTA kernel (one 128-row xq tile, K cut over a cluster of p.parts
// CTAs along z).  (1) A cluster barrier: every CTA's main loop is done, so every ring is free.  (2)
// Each warp whose 32 xq rows include valid ones pushes its int32 partial sums into the shared memory
// of the CTA owning each channel (BN / parts channels per CTA), column-major recv[part][channel][row]
// so that a warp (32 consecutive rows) stores 128 contiguous bytes per channel.  (3) A cluster
// barrier, then each CTA adds the parts of its channels in part order - integer sums, so the result
// equals the unsplit kernel's bit for bit - and applies the epilogue arithmetic of i8_epilogue.
template <int BN>
__device__ __forceinline__ void i8_splitk_epilogue(const GemmI8Params& p, uint8_t* smem, uint64_t* done,
                                                   int* abort_flag, const float* s_scale, const float* s_bias,
                                                   const float* s_f, const int32_t* s_zr, uint32_t tmem, int m0,
                                                   int n0, int part) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = warp & 3, h = warp >> 2;
    const int share = BN / p.parts;
    int32_t* recv = reinterpret_cast<int32_t*>(smem);  // [parts][share][kI8BM]
    int waited = 1;
    if (lane == 0) waited = tc::mbar_wait_backoff(done, 0) && !*(volatile int*)abort_flag;
    const bool ok = __shfl_sync(0xffffffffu, waited, 0) != 0;
    tc::fence_after_sync();
    tc::cluster_sync();
    if (m0 + g * 32 < p.m) {
        const uint32_t lane_base = tmem + ((uint32_t)(g * 32) << 16);
        const int row = g * 32 + lane;
#pragma unroll 1
        for (int b = h; b < BN / 32; b += 2) {
            uint32_t r[32];
            tc::tmem_ld_32x32b_x32(lane_base + b * 32, r);
            tc::tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const int c = b * 32 + j, q = c / share;
                const uint32_t a = tc::cluster_addr(recv + ((part * share + (c - q * share)) * kI8BM + row), (uint32_t)q);
                const int32_t v = ok ? (int32_t)r[j] : 0;
                asm volatile("st.shared::cluster.s32 [%0], %1;" ::"r"(a), "r"(v) : "memory");
            }
        }
    }
    tc::cluster_sync();
    asm volatile("griddepcontrol.wait;" ::: "memory");  // s_x (per token) and y belong to the previous kernel's era
    const bool per_tensor = p.s_stride == 0;
    const int rows = p.m - m0 < kI8BM ? p.m - m0 : kI8BM;
    for (int e = threadIdx.x; e < rows * share; e += blockDim.x) {
        const int cl = e % share, row = e / share;  // channels fastest: y stores along a row
        const int c = part * share + cl, n = n0 + c;
        if (n >= p.n) continue;
        int32_t acc = recv[cl * kI8BM + row];
        for (int q = 1; q < p.parts; ++q) acc += recv[(q * share + cl) * kI8BM + row];
        const int t = m0 + row;
        const int32_t a = acc - (per_tensor ? s_zr[c] : 0);
        const float f = per_tensor ? s_f[c] : __fmul_rn(p.s_x[t], s_scale[c]);
        const float af = __int2float_rn(a);
        p.y[(int64_t)t * p.ldy + n] = p.bias ? __fmaf_rn(af, f, s_bias[c]) : __fmul_rn(af, f);
        if (p.acc_out) p.acc_out[(int64_t)t * p.n + n] = a;
    }
}

// Warp 0: TMA producer.  Warp 1: MMA issuer.  Warp 2: TMEM allocation.  Warps 2, 3: per-channel
// epilogue factors.  All eight warps: epilogue (warp w reads accumulator lanes 32 (w % 4) ..).
template <int BN, bool A_SIGNED>
__global__ void __launch_bounds__(kI8Threads, 1) gemm_w8a8_kernel(const __grid_constant__ CUtensorMap tmap_a,
                                                                 const __grid_constant__ CUtensorMap tmap_b,
                                                                 const __grid_constant__ CUtensorMap tmap_y,
                                                                 const GemmI8Params p) {
    using S = I8Smem<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kRing);
    uint64_t* empty = full + S::kStages;
    uint64_t* done = empty + S::kStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
    float* s_scale = reinterpret_cast<float*>(smem + S::kRing + 256);
    float* s_bias = s_scale + BN;
    int32_t* s_rowsum = reinterpret_cast<int32_t*>(s_bias + BN);
    float* s_f = reinterpret_cast<float*>(s_rowsum + BN);   // s_x * scale[n] (per-tensor mode)
    int32_t* s_zr = reinterpret_cast<int32_t*>(s_f + BN);   // zp * rowsum[n]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.y * kI8BM, n0 = blockIdx.x * BN;
    const int part = p.parts > 1 ? (int)tc::cluster_ctarank() : 0;  // K part (cluster along z)
    const int kb0 = part * p.num_kb / p.parts;
    const int nkb = (part + 1) * p.num_kb / p.parts - kb0;
    const uint32_t stage_bytes = (uint32_t)(p.a_rows * kI8BK + S::kB);  // the xq box plus the weight tile

    if (threadIdx.x == 0) {
        for (int s = 0; s < S::kStages; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 1);
        }
        tc::mbar_init(done, 1);
        *abort_flag = 0;
        tc::fence_mbar_init();
        tc::prefetch_tmap(&tmap_a);
        tc::prefetch_tmap(&tmap_b);
        if (p.tma_y) tc::prefetch_tmap(&tmap_y);
    }
    if (warp == 2) {
        tc::tmem_alloc(tmem_slot, BN);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---- producer.  The weight tiles do not depend on the previous kernel (the activation
            // quantisation, when launched from sbq_linear_dyn as its programmatic dependent): those of
            // the first stages are requested before griddepcontrol.wait, the activation tiles after it.
            const int pre = nkb < S::kStages ? nkb : S::kStages;
            for (int i = 0; i < pre; ++i) {
                uint8_t* b_s = smem + i * S::kStage + S::kA;
                const int kb = kb0 + i;
                tc::mbar_arrive_expect_tx(&full[i], stage_bytes);
                tc::tma_load_4d(b_s, &tmap_b, &full[i], 0, 0, 2 * kb, n0 / 16);
                tc::tma_load_4d(b_s + BN * 64, &tmap_b, &full[i], 0, 0, 2 * kb + 1, n0 / 16);
            }
            asm volatile("griddepcontrol.wait;" ::: "memory");
            for (int i = 0; i < pre; ++i) tc::tma_load_2d(smem + i * S::kStage, &tmap_a, &full[i], (kb0 + i) * kI8BK, m0);
            for (int i = pre; i < nkb; ++i) {
                const int s = i % S::kStages, kb = kb0 + i;
                const uint32_t phase = (i / S::kStages) & 1;
                if (!tc::mbar_wait(&empty[s], phase ^ 1)) { *abort_flag = 1; break; }
                if (*(volatile int*)abort_flag) break;
                uint8_t* a_s = smem + s * S::kStage;
                uint8_t* b_s = a_s + S::kA;
                tc::mbar_arrive_expect_tx(&full[s], stage_bytes);
                tc::tma_load_2d(a_s, &tmap_a, &full[s], kb * kI8BK, m0);
                tc::tma_load_4d(b_s, &tmap_b, &full[s], 0, 0, 2 * kb, n0 / 16);
                tc::tma_load_4d(b_s + BN * 64, &tmap_b, &full[s], 0, 0, 2 * kb + 1, n0 / 16);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer
            constexpr uint32_t idesc = tc::idesc_i8(A_SIGNED, kI8BM, BN);
            for (int i = 0; i < nkb; ++i) {
                const int s = i % S::kStages;
                const uint32_t phase = (i / S::kStages) & 1;
                if (!tc::mbar_wait(&full[s], phase)) { *abort_flag = 1; break; }
                tc::fence_after_sync();
                const uint8_t* a_s = smem + s * S::kStage;
                const uint8_t* b_s = a_s + S::kA;
#pragma unroll
                for (int j = 0; j < kI8BK / 32; ++j) {
                    const uint64_t ad = tc::smem_desc(a_s + j * 32, tc::kSwizzle128B, 1024);
                    const uint64_t bd = tc::smem_desc(b_s + (j >> 1) * (BN * 64) + (j & 1) * 32, tc::kSwizzle64B, 512);
                    tc::mma_i8(tmem, ad, bd, idesc, (i | j) != 0);
                }
                tc::mma_commit(&empty[s]);
            }
            tc::mma_commit(done);
        }
    } else if (warp == 2 || warp == 3) {
        i8_load_factors<BN>(p, n0, s_scale, s_bias, s_rowsum, s_f, s_zr);  // off the producer's critical path
    }
    __syncwarp();
    if (p.parts > 1) {
        __syncthreads();  // the factors of warps 2, 3 are in shared memory
        i8_splitk_epilogue<BN>(p, smem, done, abort_flag, s_scale, s_bias, s_f, s_zr, tmem, m0, n0, part);
    } else {
        i8_epilogue<BN>(p, &tmap_y, smem, done, abort_flag, s_scale, s_bias, s_rowsum, s_f, s_zr, tmem, m0, n0);
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 2) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, BN);
    }
}

// ---- CTA-pair variant (more than 128 xq rows) ---------------------------------------------------
// A 2-CTA cluster computes a 256 (xq rows) x BN (weight rows) tile with
// tcgen05.mma.cta_group::2.kind::i8 (M = 256 over both CTAs' tensor memory): each CTA loads its own
// 128 xq rows and half of the BN weight rows, so a 128-deep k-block moves 16 + BN/2 * 128 / 1024 KiB
// into each SM instead of 16 + BN * 128 / 1024 KiB.  Timed without MMAs, the single-CTA loop ran at
// the SM's L2 -> shared-memory rate (32 KiB per k-block in ~0.25 us), above the MMA time.  Each
// stage holds kKH k-blocks so the MMA thread's wait and commit cover 4 kKH MMAs.  All loads of a
// stage complete on the leader's (rank 0's) barrier; the leader's commits release each CTA's stage.
#ifndef SBQ_I8P_KH
#define SBQ_I8P_KH 2
#endif

template <int BN>
struct I8PairSmem {
    static constexpr int kKH = SBQ_I8P_KH;              // 128-deep k-blocks per stage
    static constexpr int kASub = kI8BM * kI8BK;         // 16 KiB: this CTA's 128 xq rows
    static constexpr int kBHalf = (BN / 2) * 64;        // one 64-byte column of this CTA's BN/2 weight rows
    static constexpr int kBSub = 2 * kBHalf;
    static constexpr int kStage = kKH * (kASub + kBSub);
    static constexpr int kStages = (200 * 1024) / kStage < 8 ? (200 * 1024) / kStage : 8;
    static constexpr int kRing = kStages * kStage;
    static constexpr int kTail = 256 /* barriers */ + BN * 5 * 4;
    static constexpr int kBytes = kRing + 1024 /* alignment */ + kTail;
    static_assert(kStages >= 2, "pipeline depth");
    static_assert((BN / 32) * kI8SlotBytes <= kRing, "epilogue staging fits in the ring");
    static_assert(kBytes <= 227 * 1024, "shared memory per CTA");
};

template <int BN, bool A_SIGNED>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kI8Threads, 1)
    gemm_w8a8_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                          const __grid_constant__ CUtensorMap tmap_y, const GemmI8Params p) {
    using S = I8PairSmem<BN>;
    constexpr int kStages = S::kStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kRing);  // the leader's: both CTAs' loads landed
    uint64_t* empty = full + kStages;                               // this CTA's stage read by the pair's MMAs
    uint64_t* done = empty + kStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
    float* s_scale = reinterpret_cast<float*>(smem + S::kRing + 256);
    float* s_bias = s_scale + BN;
    int32_t* s_rowsum = reinterpret_cast<int32_t*>(s_bias + BN);
    float* s_f = reinterpret_cast<float*>(s_rowsum + BN);
    int32_t* s_zr = reinterpret_cast<int32_t*>(s_f + BN);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = tc::cluster_ctarank();
    const bool leader = rank == 0;
    const int m0 = blockIdx.x * kI8BM;          // this CTA's 128 xq rows (the pair's 256 are adjacent)
    const int n0 = blockIdx.y * BN;             // the pair's BN weight rows (output columns)
    const int nb0 = n0 + (int)rank * (BN / 2);  // the half this CTA loads
    const int nkb = p.num_kb;                   // stages (kKH k-blocks each)

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 1);
        }
        tc::mbar_init(done, 1);
        *abort_flag = 0;
        tc::fence_mbar_init();
        tc::prefetch_tmap(&tmap_a);
        tc::prefetch_tmap(&tmap_b);
        if (p.tma_y) tc::prefetch_tmap(&tmap_y);
    }
    if (warp == 2) {
        tc::tmem_alloc_pair(tmem_slot, BN);
        tc::tmem_relinquish_pair();
    }
    tc::fence_before_sync();
    tc::cluster_sync();  // both CTAs' barriers exist before either CTA's loads or commits reach them
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---- producer (both CTAs).  Weight tiles of the first stages before griddepcontrol.wait
            // (they do not depend on the activation quantisation), activation tiles after it.
            const int pre = nkb < kStages ? nkb : kStages;
            for (int i = 0; i < pre; ++i) {
                uint8_t* b_s = smem + i * S::kStage + S::kKH * S::kASub;
                const uint32_t fb = tc::cluster_addr(&full[i], 0);
                if (leader) tc::mbar_arrive_expect_tx(&full[i], 2 * S::kStage);
#pragma unroll
                for (int h = 0; h < S::kKH; ++h) {
                    const int kc = 2 * (i * S::kKH + h);  // 64-byte weight tile column
                    tc::tma_load_4d_pair(b_s + h * S::kBSub, &tmap_b, fb, 0, 0, kc, nb0 / 16);
                    tc::tma_load_4d_pair(b_s + h * S::kBSub + S::kBHalf, &tmap_b, fb, 0, 0, kc + 1, nb0 / 16);
                }
            }
            asm volatile("griddepcontrol.wait;" ::: "memory");
            for (int i = 0; i < pre; ++i) {
                const uint32_t fb = tc::cluster_addr(&full[i], 0);
#pragma unroll
                for (int h = 0; h < S::kKH; ++h)
                    tc::tma_load_2d_pair(smem + i * S::kStage + h * S::kASub, &tmap_a, fb, (i * S::kKH + h) * kI8BK, m0);
            }
            for (int i = pre; i < nkb; ++i) {
                const int s = i % kStages;
                const uint32_t phase = (i / kStages) & 1;
                if (!tc::mbar_wait(&empty[s], phase ^ 1)) { *abort_flag = 1; break; }
                if (*(volatile int*)abort_flag) break;
                uint8_t* a_s = smem + s * S::kStage;
                uint8_t* b_s = a_s + S::kKH * S::kASub;
                const uint32_t fb = tc::cluster_addr(&full[s], 0);
                if (leader) tc::mbar_arrive_expect_tx(&full[s], 2 * S::kStage);
#pragma unroll
                for (int h = 0; h < S::kKH; ++h) {
                    const int kc = 2 * (i * S::kKH + h);
                    tc::tma_load_2d_pair(a_s + h * S::kASub, &tmap_a, fb, (i * S::kKH + h) * kI8BK, m0);
                    tc::tma_load_4d_pair(b_s + h * S::kBSub, &tmap_b, fb, 0, 0, kc, nb0 / 16);
                    tc::tma_load_4d_pair(b_s + h * S::kBSub + S::kBHalf, &tmap_b, fb, 0, 0, kc + 1, nb0 / 16);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            // ---- MMA issuer (the leader only)
            constexpr uint32_t idesc = tc::idesc_i8(A_SIGNED, 2 * kI8BM, BN);
            for (int i = 0; i < nkb; ++i) {
                const int s = i % kStages;
                const uint32_t phase = (i / kStages) & 1;
                if (!tc::mbar_wait(&full[s], phase)) { *abort_flag = 1; break; }
                tc::fence_after_sync();
                const uint8_t* a_s = smem + s * S::kStage;
                const uint8_t* b_s = a_s + S::kKH * S::kASub;
#pragma unroll
                for (int h = 0; h < S::kKH; ++h) {
#pragma unroll
                    for (int j = 0; j < kI8BK / 32; ++j) {
                        const uint64_t ad = tc::smem_desc(a_s + h * S::kASub + j * 32, tc::kSwizzle128B, 1024);
                        const uint64_t bd = tc::smem_desc(b_s + h * S::kBSub + (j >> 1) * S::kBHalf + (j & 1) * 32,
                                                          tc::kSwizzle64B, 512);
                        tc::mma_i8_pair(tmem, ad, bd, idesc, (i | h | j) != 0);
                    }
                }
                tc::mma_commit_pair(tc::cluster_addr(&empty[s], 0));
                tc::mma_commit_pair(tc::cluster_addr(&empty[s], 1));
            }
            tc::mma_commit_pair(tc::cluster_addr(done, 0));
            tc::mma_commit_pair(tc::cluster_addr(done, 1));
        }
    } else if (warp == 2 || warp == 3) {
        i8_load_factors<BN>(p, n0, s_scale, s_bias, s_rowsum, s_f, s_zr);
    }
    __syncwarp();
    i8_epilogue<BN>(p, &tmap_y, smem, done, abort_flag, s_scale, s_bias, s_rowsum, s_f, s_zr, tmem, m0, n0);
    tc::fence_before_sync();
    // neither CTA frees its tensor memory or exits while the pair's MMAs, loads or commits may still
    // reach its shared or tensor memory
    tc::cluster_sync();
    if (warp == 2) {
        tc::fence_after_sync();
        tc::tmem_dealloc_pair(tmem, BN);
    }
}

// ============================================================================ host side ======

SBQ_DEFINE_ERROR_POLL(poll_error_dyn)

static int check_x(const void* x, int x_dtype, int64_t ldx, int64_t m, int64_t k) {
    if (!x) return set_error(SBQ_ERR_INVALID_ARGUMENT, "null activation pointer");
    if (m <= 0 || k <= 0) return set_error(SBQ_ERR_INVALID_ARGUMENT, "m and k must be positive");
    if (x_dtype != SBQ_F32 && x_dtype != SBQ_F16 && x_dtype != SBQ_BF16)
        return set_error(SBQ_ERR_UNSUPPORTED, "activation dtype %d (f32, f16, bf16)", x_dtype);
    if (k % 16) return set_error(SBQ_ERR_UNSUPPORTED, "k must be a multiple of 16 (k=%lld)", (long long)k);
    const int es = x_dtype == SBQ_F32 ? 4 : 2;
    if (ldx < k) return set_error(SBQ_ERR_INVALID_ARGUMENT, "row stride smaller than the row");
    if (reinterpret_cast<uintptr_t>(x) % 16 || (ldx * es) % 16)
        return set_error(SBQ_ERR_ALIGNMENT, "activation rows must be 16-byte aligned");
    if (m >= (int64_t(1) << 31) || k >= (int64_t(1) << 30)) return set_error(SBQ_ERR_UNSUPPORTED, "shape too large");
    return SBQ_OK;
}

static size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// Workspace layout: [partials: kMaxPartials float2][xq: m*k bytes][s: m floats][zp: 1 int].
struct DynWorkspace {
    float2* partials;
    uint8_t* xq;
    float* s;
    int32_t* zp;
    size_t bytes;
};

static DynWorkspace dyn_workspace(void* base, int64_t m, int64_t k) {
    DynWorkspace w{};
    uint8_t* p = static_cast<uint8_t*>(base);
    size_t off = 0;
    w.partials = reinterpret_cast<float2*>(p + off);
    off += align256(kMaxPartials * sizeof(float2));
    w.xq = p + off;
    off += align256((size_t)(m * k));
    w.s = reinterpret_cast<float*>(p + off);
    off += align256((size_t)m * sizeof(float));
    w.zp = reinterpret_cast<int32_t*>(p + off);
    off += 256;
    w.bytes = off;
    return w;
}

// Launches `kernel` after the previous work on the stream with programmatic stream serialisation:
// it may start once every CTA of the previous grid has run griddepcontrol.launch_dependents, and
// must run griddepcontrol.wait before it reads anything that grid writes.
template <typename... Params, typename... Args>
static void launch_dependent(void (*kernel)(Params...), dim3 grid, int threads, int smem, cudaStream_t st,
                             Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = dim3((unsigned)threads);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kernel, static_cast<Params>(args)...);
}

// Step 1 is an ordinary launch (x may be the previous kernel's output); step 3 depends on it
// programmatically.
// SMs of the current device, cached per device (atomics: first calls may come from several threads)
static int sm_count_dyn() {
    static std::atomic<int> count[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    int c = count[dev].load(std::memory_order_relaxed);
    if (c == 0) {
        cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev);
        c = c > 0 ? c : 148;
        count[dev].store(c, std::memory_order_relaxed);
    }
    return c;
}

// CTAs of the two per-tensor steps: kQuantVecs vectors per thread, at most kMaxPartials CTAs.
static int minmax_blocks(int64_t m, int64_t k, int vec) {
    const int64_t vecs = m * (k / vec);
    int64_t b = (vecs + kQuantThreads * kQuantVecs - 1) / (kQuantThreads * kQuantVecs);
    if (b > kMaxPartials) b = kMaxPartials;
    return (int)(b < 1 ? 1 : b);
}


template <typename T>
static cudaError_t launch_quant_tensor(const void* x, int64_t ldx, int m, int k, float2* partials, uint8_t* xq,
                                       float* s, int32_t* zp, cudaStream_t st) {
    const int64_t vecs = (int64_t)m * (k / Vec<T>::kN);
    if (vecs <= (int64_t)kFusedThreads * FusedVecs<T>::kN) {
        // small x (up to 64 KiB, e.g. decode rows): the one-launch kernel with a single CTA, which
        // needs no grid barrier - one launch instead of two
        quantize_per_tensor_fused_kernel<T><<<1, kFusedThreads, 0, st>>>(static_cast<const T*>(x), ldx, m, k, partials,
                                                                          xq, s, zp, 0);
        return cudaGetLastError();
    }
    if ((int64_t)m * k * (int64_t)sizeof(T) < kFusedMinBytes) {
        const int nb = minmax_blocks(m, k, Vec<T>::kN);
        minmax_partial_kernel<T><<<nb, kQuantThreads, 0, st>>>(static_cast<const T*>(x), ldx, m, k, partials);
        launch_dependent(quantize_per_tensor_kernel<T>, dim3(nb), kQuantThreads, 0, st, static_cast<const T*>(x), ldx,
                         m, k, static_cast<const float2*>(partials), nb, xq, s, zp);
        return cudaSuccess;
    }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    auto kernel = quantize_per_tensor_fused_kernel<T>;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kFusedThreads, 0);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) per_sm = 1;
    // as many CTAs as hold x in registers (at most the resident limit, and the partials' capacity)
    int64_t nb = ceil_div(vecs, (int64_t)kFusedThreads * FusedVecs<T>::kN);
    const int64_t cap = (int64_t)per_sm * sm_count_dyn();
    if (nb > cap) nb = cap;
    if (nb > kMaxPartials) nb = kMaxPartials;
    if (nb < 1) nb = 1;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)nb);
    cfg.blockDim = dim3(kFusedThreads);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = SBQ_QUANT_COOP ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<const T*>(x), ldx, m, k, partials, xq, s, zp,
                              stream_lane(st, dev));
}

template <typename T>
static void launch_quant_token(const void* x, int64_t ldx, int m, int k, int8_t* xq, float* s, cudaStream_t st) {
    quantize_per_token_kernel<T><<<m, kTokThreads, 0, st>>>(static_cast<const T*>(x), ldx, m, k, xq, s);
}

static int quant_tensor(const void* x, int x_dtype, int64_t ldx, int64_t m, int64_t k, float2* partials, uint8_t* xq,
                        float* s, int32_t* zp, cudaStream_t st) {
    cudaError_t e;
    switch (x_dtype) {
        case SBQ_F32: e = launch_quant_tensor<float>(x, ldx, (int)m, (int)k, partials, xq, s, zp, st); break;
        case SBQ_F16: e = launch_quant_tensor<__half>(x, ldx, (int)m, (int)k, partials, xq, s, zp, st); break;
        default: e = launch_quant_tensor<__nv_bfloat16>(x, ldx, (int)m, (int)k, partials, xq, s, zp, st); break;
    }
    if (e != cudaSuccess) return set_error(SBQ_ERR_CUDA, "quantize activation (per tensor): %s", cudaGetErrorString(e));
    return check_launch("quantize activation (per tensor)");
}

static int quant_token(const void* x, int x_dtype, int64_t ldx, int64_t m, int64_t k, int8_t* xq, float* s,
                       cudaStream_t st) {
    switch (x_dtype) {
        case SBQ_F32: launch_quant_token<float>(x, ldx, (int)m, (int)k, xq, s, st); break;
        case SBQ_F16: launch_quant_token<__half>(x, ldx, (int)m, (int)k, xq, s, st); break;
        default: launch_quant_token<__nv_bfloat16>(x, ldx, (int)m, (int)k, xq, s, st); break;
    }
    return check_launch("quantize activation (per token)");
}

// Tensor maps: xq [m, k] bytes (SW128, 128 x 128 box) and the packed weight viewed as
// {64 bytes, 16 rows, KT tiles, NT tile-rows} (SW64, one 64-wide tile column of BN rows per box).
static int make_gemm_maps(CUtensorMap* ma, CUtensorMap* mb, const void* xq, int64_t m, int64_t k, const void* packed,
                          int64_t n, int bn, int a_rows) {
    const uint64_t kt = (uint64_t)ceil_div(k, kTileCols), nt = (uint64_t)ceil_div(n, kTileRows);
    {
        const uint64_t dims[2] = {(uint64_t)k, (uint64_t)m};
        const uint64_t strides[1] = {(uint64_t)k};
        const uint32_t box[2] = {kI8BK, (uint32_t)a_rows};
        int st = encode_tmap(ma, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, xq, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_128B);
        if (st) return st;
    }
    {
        const uint64_t dims[4] = {64, 16, kt, nt};
        const uint64_t strides[3] = {64, 1024, kt * 1024};
        const uint32_t box[4] = {64, 16, 1, (uint32_t)(bn / 16)};
        int st = encode_tmap(mb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, packed, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_64B);
        if (st) return st;
    }
    return SBQ_OK;
}


// Tile width: 256 weight rows when those tiles still give every SM one (the wider MMA does twice the
// work per issue), else 128 (twice the tiles, as fast in total where 256-wide tiles leave SMs idle).
static int i8_tile_n(int64_t m, int64_t n) {
    const int64_t tiles256 = ceil_div(m, kI8BM) * ceil_div(n, 256);
    return tiles256 * 10 >= (int64_t)sm_count_dyn() * 9 ? 256 : 128;
}

template <int BN>
static int launch_gemm_bn(bool a_signed, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& my,
                          const GemmI8Params& q, bool dependent, cudaStream_t st) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)ceil_div(q.n, BN), (unsigned)ceil_div(q.m, kI8BM), (unsigned)q.parts);
    cfg.blockDim = dim3(kI8Threads);
    cfg.dynamicSmemBytes = (size_t)I8Smem<BN>::kBytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (dependent) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    if (q.parts > 1) {  // split K: the parts of a tile form a cluster along z
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = 1;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = (unsigned)q.parts;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    auto kernel = a_signed ? gemm_w8a8_kernel<BN, true> : gemm_w8a8_kernel<BN, false>;
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, I8Smem<BN>::kBytes);
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, ma, mb, my, q);
    if (e != cudaSuccess) return set_error(SBQ_ERR_CUDA, "gemm_w8a8 launch: %s", cudaGetErrorString(e));
    return check_launch("gemm_w8a8");
}

template <int BN>
static int launch_gemm_pair_bn(bool a_signed, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& my,
                               const GemmI8Params& q, bool dependent, cudaStream_t st) {
    using S = I8PairSmem<BN>;
    GemmI8Params p = q;
    p.num_kb = (int)ceil_div(q.k, (int64_t)kI8BK * S::kKH);  // k past the end reads zeros (TMA fill)
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)(2 * ceil_div(q.m, 2 * kI8BM)), (unsigned)ceil_div(q.n, BN));
    cfg.blockDim = dim3(kI8Threads);
    cfg.dynamicSmemBytes = (size_t)S::kBytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = dependent ? 1 : 0;
    auto kernel = a_signed ? gemm_w8a8_pair_kernel<BN, true> : gemm_w8a8_pair_kernel<BN, false>;
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kBytes);
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, ma, mb, my, p);
    if (e != cudaSuccess) return set_error(SBQ_ERR_CUDA, "gemm_w8a8 (CTA pairs) launch: %s", cudaGetErrorString(e));
    return check_launch("gemm_w8a8 (CTA pairs)");
}

#ifndef SBQ_I8_PAIR
#define SBQ_I8_PAIR 1
#endif

// Tile of the CTA-pair kernel: BN = 256 weight rows when those pairs still give every SM a CTA, else 128.
static int i8_pair_tile_n(int64_t m, int64_t n) {
    const int64_t ctas256 = 2 * ceil_div(m, 2 * kI8BM) * ceil_div(n, 256);
    return ctas256 * 10 >= (int64_t)sm_count_dyn() * 9 ? 256 : 128;
}

// dependent: launched as a programmatic dependent of the activation quantisation (sbq_linear_dyn),
// which lets the pipeline set-up and the first weight tiles overlap that kernel.  Direct calls of
// sbq_gemm_w8a8 launch in plain stream order: there the scale, bias and row sums read in the
// prologue could be the previous kernel's output.
static int launch_gemm_i8(const void* xq, bool a_signed, const void* packed, const GemmI8Params& p, bool dependent,
                          cudaStream_t st) {
    const bool pair = SBQ_I8_PAIR && p.m > kI8BM;  // more than one 128-row tile of xq: CTA pairs
    const int bn = pair ? i8_pair_tile_n(p.m, p.n) : i8_tile_n(p.m, p.n);
    GemmI8Params q = p;
    q.parts = 1;
    if (!pair && p.m <= 32) {
        // decode sizes (up to 32 rows of xq): the weight stream of ceil(n / bn) CTAs alone is too
        // narrow, so K is split over a cluster - the largest power of two up to 8 that keeps one CTA
        // per SM and at least 2 k-blocks per part (int32 partial sums: the result is unchanged).
        // Measured at n = k = 4096: m = 1 17.5 -> 13.6 us, m = 16 18.2 -> 15.0 us per quantise +
        // GEMM call; at m = 64 no change and at m = 128 slower (24.9 us: the exchange of 128 rows)
        const int64_t tiles = ceil_div(p.n, bn);
        while (q.parts < 8 && tiles * (2 * q.parts) <= (int64_t)sm_count_dyn() && p.num_kb / (2 * q.parts) >= 2)
            q.parts *= 2;
    }
    CUtensorMap ma, mb, my;
    // the single-CTA kernel loads only the xq rows that exist (in 16-row steps), the pair kernel 128
    q.a_rows = pair ? kI8BM : (int)(p.m >= kI8BM ? kI8BM : ceil_div(p.m, 16) * 16);
    int rc = make_gemm_maps(&ma, &mb, xq, p.m, p.k, packed, p.n, pair ? bn / 2 : bn, q.a_rows);  // a pair CTA loads bn/2 rows
    if (rc) return rc;
    std::memset(&my, 0, sizeof(my));
    q.tma_y = !p.acc_out && reinterpret_cast<uintptr_t>(p.y) % 16 == 0 && p.ldy % 4 == 0;
    q.vec_y = reinterpret_cast<uintptr_t>(p.y) % 16 == 0 && p.ldy % 4 == 0 && p.n % 4 == 0 &&
              (!p.acc_out || reinterpret_cast<uintptr_t>(p.acc_out) % 16 == 0);
    if (q.tma_y) {
        // y [m, n] fp32 as 32 x 32 boxes, 128-byte swizzle (one 128-byte line per box row)
        const uint64_t dims[2] = {(uint64_t)p.n, (uint64_t)p.m};
        const uint64_t strides[1] = {(uint64_t)p.ldy * 4};
        const uint32_t box[2] = {32, 32};
        rc = encode_tmap(&my, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, p.y, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    if (pair)
        return bn == 256 ? launch_gemm_pair_bn<256>(a_signed, ma, mb, my, q, dependent, st)
                         : launch_gemm_pair_bn<128>(a_signed, ma, mb, my, q, dependent, st);
    return bn == 256 ? launch_gemm_bn<256>(a_signed, ma, mb, my, q, dependent, st)
                     : launch_gemm_bn<128>(a_signed, ma, mb, my, q, dependent, st);
}

}  // namespace sbq

using namespace sbq;

extern "C" size_t sbq_dyn_workspace_bytes(int64_t m, int64_t k, int mode) {
    (void)mode;
    if (m <= 0 || k <= 0) return 0;
    return dyn_workspace(nullptr, m, k).bytes;
}

extern "C" int sbq_quant_act_per_tensor(const void* x, int x_dtype, int64_t ldx, int64_t m, int64_t k, uint8_t* xq,
                                        float* s_x, int32_t* zp, void* workspace, size_t workspace_bytes,
                                        void* stream) {
    int st = check_x(x, x_dtype, ldx, m, k);
    if (st) return st;
    if (!xq || !s_x || !zp || !workspace) return set_error(SBQ_ERR_INVALID_ARGUMENT, "null output or workspace pointer");
    if (workspace_bytes < kMaxPartials * sizeof(float2))
        return set_error(SBQ_ERR_WORKSPACE, "workspace needs %zu bytes", (size_t)(kMaxPartials * sizeof(float2)));
    if (reinterpret_cast<uintptr_t>(xq) % 16) return set_error(SBQ_ERR_ALIGNMENT, "xq must be 16-byte aligned");
    return quant_tensor(x, x_dtype, ldx, m, k, static_cast<float2*>(workspace), xq, s_x, zp,
                        static_cast<cudaStream_t>(stream));
}

extern "C" int sbq_quant_act_per_token(const void* x, int x_dtype, int64_t ldx, int64_t m, int64_t k, int8_t* xq,
                                       float* s_tok, void* stream) {
    int st = check_x(x, x_dtype, ldx, m, k);
    if (st) return st;
    if (!xq || !s_tok) return set_error(SBQ_ERR_INVALID_ARGUMENT, "null output pointer");
    if (reinterpret_cast<uintptr_t>(xq) % 16) return set_error(SBQ_ERR_ALIGNMENT, "xq must be 16-byte aligned");
    return quant_token(x, x_dtype, ldx, m, k, xq, s_tok, static_cast<cudaStream_t>(stream));
}

static int check_gemm(const void* xq, int mode, const void* packed, const int32_t* rowsum, const float* s_x,
                      const int32_t* zp, const float* scale, int64_t m, int64_t n, int64_t k, const float* y,
                      int64_t ldy) {
    if (!xq || !packed || !s_x || !scale || !y) return set_error(SBQ_ERR_INVALID_ARGUMENT, "null pointer");
    if (mode != SBQ_ACT_PER_TENSOR && mode != SBQ_ACT_PER_TOKEN)
        return set_error(SBQ_ERR_INVALID_ARGUMENT, "unknown activation mode %d", mode);
    if (mode == SBQ_ACT_PER_TENSOR && (!rowsum || !zp))
        return set_error(SBQ_ERR_INVALID_ARGUMENT, "per-tensor mode needs rowsum and zp");
    if (m <= 0 || n <= 0 || k <= 0) return set_error(SBQ_ERR_INVALID_ARGUMENT, "m, n, k must be positive");
    if (k % 16) return set_error(SBQ_ERR_UNSUPPORTED, "k must be a multiple of 16");
    if (ldy < n) return set_error(SBQ_ERR_INVALID_ARGUMENT, "ldy < n");
    if (reinterpret_cast<uintptr_t>(xq) % 16 || reinterpret_cast<uintptr_t>(packed) % 256)
        return set_error(SBQ_ERR_ALIGNMENT, "xq must be 16-byte and packed 256-byte aligned");
    if (m >= (int64_t(1) << 31) || n >= (int64_t(1) << 31) || k >= (int64_t(1) << 30))
        return set_error(SBQ_ERR_UNSUPPORTED, "shape too large");
    return SBQ_OK;
}

static int gemm_w8a8(const void* xq, int mode, const void* packed, const int32_t* rowsum, const float* s_x,
                     const int32_t* zp, const float* scale, const float* bias, int64_t m, int64_t n, int64_t k, float* y,
                     int64_t ldy, int32_t* acc_out, bool dependent, void* stream) {
    int st = check_gemm(xq, mode, packed, rowsum, s_x, zp, scale, m, n, k, y, ldy);
    if (st) return st;
    GemmI8Params p{};
    p.m = (int)m;
    p.n = (int)n;
    p.k = (int)k;
    p.num_kb = (int)ceil_div(k, kI8BK);
    const bool per_tensor = mode == SBQ_ACT_PER_TENSOR;
    p.rowsum = per_tensor ? rowsum : nullptr;
    p.s_x = s_x;
    p.s_stride = per_tensor ? 0 : 1;
    p.zp = per_tensor ? zp : nullptr;
    p.scale = scale;
    p.bias = bias;
    p.y = y;
    p.ldy = ldy;
    p.acc_out = acc_out;
    return launch_gemm_i8(xq, !per_tensor, packed, p, dependent, static_cast<cudaStream_t>(stream));
}

extern "C" int sbq_gemm_w8a8(const void* xq, int mode, const void* packed, const int32_t* rowsum, const float* s_x,
                             const int32_t* zp, const float* scale, const float* bias, int64_t m, int64_t n, int64_t k,
                             float* y, int64_t ldy, int32_t* acc_out, void* stream) {
    return gemm_w8a8(xq, mode, packed, rowsum, s_x, zp, scale, bias, m, n, k, y, ldy, acc_out, false, stream);
}

extern "C" int sbq_linear_dyn(const void* x, int x_dtype, int64_t ldx, int mode, const void* packed,
                              const int32_t* rowsum, const float* scale, const float* bias, int64_t m, int64_t n,
                              int64_t k, float* y, int64_t ldy, void* workspace, size_t workspace_bytes,
                              void* stream) {
    int st = check_x(x, x_dtype, ldx, m, k);
    if (st) return st;
    if (!workspace) return set_error(SBQ_ERR_INVALID_ARGUMENT, "null workspace");
    if (reinterpret_cast<uintptr_t>(workspace) % 256) return set_error(SBQ_ERR_ALIGNMENT, "workspace must be 256-byte aligned");
    DynWorkspace w = dyn_workspace(workspace, m, k);
    if (workspace_bytes < w.bytes) return set_error(SBQ_ERR_WORKSPACE, "workspace needs %zu bytes", w.bytes);
    // every GEMM argument is checked before the quantisation is launched: a call that fails launches
    // nothing (and leaves the workspace untouched)
    st = check_gemm(w.xq, mode, packed, rowsum, w.s, w.zp, scale, m, n, k, y, ldy);
    if (st) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (mode == SBQ_ACT_PER_TENSOR) {
        st = quant_tensor(x, x_dtype, ldx, m, k, w.partials, w.xq, w.s, w.zp, s);
    } else if (mode == SBQ_ACT_PER_TOKEN) {
        st = quant_token(x, x_dtype, ldx, m, k, reinterpret_cast<int8_t*>(w.xq), w.s, s);
    } else {
        return set_error(SBQ_ERR_INVALID_ARGUMENT, "unknown activation mode %d", mode);
    }
    if (st) return st;
    return gemm_w8a8(w.xq, mode, packed, rowsum, w.s, w.zp, scale, bias, m, n, k, y, ldy, nullptr, true, stream);
}

// ============================================================================ no-allocation variant

// sbq_linear_dyn without a caller-provided workspace.  Its scratch (min/max partials, quantised
// activations, per-row scales, zero point) lives in this fixed device array, which every GPU that
// loads the library holds until the process exits.  The array is only ever written before it is
// read within one call, so nothing in it has to start at zero; calls that overlap on the GPU share
// it and race.
#include <mutex>

namespace sbq {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;  // 4 MiB
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kNoAllocMaxDevices = 64;

// Host-side address of the array on the current device, looked up once per device.
static int noalloc_scratch(void** out) {
    static std::mutex mu;
    static void* addr[kNoAllocMaxDevices] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return check_launch("cudaGetDevice");
    if (dev < 0 || dev >= kNoAllocMaxDevices) return set_error(SBQ_ERR_DEVICE, "device ordinal %d out of range", dev);
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess)
            return set_error(SBQ_ERR_CUDA, "cudaGetSymbolAddress of the scratch array failed: %s", cudaGetErrorString(e));
        addr[dev] = p;
    }
    *out = addr[dev];
    return SBQ_OK;
}

}  // namespace sbq

extern "C" int sbq_linear_dyn_noalloc(const void* x, int x_dtype, int64_t ldx, int mode, const void* packed,
                                      const int32_t* rowsum, const float* scale, const float* bias, int64_t m,
                                      int64_t n, int64_t k, float* y, int64_t ldy, void* stream) {
    int st = check_x(x, x_dtype, ldx, m, k);
    if (st) return st;
    const size_t need = dyn_workspace(nullptr, m, k).bytes;
    if (need > kNoAllocScratchBytes)
        return set_error(SBQ_ERR_WORKSPACE,
                         "m=%lld x k=%lld needs %zu bytes of scratch, above the fixed %zu-byte array of "
                         "sbq_linear_dyn_noalloc; use sbq_linear_dyn with a workspace",
                         (long long)m, (long long)k, need, kNoAllocScratchBytes);
    void* scratch = nullptr;
    st = noalloc_scratch(&scratch);
    if (st) return st;
    return sbq_linear_dyn(x, x_dtype, ldx, mode, packed, rowsum, scale, bias, m, n, k, y, ldy, scratch,
                          kNoAllocScratchBytes, stream);
}
