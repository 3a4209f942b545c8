// Prefill GEMM of the int8 weight-only format: Y[m, n] = (X[m, k] . Wq[n, k]^T) * scale[n].
//
// Reference: Int8Linear.forward (spikingbrain_cpu/quant.py:41-53) at prefill shapes (512-token
// chunks, model.py:439).  The reference dequantises 128-row weight blocks to fp32 and runs an fp32
// sgemm, then scales.  Here:
//   * warp 0 (one thread) streams 128 x 64 fp16 activation tiles (TMA, 128-byte swizzle) and the
//     matching 256 x 64 int8 weight tiles (TMA over the packed layout, no swizzle) into a 4-stage ring;
//   * warps 4-7 convert each int8 tile to fp16 (exact) into a 2-deep ring of K-major,
//     128-byte-swizzled operand buffers, then hand them to the MMA thread;
//   * warp 1 (one thread) issues tcgen05.mma.cta_group::1.kind::f16 (128 x 256 x 16, fp32
//     accumulators in tensor memory) and commits each stage back to its producers;
//   * warps 4-7 finally read the accumulators (tcgen05.ld), apply the fp32 per-row scale (and bias)
//     and store fp16 or fp32 output.
// The scale stays in the fp32 epilogue, as in the reference: int8 values are exact in fp16.
#include "tc.cuh"

namespace sbq {

struct GemmW16Params {
    int m, n, k, num_kb;
    const float* scale;
    const float* bias;
    void* y;
    int64_t ldy;
    int out_f16;
};

constexpr int kWBM = 128;      // activation rows per CTA (MMA M)
constexpr int kWBN = 256;      // output channels per CTA (MMA N)
constexpr int kWBK = 64;       // k per stage (one 128-byte fp16 row, one packed tile column)
constexpr int kWRaw = 4;       // raw (TMA) stages
constexpr int kWDq = 2;        // dequantised weight buffers
constexpr int kWThreads = 256; // 8 warps

struct W16Smem {
    static constexpr int kX = kWBM * kWBK * 2;   // 16 KiB fp16 activation tile
    static constexpr int kW8 = kWBN * kWBK;      // 16 KiB int8 weight tile
    static constexpr int kRaw = kX + kW8;
    static constexpr int kW16 = kWBN * kWBK * 2; // 32 KiB fp16 weight operand
    static constexpr int kBarOff = kWRaw * kRaw + kWDq * kW16;
    static constexpr int kBytes = kBarOff + 256 + kWBN * 8 + 1024;
};

template <bool OUT_F16>
__global__ void __launch_bounds__(kWThreads, 1) gemm_w8a16_kernel(const __grid_constant__ CUtensorMap tmap_x,
                                                                  const __grid_constant__ CUtensorMap tmap_w,
                                                                  const GemmW16Params p) {
    using S = W16Smem;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* raw_base = smem;
    uint8_t* w16_base = smem + kWRaw * S::kRaw;
    uint64_t* raw_full = reinterpret_cast<uint64_t*>(smem + S::kBarOff);
    uint64_t* raw_empty = raw_full + kWRaw;
    uint64_t* dq_full = raw_empty + kWRaw;
    uint64_t* dq_empty = dq_full + kWDq;
    uint64_t* done = dq_empty + kWDq;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    float* s_scale = reinterpret_cast<float*>(smem + S::kBarOff + 256);
    float* s_bias = s_scale + kWBN;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.y * kWBM, n0 = blockIdx.x * kWBN;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kWRaw; ++s) {
            tc::mbar_init(&raw_full[s], 1);
            tc::mbar_init(&raw_empty[s], 4 + 1);  // 4 dequant warps (weight read) + MMA commit (x read)
        }
        for (int d = 0; d < kWDq; ++d) {
            tc::mbar_init(&dq_full[d], 4);
            tc::mbar_init(&dq_empty[d], 1);
        }
        tc::mbar_init(done, 1);
        tc::fence_mbar_init();
        tc::prefetch_tmap(&tmap_x);
        tc::prefetch_tmap(&tmap_w);
    }
    if (warp == 2) {
        tc::tmem_alloc(tmem_slot, kWBN);
        tc::tmem_relinquish();
    }
    for (int i = threadIdx.x; i < kWBN; i += blockDim.x) {
        const int n = n0 + i;
        s_scale[i] = n < p.n ? p.scale[n] : 0.0f;
        s_bias[i] = (p.bias && n < p.n) ? p.bias[n] : 0.0f;
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    bool failed = false;

    if (warp == 0) {
        if (lane == 0) {
            for (int kb = 0; kb < p.num_kb; ++kb) {
                const int s = kb % kWRaw;
                const uint32_t ph = (kb / kWRaw) & 1;
                if (!tc::mbar_wait(&raw_empty[s], ph ^ 1)) break;
                uint8_t* xs = raw_base + s * S::kRaw;
                tc::mbar_arrive_expect_tx(&raw_full[s], S::kRaw);
                tc::tma_load_2d(xs, &tmap_x, &raw_full[s], kb * kWBK, m0);
                tc::tma_load_4d(xs + S::kX, &tmap_w, &raw_full[s], 0, 0, kb, n0 / 16);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_f16(kWBM, kWBN);
            for (int kb = 0; kb < p.num_kb; ++kb) {
                const int s = kb % kWRaw, d = kb % kWDq;
                const uint32_t ph = (kb / kWRaw) & 1, phd = (kb / kWDq) & 1;
                if (!tc::mbar_wait(&raw_full[s], ph)) break;
                if (!tc::mbar_wait(&dq_full[d], phd)) break;
                tc::fence_after_sync();
                const uint8_t* xs = raw_base + s * S::kRaw;
                const uint8_t* ws = w16_base + d * S::kW16;
#pragma unroll
                for (int j = 0; j < kWBK / 16; ++j) {
                    const uint64_t ad = tc::smem_desc(xs + j * 32, tc::kSwizzle128B, 1024);
                    const uint64_t bd = tc::smem_desc(ws + j * 32, tc::kSwizzle128B, 1024);
                    tc::mma_f16(tmem, ad, bd, idesc, (kb | j) != 0);
                }
                tc::mma_commit(&raw_empty[s]);
                tc::mma_commit(&dq_empty[d]);
            }
            tc::mma_commit(done);
        }
    } else if (warp >= 4) {
        // ---- dequantise: int8 tile [256 rows][64 B] -> fp16 [256 rows][128 B], K-major, 128-byte swizzle
        const int t = threadIdx.x - 128;
        for (int kb = 0; kb < p.num_kb && !failed; ++kb) {
            const int s = kb % kWRaw, d = kb % kWDq;
            const uint32_t ph = (kb / kWRaw) & 1, phd = (kb / kWDq) & 1;
            // warp-uniform waits, so a lane never leaves the loop alone (__syncwarp below)
            if (!__all_sync(0xffffffffu, tc::mbar_wait(&raw_full[s], ph))) { failed = true; break; }
            if (!__all_sync(0xffffffffu, tc::mbar_wait(&dq_empty[d], phd ^ 1))) { failed = true; break; }
            const uint8_t* w8 = raw_base + s * S::kRaw + S::kX;
            uint8_t* w16 = w16_base + d * S::kW16;
#pragma unroll 4
            for (int i = 0; i < (kWBN * kWBK / 16) / 128; ++i) {
                const int q = t + 128 * i;          // 16-byte chunk of the int8 tile
                const int row = q >> 2, c = q & 3;  // row of the tile, 16-wide k group
                const uint4 v = *reinterpret_cast<const uint4*>(w8 + q * 16);
                uint32_t h[8];
                i8x4_to_half2x2(v.x, h[0], h[1]);
                i8x4_to_half2x2(v.y, h[2], h[3]);
                i8x4_to_half2x2(v.z, h[4], h[5]);
                i8x4_to_half2x2(v.w, h[6], h[7]);
                uint8_t* rowp = w16 + (row >> 3) * 1024 + (row & 7) * 128;
                const int sw = row & 7;
                *reinterpret_cast<uint4*>(rowp + (((2 * c) ^ sw) << 4)) = make_uint4(h[0], h[1], h[2], h[3]);
                *reinterpret_cast<uint4*>(rowp + (((2 * c + 1) ^ sw) << 4)) = make_uint4(h[4], h[5], h[6], h[7]);
            }
            tc::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                tc::mbar_arrive(&dq_full[d]);
                tc::mbar_arrive(&raw_empty[s]);
            }
        }
        // ---- epilogue: accumulators (lanes 32 (warp - 4) ..) -> scale -> global
        // warp-uniform decision: tcgen05.ld below is a warp-collective instruction
        const bool ok = __all_sync(0xffffffffu, !failed && tc::mbar_wait(done, 0));
        tc::fence_after_sync();
        if (ok) {
            const int wq = warp - 4;
            const int row = m0 + wq * 32 + lane;
#pragma unroll 1
            for (int c = 0; c < kWBN / 32; ++c) {
                uint32_t r[32];
                tc::tmem_ld_32x32b_x32(tmem + ((uint32_t)(wq * 32) << 16) + c * 32, r);
                tc::tmem_wait_ld();
                if (row >= p.m) continue;
                const int nb = n0 + c * 32;
                float v[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int i = c * 32 + j;
                    v[j] = __fmul_rn(__uint_as_float(r[j]), s_scale[i]);
                    if (p.bias) v[j] = __fadd_rn(v[j], s_bias[i]);
                }
                if (OUT_F16) {
                    __half* yr = static_cast<__half*>(p.y) + (int64_t)row * p.ldy;
                    if (nb + 32 <= p.n && (p.ldy % 8) == 0) {
#pragma unroll
                        for (int j = 0; j < 32; j += 8) {
                            uint4 o;
                            __half2 a = __floats2half2_rn(v[j], v[j + 1]), b = __floats2half2_rn(v[j + 2], v[j + 3]);
                            __half2 cc = __floats2half2_rn(v[j + 4], v[j + 5]), dd = __floats2half2_rn(v[j + 6], v[j + 7]);
                            o.x = *reinterpret_cast<uint32_t*>(&a);
                            o.y = *reinterpret_cast<uint32_t*>(&b);
                            o.z = *reinterpret_cast<uint32_t*>(&cc);
                            o.w = *reinterpret_cast<uint32_t*>(&dd);
                            *reinterpret_cast<uint4*>(yr + nb + j) = o;
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (nb + j < p.n) yr[nb + j] = __float2half_rn(v[j]);
                    }
                } else {
                    float* yr = static_cast<float*>(p.y) + (int64_t)row * p.ldy;
                    if (nb + 32 <= p.n && (p.ldy % 4) == 0) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4)
                            *reinterpret_cast<float4*>(yr + nb + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (nb + j < p.n) yr[nb + j] = v[j];
                    }
                }
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 2) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, kWBN);
    }
}

SBQ_DEFINE_ERROR_POLL(poll_error_w8a16)

int check_linear_args(const void* x, int x_dtype, int64_t ldx, const void* packed, const float* scale, int64_t m,
                      int64_t n, int64_t k, const void* y, int y_dtype, int64_t ldy);

}  // namespace sbq

using namespace sbq;

extern "C" int sbq_gemm_w8a16(const void* x, int x_dtype, int64_t ldx, const void* packed, const float* scale,
                              const float* bias, int64_t m, int64_t n, int64_t k, void* y, int y_dtype, int64_t ldy,
                              void* stream) {
    int st = check_linear_args(x, x_dtype, ldx, packed, scale, m, n, k, y, y_dtype, ldy);
    if (st) return st;
    if (x_dtype != SBQ_F16) return set_error(SBQ_ERR_UNSUPPORTED, "sbq_gemm_w8a16 takes fp16 activations");
    CUtensorMap mx, mw;
    {
        const uint64_t dims[2] = {(uint64_t)k, (uint64_t)m};
        const uint64_t strides[1] = {(uint64_t)ldx * 2};
        const uint32_t box[2] = {kWBK, kWBM};
        st = encode_tmap(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, x, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (st) return st;
    }
    {
        const uint64_t kt = (uint64_t)ceil_div(k, kTileCols), nt = (uint64_t)ceil_div(n, kTileRows);
        const uint64_t dims[4] = {64, 16, kt, nt};
        const uint64_t strides[3] = {64, 1024, kt * 1024};
        const uint32_t box[4] = {64, 16, 1, kWBN / 16};
        st = encode_tmap(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, packed, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (st) return st;
    }
    GemmW16Params p{};
    p.m = (int)m;
    p.n = (int)n;
    p.k = (int)k;
    p.num_kb = (int)ceil_div(k, kWBK);
    p.scale = scale;
    p.bias = bias;
    p.y = y;
    p.ldy = ldy;
    p.out_f16 = y_dtype == SBQ_F16;
    const dim3 grid((unsigned)ceil_div(n, kWBN), (unsigned)ceil_div(m, kWBM));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int smem = W16Smem::kBytes;
    if (p.out_f16) {
        cudaFuncSetAttribute(gemm_w8a16_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        gemm_w8a16_kernel<true><<<grid, kWThreads, smem, s>>>(mx, mw, p);
    } else {
        cudaFuncSetAttribute(gemm_w8a16_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        gemm_w8a16_kernel<false><<<grid, kWThreads, smem, s>>>(mx, mw, p);
    }
    return check_launch("gemm_w8a16");
}
