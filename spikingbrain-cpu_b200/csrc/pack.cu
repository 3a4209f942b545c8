// One-time weight preparation: per-output-channel int8 quantisation on the device and the
// packed (16 x 64 tile) layout.
//
// Reference: spikingbrain_cpu/quant.py:25-29 (quantize_per_channel) and the qweight / scale
// buffers of Int8Linear (quant.py:35-37).  The arithmetic is the reference's, bit for bit:
//   scale[r] = max(max_c |w[r, c]|, 1e-8f) / 127.0f          (fp32, IEEE division)
//   q[r, c]  = clamp(rint(w[r, c] / scale[r]), -127, 127)    (IEEE division, ties to even)
#include "common.cuh"

namespace sbq {

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

__device__ __forceinline__ int64_t packed_offset(int64_t r, int64_t c, int64_t kt_total) {
    return ((r >> 4) * kt_total + (c >> 6)) * kTileBytes + (r & 15) * kTileCols + (c & 63);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ int warp_sum(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// One warp per row: amax, scale, then quantise into the packed tiles (+ row sum).
template <typename T>
__global__ void __launch_bounds__(256) quantize_pack_kernel(const T* __restrict__ w, int64_t n, int64_t k,
                                                            int64_t ldw, int8_t* __restrict__ packed,
                                                            float* __restrict__ scale,
                                                            int32_t* __restrict__ rowsum) {
    const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= n) return;
    const T* row = w + r * ldw;
    const int64_t kt_total = ceil_div(k, kTileCols);
    float amax = 0.0f;
    for (int64_t c = lane; c < k; c += 32) amax = fmaxf(amax, fabsf(to_f32(row[c])));
    amax = warp_max(amax);
    const float s = __fdiv_rn(fmaxf(amax, 1e-8f), 127.0f);
    int sum = 0;
    for (int64_t c = lane; c < k; c += 32) {
        float t = rintf(__fdiv_rn(to_f32(row[c]), s));
        t = fminf(fmaxf(t, -127.0f), 127.0f);
        const int qv = (int)t;
        sum += qv;
        packed[packed_offset(r, c, kt_total)] = (int8_t)qv;
    }
    sum = warp_sum(sum);
    if (lane == 0) {
        scale[r] = s;
        if (rowsum) rowsum[r] = sum;
    }
}

__global__ void __launch_bounds__(256) pack_int8_kernel(const int8_t* __restrict__ q, int64_t n, int64_t k,
                                                        int64_t ldq, int8_t* __restrict__ packed,
                                                        int32_t* __restrict__ rowsum) {
    const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= n) return;
    const int64_t kt_total = ceil_div(k, kTileCols);
    int sum = 0;
    for (int64_t c = lane; c < k; c += 32) {
        const int8_t v = q[r * ldq + c];
        sum += v;
        packed[packed_offset(r, c, kt_total)] = v;
    }
    sum = warp_sum(sum);
    if (lane == 0 && rowsum) rowsum[r] = sum;
}

__global__ void __launch_bounds__(256) unpack_int8_kernel(const int8_t* __restrict__ packed, int64_t n,
                                                          int64_t k, int8_t* __restrict__ q, int64_t ldq) {
    const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= n) return;
    const int64_t kt_total = ceil_div(k, kTileCols);
    for (int64_t c = lane; c < k; c += 32) q[r * ldq + c] = packed[packed_offset(r, c, kt_total)];
}

static int check_pack_args(const void* a, const void* packed, int64_t n, int64_t k, int64_t ld) {
    if (!a || !packed) return set_error(SBQ_ERR_INVALID_ARGUMENT, "null pointer");
    if (n <= 0 || k <= 0) return set_error(SBQ_ERR_INVALID_ARGUMENT, "n and k must be positive (n=%lld k=%lld)",
                                           (long long)n, (long long)k);
    if (ld < k) return set_error(SBQ_ERR_INVALID_ARGUMENT, "row stride %lld < k %lld", (long long)ld, (long long)k);
    if (reinterpret_cast<uintptr_t>(packed) % 256)
        return set_error(SBQ_ERR_ALIGNMENT, "packed weight must be 256-byte aligned");
    if (n >= (int64_t(1) << 31) || k >= (int64_t(1) << 30))
        return set_error(SBQ_ERR_UNSUPPORTED, "weight too large");
    return SBQ_OK;
}

}  // namespace sbq

using namespace sbq;

extern "C" size_t sbq_packed_bytes(int64_t n, int64_t k) {
    if (n <= 0 || k <= 0) return 0;
    return (size_t)(ceil_div(n, kTileRows) * ceil_div(k, kTileCols) * kTileBytes);
}

extern "C" int sbq_quantize_pack(const void* w, int w_dtype, int64_t n, int64_t k, int64_t ldw, void* packed,
                                 float* scale, int32_t* rowsum, void* stream) {
    int st = check_pack_args(w, packed, n, k, ldw);
    if (st) return st;
    if (!scale) return set_error(SBQ_ERR_INVALID_ARGUMENT, "null scale pointer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (cudaMemsetAsync(packed, 0, sbq_packed_bytes(n, k), s) != cudaSuccess) return check_launch("memset packed");
    const dim3 block(256), grid((unsigned)ceil_div(n, 8));
    int8_t* out = static_cast<int8_t*>(packed);
    switch (w_dtype) {
        case SBQ_F32:
            quantize_pack_kernel<float><<<grid, block, 0, s>>>(static_cast<const float*>(w), n, k, ldw, out, scale, rowsum);
            break;
        case SBQ_F16:
            quantize_pack_kernel<__half><<<grid, block, 0, s>>>(static_cast<const __half*>(w), n, k, ldw, out, scale, rowsum);
            break;
        case SBQ_BF16:
            quantize_pack_kernel<__nv_bfloat16>
                <<<grid, block, 0, s>>>(static_cast<const __nv_bfloat16*>(w), n, k, ldw, out, scale, rowsum);
            break;
        default:
            return set_error(SBQ_ERR_UNSUPPORTED, "weight dtype %d not supported (f32, f16, bf16)", w_dtype);
    }
    return check_launch("quantize_pack");
}

extern "C" int sbq_pack_int8(const int8_t* q, int64_t n, int64_t k, int64_t ldq, void* packed, int32_t* rowsum,
                             void* stream) {
    int st = check_pack_args(q, packed, n, k, ldq);
    if (st) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (cudaMemsetAsync(packed, 0, sbq_packed_bytes(n, k), s) != cudaSuccess) return check_launch("memset packed");
    pack_int8_kernel<<<(unsigned)ceil_div(n, 8), 256, 0, s>>>(q, n, k, ldq, static_cast<int8_t*>(packed), rowsum);
    return check_launch("pack_int8");
}

extern "C" int sbq_unpack_int8(const void* packed, int64_t n, int64_t k, int8_t* q, int64_t ldq, void* stream) {
    int st = check_pack_args(q, packed, n, k, ldq);
    if (st) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    unpack_int8_kernel<<<(unsigned)ceil_div(n, 8), 256, 0, s>>>(static_cast<const int8_t*>(packed), n, k, q, ldq);
    return check_launch("unpack_int8");
}
