// Shared device/host helpers for the sm_100a int8 quantised-linear kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "sbq.h"

namespace sbq {

// ---------------------------------------------------------------------------------------------
// Packed weight layout ("tile-swizzled" int8).
//
// The [N, K] int8 weight is cut into 16-row x 64-column tiles of 1 KiB.  Tile (nt, kt) starts at
// byte (nt * KT + kt) * 1024 and holds its 16 rows row-major (row r, column c at r * 64 + c).
// N is padded to a multiple of 16 and K to a multiple of 64 with zeros.
//
// Why this shape: a warp streaming one tile issues two fully contiguous 512-byte loads (lane l
// reads bytes 16 l .. 16 l + 15 of each half).  Lane l then holds 16 consecutive k of row
// (l / 4) and of row (l / 4) + 8, which is exactly the row pairing of an m16n8k16 A fragment once
// the k order inside each 64-wide span is permuted (the activations use the same permutation, so
// the dot product is unchanged).  The same tiles feed the tensor-memory GEMMs through TMA.
// ---------------------------------------------------------------------------------------------
constexpr int kTileRows = 16;
constexpr int kTileCols = 64;
constexpr int kTileBytes = kTileRows * kTileCols;

// Rows of x above which the int8 weight-only format runs the tensor-memory GEMM (sbq_linear_w8,
// sbq_mlp_gateup_w8) instead of the decode GEMV, which streams the weight once per 16 rows.
#ifndef SBQ_GEMM_MIN_ROWS
#define SBQ_GEMM_MIN_ROWS 16
#endif
constexpr int64_t kGemmMinRows = SBQ_GEMM_MIN_ROWS;

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Stream lanes (host): each (device, stream) pair is given one of kStreamLanes lanes, round robin on
// first use, so that launches on up to kStreamLanes distinct streams of a device use disjoint
// library-internal counters and scratch.  A CUDA graph keeps the lane of the stream it was captured on.
constexpr int kStreamLanes = 8;
int stream_lane(cudaStream_t s, int dev);

// ---------------------------------------------------------------------------------------------
// Loads.
// ---------------------------------------------------------------------------------------------

// Weights are read exactly once per launch: no L1 allocation, 256-byte L2 prefetch.
__device__ __forceinline__ uint4 ld_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// Activations are small and re-read by many warps: read-only path, cached.
__device__ __forceinline__ uint4 ld_act(const void* p) {
    return __ldg(reinterpret_cast<const uint4*>(p));
}

// ---------------------------------------------------------------------------------------------
// int8 -> 16-bit float conversion in registers (exact: |q| <= 127).
// ---------------------------------------------------------------------------------------------

// Four int8 in one word -> two half2: lo = (q0, q1), hi = (q2, q3).
// Offset binary: u = q ^ 0x80 = q + 128; half(0x6400 | u) = 1024 + u; subtract 1152.
__device__ __forceinline__ void i8x4_to_half2x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
    const uint32_t u = w ^ 0x80808080u;
    lo = __byte_perm(u, 0x64646464u, 0x5140);
    hi = __byte_perm(u, 0x64646464u, 0x7362);
    const uint32_t bias = 0x64806480u;  // half2(1152, 1152)
    asm("sub.f16x2 %0, %0, %1;" : "+r"(lo) : "r"(bias));
    asm("sub.f16x2 %0, %0, %1;" : "+r"(hi) : "r"(bias));
}

// Four int8 -> two bf16x2.  float(0x4B000000 | u) = 2^23 + u; subtract 2^23 + 128; the result
// (an integer of magnitude <= 128) is exact in bf16, so its upper half is the bf16 value.
__device__ __forceinline__ void i8x4_to_bf162x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
    const uint32_t u = w ^ 0x80808080u;
    const float k = 8388736.0f;  // 2^23 + 128
    float f0 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7650)) - k;
    float f1 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7651)) - k;
    float f2 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7652)) - k;
    float f3 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7653)) - k;
    lo = __byte_perm(__float_as_uint(f0), __float_as_uint(f1), 0x7632);
    hi = __byte_perm(__float_as_uint(f2), __float_as_uint(f3), 0x7632);
}

// ---------------------------------------------------------------------------------------------
// Warp-level MMA (register fragments).  The decode GEMV is HBM-bound, so the register-resident
// m16n8k16 form is used there; the dense prefill/int8-dyn GEMMs use tcgen05 + tensor memory.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---------------------------------------------------------------------------------------------
// Host-side error reporting (thread-local last message, read through sbq_last_error()).
// ---------------------------------------------------------------------------------------------
int set_error(int status, const char* fmt, ...);
int check_launch(const char* what);

}  // namespace sbq
