// Prefill GEMM of the int8 weight-only format: Y[m, n] = (X[m, k] . Wq[n, k]^T) * scale[n].
//
// Reference: Int8Linear.forward (spikingbrain_cpu/quant.py:41-53) at prefill shapes (512-token
// chunks, model.py:439).  The reference dequantises 128-row weight blocks to fp32 and runs an fp32
// sgemm, then scales.  Here one CTA computes a 128-channel x 256-token tile, transposed (channels
// are the MMA's M):
//   * warp 0 (one thread) streams 256 x 64 fp16 activation tiles (TMA, 128-byte swizzle) and the
//     matching 128 x 64 int8 weight tiles (TMA over the packed layout, 64-byte swizzle) into a
//     5-stage ring;
//   * warps 4-7 and 8-11 (two warpgroups taking alternate k-blocks; one weight row per thread)
//     convert each int8 row to fp16 in registers (exact) and write it straight into tensor memory
//     with tcgen05.st - the MMA's A operand - in a 4-deep ring;
//   * warp 1 (one thread) issues tcgen05.mma.cta_group::1.kind::f16 with A from tensor memory and
//     the activation tile from shared memory (128 x 256 x 16, fp32 accumulators in TMEM);
//   * both warpgroups finally read their channel's accumulators (tcgen05.ld; one half of the
//     tokens each), apply the fp32 per-row scale (and bias) and store fp16 or fp32 output,
//     consecutive channels per warp store.
// The scale stays in the fp32 epilogue, as in the reference: int8 values are exact in fp16.
//
// Activation kinds: fp16 (int8 -> fp16 weights, kind::f16 with f16 operands), bf16 (int8 -> bf16
// weights, bf16 operands) and fp32 split into a bf16 high and low part (x = hi + lo to ~2^-17
// relative; both parts are tiles of the same stage and each k-step issues one MMA per part into the
// same accumulator, so the weight operand is converted once).  int8 x bf16 products are exact in
// fp32, so the fp32 path loses only the split's rounding and the fp32 accumulation.
#include <atomic>

#include "tc.cuh"

namespace sbq {

struct GemmW16Params {
    int m, n, k, num_kb;
    const float* scale;
    const float* bias;
    void* y;
    int64_t ldy;
    int gated;  // y already holds the gate projection: store silu(gate) * result in its place
};

// One output element.  With `gated`, y holds the gate projection of the same rows (written by an
// earlier launch into this buffer) and receives silu(gate) * v (GatedMLP.forward, model.py:239-240).
template <bool OUT_F16, class P>
__device__ __forceinline__ float load_y(const P& p, int t, int n) {
    const int64_t idx = (int64_t)t * p.ldy + n;
    return OUT_F16 ? __half2float(static_cast<const __half*>(p.y)[idx]) : static_cast<const float*>(p.y)[idx];
}

template <bool OUT_F16, class P>
__device__ __forceinline__ void put_y(const P& p, int t, int n, float v) {
    const int64_t idx = (int64_t)t * p.ldy + n;
    if (OUT_F16)
        static_cast<__half*>(p.y)[idx] = __float2half_rn(v);
    else
        static_cast<float*>(p.y)[idx] = v;
}

template <bool OUT_F16, class P>
__device__ __forceinline__ void store_y(const P& p, int t, int n, float v) {
    const int64_t idx = (int64_t)t * p.ldy + n;
    if (p.gated) {
        const float g = OUT_F16 ? __half2float(static_cast<const __half*>(p.y)[idx]) : static_cast<const float*>(p.y)[idx];
        v = g / (1.0f + expf(-g)) * v;
    }
    if (OUT_F16)
        static_cast<__half*>(p.y)[idx] = __float2half_rn(v);
    else
        static_cast<float*>(p.y)[idx] = v;
}

// Activation kinds of the tensor-memory GEMMs.
enum AKind { kAF16 = 0, kABF16 = 1, kABF16x2 = 2 };

// int8 weight row (64 bytes at w8, 64-byte swizzle of row `row`) -> 32 words of 16-bit pairs in
// the activation's type (exact: |q| <= 127).
template <int AK>
__device__ __forceinline__ void convert_row(const uint8_t* w8, int row, uint32_t (&h)[32]) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const uint4 v = *reinterpret_cast<const uint4*>(w8 + ((c ^ ((row >> 1) & 3)) << 4));
        if (AK == kAF16) {
            i8x4_to_half2x2(v.x, h[8 * c + 0], h[8 * c + 1]);
            i8x4_to_half2x2(v.y, h[8 * c + 2], h[8 * c + 3]);
            i8x4_to_half2x2(v.z, h[8 * c + 4], h[8 * c + 5]);
            i8x4_to_half2x2(v.w, h[8 * c + 6], h[8 * c + 7]);
        } else {
            i8x4_to_bf162x2(v.x, h[8 * c + 0], h[8 * c + 1]);
            i8x4_to_bf162x2(v.y, h[8 * c + 2], h[8 * c + 3]);
            i8x4_to_bf162x2(v.z, h[8 * c + 4], h[8 * c + 5]);
            i8x4_to_bf162x2(v.w, h[8 * c + 6], h[8 * c + 7]);
        }
    }
}

constexpr int kWCh = 128;      // output channels per CTA (one per TMEM lane)
constexpr int kWBK = 64;       // k per k-block (one 128-byte 16-bit row, one packed tile column)
constexpr int kWThreads = 384; // 12 warps: producer, MMA, TMEM, idle, then two converter warpgroups
constexpr uint32_t kWTmemCols = 512;
constexpr uint32_t kWAccCol = 0;    // accumulator from column 0; weight operand buffers after it

// ---------------------------------------------------------------------------------------------
// Prefill GEMM (more than 128 activation rows), CTA pairs: a 2-CTA cluster computes a 256-channel x
// 256-token tile with tcgen05.mma.cta_group::2 (M = 256 over both CTAs' tensor memory, N = 256 over
// both CTAs' shared memory).  Each CTA converts its own 128 weight rows (int8 -> 16-bit, exact) into
// its own tensor memory and loads half of the activation tile (128 tokens), so a 64-deep k-block
// moves 24 KiB into each SM instead of the 40 KiB of a one-CTA 128 x 256 tile: a per-k-block trace
// of that one-CTA kernel showed its converters waiting ~0.6 us per k-block for TMA data, the loop
// bound by the L2 -> shared-memory traffic of the activation tile each CTA re-read.  Both CTAs'
// activation loads complete on the leader's (rank 0's) barrier, both CTAs' converters arrive on the
// leader's operand barrier, and the leader's MMA commits release each CTA's stage and operand buffer
// (one commit per barrier, no multicast).  Roles: warp 0 TMA producer, warp 1 MMA issuer (leader),
// warp 2 TMEM allocation, warps 4-11 two converter warpgroups (alternate k-blocks), then the
// epilogue (each thread one channel, each warpgroup one half of the 256 tokens).
#ifndef SBQ_W16_PAIR_KH
#define SBQ_W16_PAIR_KH 2
#endif
#ifndef SBQ_W16_PAIR_STAGES
#define SBQ_W16_PAIR_STAGES 4
#endif
#ifndef SBQ_W16_PAIR_STAGES_X2
#define SBQ_W16_PAIR_STAGES_X2 5
#endif
constexpr int kPThreads = kWThreads;

// TOK: the pair's tokens per tile (the MMA's N): 256, or 128 when 256-token tiles leave SMs idle
// (the reference's 512-token prefill chunks); each CTA loads TOK / 2 of them.
template <int AK, int TOK>
struct PairSmem {
    static_assert(TOK == 128 || TOK == 256, "token tile");
    static constexpr int kTokHalf = TOK / 2;
    // k per stage: kKH sub-blocks of 64 (128 for 16-bit x, so that the MMA thread's two waits and two
    // commits per stage cover 8 MMAs; 64 for a split fp32 x, whose stage is twice as large)
    static constexpr int kKH = AK == kABF16x2 ? 1 : SBQ_W16_PAIR_KH;
    static constexpr int kXSub = kTokHalf * kWBK * 2;      // this CTA's tokens x 64 k (16 or 8 KiB)
    static constexpr int kXTiles = AK == kABF16x2 ? 2 : 1;  // high and low part of a split fp32 x
    static constexpr int kXStage = kKH * kXTiles * kXSub;
    static constexpr int kW8Sub = kWCh * kWBK;             // 8 KiB: this CTA's 128 weight rows x 64 k
    static constexpr int kStage = kXStage + kKH * kW8Sub;
    static constexpr int kStages0 = AK == kABF16x2 ? SBQ_W16_PAIR_STAGES_X2 : SBQ_W16_PAIR_STAGES;
    // 128-token tiles have smaller stages: as many as fit the same ring (at most 8)
    static constexpr int kStagesFit = (196 * 1024) / kStage < 8 ? (196 * 1024) / kStage : 8;
    static constexpr int kStages = TOK == 256 ? kStages0 : kStagesFit;
    static constexpr int kBarOff = kStages * kStage;
    static constexpr int kBytes = kBarOff + 512 + kWCh * 8 + 1024;
    static_assert(kKH >= 1 && kKH <= 4, "64 to 256 k per stage");
    static_assert(kBytes <= 227 * 1024, "shared memory per CTA");
    // one weight operand buffer in tensor memory per stage (kACols columns each, after the TOK
    // accumulator columns): a stage's activation tiles and converted weights are ready together
    static constexpr uint32_t kACol = TOK;
    static constexpr int kACols = kKH * (kWBK / 2);
    static_assert(TOK + kStages * kACols <= (int)(kWTmemCols - kWAccCol), "operand buffers fit in tensor memory");
    static_assert(4 * kStages + 1 <= 60, "barriers fit in 512 bytes with the TMEM slot");
};

template <bool OUT_F16, bool GATED, int AK, int TOK>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPThreads, 1)
    gemm_w8a16_pair_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_x2,
                           const __grid_constant__ CUtensorMap tmap_w, const GemmW16Params p) {
    using S = PairSmem<AK, TOK>;
    constexpr int kStages = S::kStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* wfull = reinterpret_cast<uint64_t*>(smem + S::kBarOff);  // this CTA's weight tile landed
    // the stage is ready for the MMAs: both activation halves landed (transaction bytes) and both
    // CTAs' 4 converter warps wrote its weight operand buffer (arrivals); the leader's is used
    uint64_t* ready = wfull + kStages;
    uint64_t* conv_done = ready + kStages;  // this CTA's 4 converter warps have read the weight tile
    uint64_t* mma_done = conv_done + kStages;  // the pair's MMAs of the stage's k-block completed
    uint64_t* done = mma_done + kStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    float* s_scale = reinterpret_cast<float*>(smem + S::kBarOff + 512);
    float* s_bias = s_scale + kWCh;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = tc::cluster_ctarank();
    const bool leader = rank == 0;
    const int n0 = (blockIdx.x >> 1) * (2 * kWCh) + (int)rank * kWCh;  // this CTA's 128 channels
    const int t0 = blockIdx.y * TOK;                                    // the pair's TOK tokens
    // the next launch on the stream may start its prologue (and weight tiles) now; it waits for
    // this grid before it touches activations or outputs
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            tc::mbar_init(&wfull[s], 1);
            tc::mbar_init(&ready[s], 1 + 8);  // the leader's producer (with the bytes) + 8 converter warps
            tc::mbar_init(&conv_done[s], 4);
            tc::mbar_init(&mma_done[s], 1);
        }
        tc::mbar_init(done, 1);
        tc::fence_mbar_init();
        tc::prefetch_tmap(&tmap_x);
        if (AK == kABF16x2) tc::prefetch_tmap(&tmap_x2);
        tc::prefetch_tmap(&tmap_w);
    }
    if (warp == 2) {
        tc::tmem_alloc_pair(tmem_slot, kWTmemCols);
        tc::tmem_relinquish_pair();
    }
    for (int i = threadIdx.x; i < kWCh; i += blockDim.x) {
        const int n = n0 + i;
        s_scale[i] = n < p.n ? p.scale[n] : 0.0f;
        s_bias[i] = (p.bias && n < p.n) ? p.bias[n] : 0.0f;
    }
    tc::fence_before_sync();
    tc::cluster_sync();  // both CTAs' barriers exist before either CTA's loads or arrivals reach them
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // weight tiles of the first stages before griddepcontrol.wait (launched as a programmatic
            // dependent, the previous kernel may still run: it writes activations, never weights),
            // activation tiles after it
            const int tr = t0 + (int)rank * S::kTokHalf;
            auto load_w = [&](int kb) {
                const int s = kb % kStages;
                uint8_t* ws = smem + s * S::kStage + S::kXStage;
                tc::mbar_arrive_expect_tx(&wfull[s], S::kKH * S::kW8Sub);
#pragma unroll
                for (int h = 0; h < S::kKH; ++h)
                    tc::tma_load_4d(ws + h * S::kW8Sub, &tmap_w, &wfull[s], 0, 0, kb * S::kKH + h, n0 / 16);
            };
            auto load_x = [&](int kb) {
                const int s = kb % kStages;
                uint8_t* xs = smem + s * S::kStage;
                const uint32_t xb = tc::cluster_addr(&ready[s], 0);
                if (leader) tc::mbar_arrive_expect_tx(&ready[s], 2 * S::kXStage);
#pragma unroll
                for (int h = 0; h < S::kKH; ++h) {
                    const int kc = kb * S::kKH + h;  // 64-wide k column
                    tc::tma_load_2d_pair(xs + h * S::kXTiles * S::kXSub, &tmap_x, xb, kc * kWBK, tr);
                    if (AK == kABF16x2)
                        tc::tma_load_2d_pair(xs + (h * S::kXTiles + 1) * S::kXSub, &tmap_x2, xb, kc * kWBK, tr);
                }
            };
            const int pre = p.num_kb < kStages ? p.num_kb : kStages;
            for (int kb = 0; kb < pre; ++kb) load_w(kb);
            asm volatile("griddepcontrol.wait;" ::: "memory");
            for (int kb = 0; kb < pre; ++kb) load_x(kb);
            for (int kb = pre; kb < p.num_kb; ++kb) {
                const int s = kb % kStages;
                const uint32_t ph = (kb / kStages) & 1;
                if (!tc::mbar_wait(&conv_done[s], ph ^ 1)) break;
                if (!tc::mbar_wait(&mma_done[s], ph ^ 1)) break;
                load_w(kb);
                load_x(kb);
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            constexpr uint32_t idesc = tc::idesc_f16(2 * kWCh, TOK, AK != kAF16);
            for (int kb = 0; kb < p.num_kb; ++kb) {
                const int s = kb % kStages;
                const uint32_t ph = (kb / kStages) & 1;
                if (!tc::mbar_wait_cluster(&ready[s], ph)) break;
                tc::fence_after_sync();
                const uint8_t* xs = smem + s * S::kStage;
                const uint32_t a_col = tmem + S::kACol + s * S::kACols;
#pragma unroll
                for (int h = 0; h < S::kKH; ++h) {
                    const uint8_t* xh = xs + h * S::kXTiles * S::kXSub;
#pragma unroll
                    for (int j = 0; j < kWBK / 16; ++j) {
                        const uint64_t bd = tc::smem_desc(xh + j * 32, tc::kSwizzle128B, 1024);
                        tc::mma_f16_ts_pair(tmem + kWAccCol, a_col + h * (kWBK / 2) + j * 8, bd, idesc, (kb | h | j) != 0);
                        if (AK == kABF16x2) {
                            const uint64_t bl = tc::smem_desc(xh + S::kXSub + j * 32, tc::kSwizzle128B, 1024);
                            tc::mma_f16_ts_pair(tmem + kWAccCol, a_col + h * (kWBK / 2) + j * 8, bl, idesc, 1u);
                        }
                    }
                }
                // one barrier per CTA: frees the stage's activation half and operand buffer
                tc::mma_commit_pair(tc::cluster_addr(&mma_done[s], 0));
                tc::mma_commit_pair(tc::cluster_addr(&mma_done[s], 1));
            }
            tc::mma_commit_pair(tc::cluster_addr(done, 0));
            tc::mma_commit_pair(tc::cluster_addr(done, 1));
        }
    } else if (warp >= 4) {
        const int grp = (warp - 4) >> 2;          // converter warpgroup: even (0) or odd (1) k-blocks
        const int wq = (warp - 4) & 3;            // lanes 32 wq .. 32 wq + 31 of tensor memory
        const int row = wq * 32 + lane;           // weight row (output channel) of this thread
        const uint32_t lane_addr = (uint32_t)(wq * 32) << 16;
        bool ok = true;
        for (int kb = grp; kb < p.num_kb; kb += 2) {
            const int s = kb % kStages;
            const uint32_t ph = (kb / kStages) & 1;
            // warp-uniform waits: tcgen05.st below is warp-collective.  The stage's operand buffer
            // was last read by the MMAs of k-block kb - kStages; waiting for them first also
            // guarantees that every k-block up to there was converted, so the weight stage's earlier
            // phases are complete and its parity wait can only pass on this k-block's tile.
            if (kb >= kStages) {
                if (!__all_sync(0xffffffffu, tc::mbar_wait(&mma_done[s], ph ^ 1))) { ok = false; break; }
            }
            if (!__all_sync(0xffffffffu, tc::mbar_wait(&wfull[s], ph))) { ok = false; break; }
            tc::fence_after_sync();
#pragma unroll
            for (int hh = 0; hh < S::kKH; ++hh) {
                uint32_t h[32];
                convert_row<AK>(smem + s * S::kStage + S::kXStage + hh * S::kW8Sub + row * 64, row, h);
                tc::tmem_st_32x32b_x32(tmem + lane_addr + S::kACol + s * S::kACols + hh * (kWBK / 2), h);
            }
            tc::tmem_wait_st();
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) {
                tc::mbar_arrive_cluster(tc::cluster_addr(&ready[s], 0));
                tc::mbar_arrive(&conv_done[s]);
            }
        }
        // ---- epilogue: this thread's channel, 256 tokens of accumulators
        ok = __all_sync(0xffffffffu, ok && tc::mbar_wait(done, 0));
        tc::fence_after_sync();
        asm volatile("griddepcontrol.wait;" ::: "memory");  // y may be read (gated) or written from here
        if (ok) {
            const int n = n0 + row;
            const float sc = s_scale[row], bi = s_bias[row];
            const bool has_bias = p.bias != nullptr;
#pragma unroll 1
            for (int c = grp * (TOK / 64); c < (grp + 1) * (TOK / 64); ++c) {  // this group's token half
                uint32_t r[32];
                tc::tmem_ld_32x32b_x32(tmem + lane_addr + kWAccCol + c * 32, r);
                tc::tmem_wait_ld();
                if (n >= p.n) continue;
                const int tb = t0 + c * 32;
                if constexpr (GATED) {
                    float gv[32];
#pragma unroll
                    for (int j = 0; j < 32; ++j) gv[j] = tb + j < p.m ? load_y<OUT_F16>(p, tb + j, n) : 0.0f;
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        if (tb + j >= p.m) break;
                        float v = __fmul_rn(__uint_as_float(r[j]), sc);
                        if (has_bias) v = __fadd_rn(v, bi);
                        put_y<OUT_F16>(p, tb + j, n, gv[j] / (1.0f + expf(-gv[j])) * v);
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int t = tb + j;
                        if (t >= p.m) break;
                        float v = __fmul_rn(__uint_as_float(r[j]), sc);
                        if (has_bias) v = __fadd_rn(v, bi);
                        put_y<OUT_F16>(p, t, n, v);
                    }
                }
            }
        }
    }
    tc::fence_before_sync();
    // neither CTA frees its tensor memory or leaves while the pair's MMAs or commits may still use
    // its shared or tensor memory
    tc::cluster_sync();
    if (warp == 2) {
        tc::fence_after_sync();
        tc::tmem_dealloc_pair(tmem, kWTmemCols);
    }
}

// ---------------------------------------------------------------------------------------------
// Small-batch variant (17..128 activation rows, e.g. batched decode): 128-channel x 64-token tiles,
// a 96 KiB TMA ring (2 CTAs per SM), and split-K over a thread-block cluster when the tiles alone
// cannot fill the GPU: the S CTAs of a cluster (one K part each) push their fp32 partial sums into
// the shared memory of the CTA owning each channel (1/S of the channels per CTA) through distributed
// shared memory, and each CTA reduces its share in part order (deterministic), then scales and
// stores.  Roles as in the prefill kernel (one CTA, no pair).
// ---------------------------------------------------------------------------------------------
constexpr int kSTok = 64;      // activation rows per CTA (MMA N)
constexpr uint32_t kSTmemCols = 256;  // accumulator [0, 64), weight operand buffers from 64
constexpr uint32_t kSACol = 64;
#ifndef SBQ_W16_SMALL_KH
#define SBQ_W16_SMALL_KH 2
#endif
#ifndef SBQ_W16_SMALL_RING_KB
#define SBQ_W16_SMALL_RING_KB 96
#endif
constexpr int kSmallCtasPerSm = SBQ_W16_SMALL_RING_KB <= 100 ? 2 : 1;

// A pipeline block is kKH 64-deep k-blocks: the MMA thread waits twice and commits twice per block,
// which at N = 64 (four short MMAs per 64-deep k-block) cost as much as the MMAs themselves.
template <int AK>
struct SmallSmem {
    static constexpr int kKH = AK == kABF16x2 ? 1 : SBQ_W16_SMALL_KH;  // 64-deep k-blocks per stage
    static constexpr int kX = kSTok * kWBK * 2;            // 8 KiB 16-bit activation tile (64 deep)
    static constexpr int kXTiles = AK == kABF16x2 ? 2 : 1;  // high and low part of a split fp32 x
    static constexpr int kW8 = kWCh * kWBK;                // 8 KiB int8 weight tile (64 deep)
    static constexpr int kXStage = kKH * kXTiles * kX;
    static constexpr int kStage = kXStage + kKH * kW8;
    static constexpr int kStages = (SBQ_W16_SMALL_RING_KB * 1024) / kStage;
    static constexpr int kBarOff = kStages * kStage;
    static constexpr int kBytes = kBarOff + 256 + kWCh * 8 + 1024;
    static constexpr int kACols = kKH * (kWBK / 2);        // tensor-memory columns of one operand buffer
    // one weight operand buffer per stage in tensor memory (a converter that has seen the stage's
    // previous MMAs complete also knows every earlier phase of the stage's barriers is complete)
    static_assert(kSACol + kStages * kACols <= (int)kSTmemCols, "operand buffers fit in tensor memory");
    static_assert(kKH >= 1 && kKH <= 2, "64 or 128 k per stage");
    static_assert(kStages >= 2, "pipeline depth");
    static_assert(4 * kStages + 1 <= 30, "barriers fit in 256 bytes with the TMEM slot");
    // split-K receive buffer: [parts][64 tokens][rs] floats, rs = ceil(128 / parts) rounded up to
    // 4: at most 6 x 64 x 24 floats (parts = 6) for parts <= 8
    static_assert(6 * kSTok * 24 * 4 <= kStages * kStage, "receive buffer fits in the ring");
    static_assert(kSmallCtasPerSm * kBytes <= 228 * 1024, "CTAs per SM");
};

struct GemmSmallParams {
    int m, n, k, num_kb, parts;
    int gated;             // as GemmW16Params::gated
    const float* scale;
    const float* bias;
    void* y;
    int64_t ldy;
};

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Shared-memory address `a` of this CTA mapped into cluster CTA `rank`'s shared memory.
__device__ __forceinline__ uint32_t dsmem_map(uint32_t a, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
    return r;
}

__device__ __forceinline__ void st_dsmem(uint32_t cluster_addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(cluster_addr), "f"(v) : "memory");
}


template <bool OUT_F16, int AK>
__global__ void __launch_bounds__(kWThreads, kSmallCtasPerSm) gemm_w8a16_small_kernel(const __grid_constant__ CUtensorMap tmap_x,
                                                                        const __grid_constant__ CUtensorMap tmap_x2,
                                                                        const __grid_constant__ CUtensorMap tmap_w,
                                                                        const GemmSmallParams p) {
    using S = SmallSmem<AK>;
    constexpr int kSStages = S::kStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* wfull = reinterpret_cast<uint64_t*>(smem + S::kBarOff);  // the stage's weight tiles landed
    uint64_t* ready = wfull + kSStages;      // activation tiles landed and the 4 converter warps wrote
    uint64_t* conv_done = ready + kSStages;  // the 4 converter warps have read the weight tiles
    uint64_t* mma_done = conv_done + kSStages;  // the stage's MMAs completed (activations, operand buffer)
    uint64_t* done = mma_done + kSStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    float* s_scale = reinterpret_cast<float*>(smem + S::kBarOff + 256);
    float* s_bias = s_scale + kWCh;
    float* recv = reinterpret_cast<float*>(smem);  // split-K receive buffer, after the main loop

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * kWCh, t0 = blockIdx.y * kSTok;
    const int part = p.parts > 1 ? (int)cluster_rank() : 0;
    const int kb0 = part * p.num_kb / p.parts, kb1 = (part + 1) * p.num_kb / p.parts;
    // the next launch on the stream may start its prologue (and weight tiles) now; it waits for
    // this grid before it touches activations or outputs
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (threadIdx.x == 0) {
        for (int s = 0; s < kSStages; ++s) {
            tc::mbar_init(&wfull[s], 1);
            tc::mbar_init(&ready[s], 1 + 4);  // the producer (with the activation bytes) + 4 converter warps
            tc::mbar_init(&conv_done[s], 4);
            tc::mbar_init(&mma_done[s], 1);
        }
        tc::mbar_init(done, 1);
        tc::fence_mbar_init();
        tc::prefetch_tmap(&tmap_x);
        if (AK == kABF16x2) tc::prefetch_tmap(&tmap_x2);
        tc::prefetch_tmap(&tmap_w);
    }
    if (warp == 2) {
        tc::tmem_alloc(tmem_slot, kSTmemCols);
        tc::tmem_relinquish();
    }
    for (int i = threadIdx.x; i < kWCh; i += blockDim.x) {
        const int n = n0 + i;
        s_scale[i] = n < p.n ? p.scale[n] : 0.0f;
        s_bias[i] = (p.bias && n < p.n) ? p.bias[n] : 0.0f;
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    const int nkb = kb1 - kb0;
    uint32_t r[32];  // a converter thread's accumulators after the main loop (split-K partial sums)

    if (warp == 0) {
        if (lane == 0) {
            // weight tiles of the first stages before griddepcontrol.wait (launched as a programmatic
            // dependent, the previous kernel may still run: it writes activations, never weights),
            // activation tiles after it
            auto load_x = [&](int i) {
                const int s = i % kSStages;
                uint8_t* xs = smem + s * S::kStage;
                tc::mbar_arrive_expect_tx(&ready[s], S::kXStage);
#pragma unroll
                for (int h = 0; h < S::kKH; ++h) {
                    const int kc = (kb0 + i) * S::kKH + h;  // 64-deep k column
                    tc::tma_load_2d(xs + h * S::kXTiles * S::kX, &tmap_x, &ready[s], kc * kWBK, t0);
                    if (AK == kABF16x2)
                        tc::tma_load_2d(xs + (h * S::kXTiles + 1) * S::kX, &tmap_x2, &ready[s], kc * kWBK, t0);
                }
            };
            auto load_w = [&](int i) {
                const int s = i % kSStages;
                uint8_t* xs = smem + s * S::kStage;
                tc::mbar_arrive_expect_tx(&wfull[s], S::kStage - S::kXStage);
#pragma unroll
                for (int h = 0; h < S::kKH; ++h)
                    tc::tma_load_4d(xs + S::kXStage + h * S::kW8, &tmap_w, &wfull[s], 0, 0, (kb0 + i) * S::kKH + h,
                                    n0 / 16);
            };
            const int pre = nkb < kSStages ? nkb : kSStages;
            for (int i = 0; i < pre; ++i) load_w(i);
            asm volatile("griddepcontrol.wait;" ::: "memory");
            for (int i = 0; i < pre; ++i) load_x(i);
            for (int i = pre; i < nkb; ++i) {
                const int s = i % kSStages;
                const uint32_t ph = (i / kSStages) & 1;
                if (!tc::mbar_wait(&conv_done[s], ph ^ 1)) break;
                if (!tc::mbar_wait(&mma_done[s], ph ^ 1)) break;
                load_w(i);
                load_x(i);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_f16(kWCh, kSTok, AK != kAF16);
            for (int i = 0; i < nkb; ++i) {
                const int s = i % kSStages;
                const uint32_t ph = (i / kSStages) & 1;
                if (!tc::mbar_wait(&ready[s], ph)) break;
                tc::fence_after_sync();
                const uint8_t* xs = smem + s * S::kStage;
                const uint32_t a_col = tmem + kSACol + s * S::kACols;
#pragma unroll
                for (int h = 0; h < S::kKH; ++h) {
                    const uint8_t* xh = xs + h * S::kXTiles * S::kX;
#pragma unroll
                    for (int j = 0; j < kWBK / 16; ++j) {
                        const uint64_t bd = tc::smem_desc(xh + j * 32, tc::kSwizzle128B, 1024);
                        tc::mma_f16_ts(tmem, a_col + h * (kWBK / 2) + j * 8, bd, idesc, (i | h | j) != 0);
                        if (AK == kABF16x2) {
                            const uint64_t bl = tc::smem_desc(xh + S::kX + j * 32, tc::kSwizzle128B, 1024);
                            tc::mma_f16_ts(tmem, a_col + h * (kWBK / 2) + j * 8, bl, idesc, 1u);
                        }
                    }
                }
                tc::mma_commit(&mma_done[s]);
            }
            tc::mma_commit(done);
        }
    } else if (warp >= 4) {
        const int grp = (warp - 4) >> 2;
        const int wq = (warp - 4) & 3;
        const int row = wq * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(wq * 32) << 16;
        // the two groups take alternate pipeline blocks; a block's kKH tensor-memory stores share
        // one wait (the MMA of a 64-token tile is short, so the conversion latency sets the pace)
        bool ok = true;
        for (int i = grp; i < nkb; i += 2) {
            const int s = i % kSStages;
            const uint32_t ph = (i / kSStages) & 1;
            // operand buffer first: the MMAs of block i - kStages are done, so every block up to
            // there was loaded and converted (the MMA thread waits in order) and the stage's earlier
            // phases are complete - the parity wait below can only pass on block i's own data.  (The
            // other group converts block i - 1; this group's previous block, i - 2, says nothing
            // about when block i - kStages landed.)
            if (i >= kSStages) {
                if (!__all_sync(0xffffffffu, tc::mbar_wait(&mma_done[s], ph ^ 1))) { ok = false; break; }
            }
            if (!__all_sync(0xffffffffu, tc::mbar_wait(&wfull[s], ph))) { ok = false; break; }
            tc::fence_after_sync();
#pragma unroll
            for (int h = 0; h < S::kKH; ++h) {
                uint32_t hv[32];
                convert_row<AK>(smem + s * S::kStage + S::kXStage + h * S::kW8 + row * 64, row, hv);
                tc::tmem_st_32x32b_x32(tmem + lane_addr + kSACol + s * S::kACols + h * (kWBK / 2), hv);
            }
            tc::tmem_wait_st();
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) {
                tc::mbar_arrive(&ready[s]);
                tc::mbar_arrive(&conv_done[s]);
            }
        }
        // ---- this thread's channel, this group's 32 tokens of accumulators
        ok = __all_sync(0xffffffffu, ok && tc::mbar_wait(done, 0));
        tc::fence_after_sync();
        asm volatile("griddepcontrol.wait;" ::: "memory");  // y may be read (gated) or written from here
        tc::tmem_ld_32x32b_x32(tmem + lane_addr + grp * 32, r);
        tc::tmem_wait_ld();
        if (!ok) {
#pragma unroll
            for (int j = 0; j < 32; ++j) r[j] = 0u;
        }
        if (p.parts == 1) {
            const int n = n0 + row;
            if (n < p.n) {
                const float sc = s_scale[row], bi = s_bias[row];
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int t = t0 + grp * 32 + j;
                    if (t >= p.m) break;
                    float v = __fmul_rn(__uint_as_float(r[j]), sc);
                    if (p.bias) v = __fadd_rn(v, bi);
                    store_y<OUT_F16>(p, t, n, v);
                }
            }
        }
    }
    if (p.parts > 1) {
        // split K.  (1) Every CTA of the cluster has finished its main loop, so every ring is free.
        // (2) Each converter thread pushes its 32 partial sums into the shared memory of the CTA
        // that owns its channel, token-major: recv[part][token][row - r0] (row stride rs), so the 32
        // lanes of a warp (32 consecutive channels) store 128 contiguous bytes per token - remote
        // stores of scattered 16-byte pieces ran at ~17 GB/s per SM.  (3) Once all have landed,
        // each CTA reduces its channel share in part order (a fixed order: deterministic), scales
        // and stores.  Every thread takes both cluster barriers.
        cluster_sync_all();
        const int share = (kWCh + p.parts - 1) / p.parts, rs = (share + 3) & ~3;
        if (warp >= 4) {
            const int row = ((warp - 4) & 3) * 32 + lane, grp = (warp - 4) >> 2;
            int q = 0;
            while (q + 1 < p.parts && (q + 1) * kWCh / p.parts <= row) ++q;
            const int qr0 = q * kWCh / p.parts;
            const uint32_t dst =
                dsmem_map(tc::smem_u32(recv + ((part * kSTok + grp * 32) * rs + row - qr0)), (uint32_t)q);
#pragma unroll
            for (int j = 0; j < 32; ++j) st_dsmem(dst + (uint32_t)(j * rs * 4), __uint_as_float(r[j]));
        }
        cluster_sync_all();
        asm volatile("griddepcontrol.wait;" ::: "memory");  // y is read (gated) or written below
        const int r0 = part * kWCh / p.parts, r1 = (part + 1) * kWCh / p.parts, nr = r1 - r0;
        const int nq = (nr + 3) / 4;  // row quads of this CTA's share (the last may be partial)
        for (int e = threadIdx.x; e < nq * kSTok; e += blockDim.x) {
            const int rq = (e % nq) * 4, t = e / nq;  // 4 channels x 1 token: y stores along channels
            if (t0 + t >= p.m) continue;
            float4 acc = *reinterpret_cast<const float4*>(recv + t * rs + rq);
#pragma unroll
            for (int q = 1; q < 8; ++q) {
                if (q < p.parts) {
                    const float4 v = *reinterpret_cast<const float4*>(recv + ((q * kSTok + t) * rs + rq));
                    acc.x += v.x, acc.y += v.y, acc.z += v.z, acc.w += v.w;
                }
            }
            const float a4[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int row = r0 + rq + j, n = n0 + row;
                if (rq + j >= nr || n >= p.n) break;
                float o = __fmul_rn(a4[j], s_scale[row]);
                if (p.bias) o = __fadd_rn(o, s_bias[row]);
                store_y<OUT_F16>(p, t0 + t, n, o);
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 2) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, kSTmemCols);
    }
}

SBQ_DEFINE_ERROR_POLL(poll_error_w8a16)

int check_linear_args(const void* x, int x_dtype, int64_t ldx, const void* packed, const float* scale, int64_t m,
                      int64_t n, int64_t k, const void* y, int y_dtype, int64_t ldy);

}  // namespace sbq

using namespace sbq;

constexpr int64_t kSmallMaxRows = 128;  // up to this many activation rows: the 64-token kernel

// SMs of the current device, cached per device (atomics: first calls may come from several threads)
static int sm_count_w16() {
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

// 16-bit activation [m, k] (row stride ldx elements) as box_rows x 64 boxes, 128-byte swizzle.
static int make_x_map(CUtensorMap* map, int ak, const void* x, int64_t ldx, int64_t m, int64_t k, int box_rows) {
    const uint64_t dims[2] = {(uint64_t)k, (uint64_t)m};
    const uint64_t strides[1] = {(uint64_t)ldx * 2};
    const uint32_t box[2] = {kWBK, (uint32_t)box_rows};
    return encode_tmap(map, ak == kAF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, dims,
                       strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

// The packed weight viewed as {64 bytes, 16 rows, KT tiles, NT tile-rows}, one 128-row tile column per box.
static int make_w_map(CUtensorMap* map, const void* packed, int64_t n, int64_t k) {
    const uint64_t kt = (uint64_t)ceil_div(k, kTileCols), nt = (uint64_t)ceil_div(n, kTileRows);
    const uint64_t dims[4] = {64, 16, kt, nt};
    const uint64_t strides[3] = {64, 1024, kt * 1024};
    const uint32_t box[4] = {64, 16, 1, kWCh / 16};
    return encode_tmap(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, packed, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B);
}

template <bool OUT_F16, int AK>
static cudaError_t launch_small(const cudaLaunchConfig_t& cfg, const CUtensorMap& mx, const CUtensorMap& mx2,
                                const CUtensorMap& mw, const GemmSmallParams& p) {
    cudaFuncSetAttribute(gemm_w8a16_small_kernel<OUT_F16, AK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)cfg.dynamicSmemBytes);
    return cudaLaunchKernelEx(&cfg, gemm_w8a16_small_kernel<OUT_F16, AK>, mx, mx2, mw, p);
}

template <int AK>
static int gemm_small(const CUtensorMap& mx, const CUtensorMap& mx2, const CUtensorMap& mw, const float* scale,
                      const float* bias, int64_t m, int64_t n, int64_t k, void* y, int y_dtype, int64_t ldy, void* stream,
                      int gated) {
    GemmSmallParams p{};
    p.gated = gated;
    p.m = (int)m;
    p.n = (int)n;
    p.k = (int)k;
    p.num_kb = (int)ceil_div(k, kWBK * SmallSmem<AK>::kKH);  // pipeline blocks; k past the end reads zeros
    p.scale = scale;
    p.bias = bias;
    p.y = y;
    p.ldy = ldy;
    // K parts per tile (the cluster size): the largest power of two up to 8 that keeps the grid within
    // ~7/8 of the CTA slots (two per SM) and gives every part at least 2 pipeline blocks.  Measured on
    // B200 (20 calls per CUDA graph, us; the chosen count marked):
    //   m x n x k          tiles  parts=1    2      4      8
    //   64 x 4096 x 4096     32    20.9   14.2   12.0  *10.8
    //   64 x 12288 x 4096    96    23.6  *17.8   21.5   31.4
    //   64 x 4096 x 12288    32    56.8   33.4   22.1  *19.0
    //   128 x 4096 x 4096    64    22.3   16.9  *12.9   21.0
    //   100 x 2560 x 2560    40    14.3   12.2  *10.3   15.6
    // (cluster sizes 3 and 6 were never better).  Larger grids leave clusters waiting for a second
    // wave: a cluster needs all its CTAs resident in one GPC at once.
    const int tiles = (int)(ceil_div(n, kWCh) * ceil_div(m, kSTok));
    const int slots = 2 * sm_count_w16();
    int parts = 1;
    while (parts < 8 && (int64_t)tiles * (2 * parts) * 8 <= (int64_t)slots * 7 && p.num_kb / (2 * parts) >= 2)
        parts *= 2;
    p.parts = parts;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)ceil_div(n, kWCh), (unsigned)ceil_div(m, kSTok), (unsigned)parts);
    cfg.blockDim = dim3(kWThreads);
    cfg.dynamicSmemBytes = SmallSmem<AK>::kBytes;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = (unsigned)parts;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // as the prefill kernel (launch_pair)
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const cudaError_t e = y_dtype == SBQ_F16 ? launch_small<true, AK>(cfg, mx, mx2, mw, p)
                                             : launch_small<false, AK>(cfg, mx, mx2, mw, p);
    if (e != cudaSuccess) return set_error(SBQ_ERR_CUDA, "gemm_w8a16 (small batch) launch: %s", cudaGetErrorString(e));
    return check_launch("gemm_w8a16_small");
}

// Both GEMMs launch as programmatic dependents of the previous kernel on the stream: they set up,
// request their first weight tiles and convert them before griddepcontrol.wait, and touch
// activations and outputs only after it.  Only kernels that call griddepcontrol.launch_dependents
// let a dependent start early, and in this library those write activations only (never packed
// weights, scales or biases); any other predecessor completes first, as in plain stream order.
template <bool OUT_F16, bool GATED, int AK, int TOK>
static cudaError_t launch_pair(dim3 grid, cudaStream_t s, const CUtensorMap& mx, const CUtensorMap& mx2,
                               const CUtensorMap& mw, const GemmW16Params& p) {
    constexpr int smem = PairSmem<AK, TOK>::kBytes;
    cudaFuncSetAttribute(gemm_w8a16_pair_kernel<OUT_F16, GATED, AK, TOK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         smem);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kPThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gemm_w8a16_pair_kernel<OUT_F16, GATED, AK, TOK>, mx, mx2, mw, p);
}

// Token tile of the CTA-pair kernel: 256 unless the 256-token tiles fill less than ~90 % of one wave
// of pairs (one pair per two SMs) and 128-token tiles give more pairs - e.g. the reference's
// 512-token prefill chunks at n = 4096: 32 pairs of 256 tokens, 64 of 128.
static int pair_tok(int64_t m, int64_t n) {
    const int64_t cols = ceil_div(n, 2 * kWCh), pairs256 = cols * ceil_div(m, 256), pairs128 = cols * ceil_div(m, 128);
    const int64_t wave = sm_count_w16() / 2;
    return (pairs256 * 10 < wave * 9 && pairs128 > pairs256) ? 128 : 256;
}

// The CTA-pair kernel over 256-channel x TOK-token tiles (clusters of two CTAs along x).
template <int AK, int TOK>
static int gemm_pair(const CUtensorMap& mx, const CUtensorMap& mx2, const CUtensorMap& mw, const float* scale,
                     const float* bias, int64_t m, int64_t n, int64_t k, void* y, int y_dtype, int64_t ldy, void* stream,
                     int gated) {
    GemmW16Params p{};
    p.gated = gated;
    p.m = (int)m;
    p.n = (int)n;
    p.k = (int)k;
    p.num_kb = (int)ceil_div(k, kWBK * PairSmem<AK, TOK>::kKH);  // k columns past k read zeros (TMA fill)
    p.scale = scale;
    p.bias = bias;
    p.y = y;
    p.ldy = ldy;
    const dim3 grid((unsigned)(2 * ceil_div(n, 2 * kWCh)), (unsigned)ceil_div(m, TOK));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e;
    if (y_dtype == SBQ_F16) {
        e = gated ? launch_pair<true, true, AK, TOK>(grid, s, mx, mx2, mw, p)
                  : launch_pair<true, false, AK, TOK>(grid, s, mx, mx2, mw, p);
    } else {
        e = gated ? launch_pair<false, true, AK, TOK>(grid, s, mx, mx2, mw, p)
                  : launch_pair<false, false, AK, TOK>(grid, s, mx, mx2, mw, p);
    }
    if (e != cudaSuccess) return set_error(SBQ_ERR_CUDA, "gemm_w8a16 (CTA pairs) launch: %s", cudaGetErrorString(e));
    return check_launch("gemm_w8a16 (CTA pairs)");
}

template <int AK>
static int gemm_run_ak(const void* x, const void* x2, int64_t ldx, const void* packed, const float* scale,
                       const float* bias, int64_t m, int64_t n, int64_t k, void* y, int y_dtype, int64_t ldy, void* stream,
                       int gated) {
    const int tok = m <= kSmallMaxRows ? 0 : pair_tok(m, n);
    const int rows = m <= kSmallMaxRows ? kSTok : tok / 2;
    CUtensorMap mx, mx2, mw;
    int st = make_x_map(&mx, AK, x, ldx, m, k, rows);
    if (st) return st;
    if (AK == kABF16x2) {
        st = make_x_map(&mx2, AK, x2, ldx, m, k, rows);
        if (st) return st;
    } else {
        mx2 = mx;
    }
    st = make_w_map(&mw, packed, n, k);
    if (st) return st;
    if (m <= kSmallMaxRows) return gemm_small<AK>(mx, mx2, mw, scale, bias, m, n, k, y, y_dtype, ldy, stream, gated);
    if (tok == 128) return gemm_pair<AK, 128>(mx, mx2, mw, scale, bias, m, n, k, y, y_dtype, ldy, stream, gated);
    return gemm_pair<AK, 256>(mx, mx2, mw, scale, bias, m, n, k, y, y_dtype, ldy, stream, gated);
}

// ---- fp32 activation split: x = hi + lo, both bf16 -------------------------------------------------
// hi = bf16(x) (round to nearest even), lo = bf16(x - hi); x - hi is exact in fp32, so hi + lo keeps
// about 17 significant bits of x and its full exponent range.  Eight elements per thread.
__global__ void __launch_bounds__(256) split_bf16x2_kernel(const float* __restrict__ x, int64_t ldx, int64_t m,
                                                           int64_t k, __nv_bfloat16* __restrict__ hi,
                                                           __nv_bfloat16* __restrict__ lo, int64_t ldo) {
    const int64_t per_row = k / 8, total = m * per_row;
    for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < total; v += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = v / per_row, c = (v - row * per_row) * 8;
        const float4* src = reinterpret_cast<const float4*>(x + row * ldx + c);
        const float4 a = __ldg(src), b = __ldg(src + 1);
        const float f[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        uint32_t h[4], l[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const __nv_bfloat162 hh = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
            const float2 hf = __bfloat1622float2(hh);
            const __nv_bfloat162 ll = __floats2bfloat162_rn(f[2 * i] - hf.x, f[2 * i + 1] - hf.y);
            h[i] = *reinterpret_cast<const uint32_t*>(&hh);
            l[i] = *reinterpret_cast<const uint32_t*>(&ll);
        }
        *reinterpret_cast<uint4*>(hi + row * ldo + c) = make_uint4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<uint4*>(lo + row * ldo + c) = make_uint4(l[0], l[1], l[2], l[3]);
    }
}

static int launch_split(const float* x, int64_t ldx, int64_t m, int64_t k, void* hi, void* lo, int64_t ldo,
                        cudaStream_t s) {
    const int64_t vecs = m * (k / 8);
    int64_t blocks = (vecs + 255) / 256;
    const int64_t cap = (int64_t)sm_count_w16() * 8;
    if (blocks > cap) blocks = cap;
    split_bf16x2_kernel<<<(unsigned)(blocks < 1 ? 1 : blocks), 256, 0, s>>>(
        x, ldx, m, k, static_cast<__nv_bfloat16*>(hi), static_cast<__nv_bfloat16*>(lo), ldo);
    return check_launch("split_bf16x2");
}

static size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

namespace sbq {
// The tensor-memory GEMM of both tile sizes for fp16 or bf16 x; `gated`: see GemmW16Params
// (sbq_mlp_gateup_w8 runs the gate projection into h, then the up projection with gated = 1).
int gemm_w8a16_run(const void* x, int x_dtype, int64_t ldx, const void* packed, const float* scale, const float* bias,
                   int64_t m, int64_t n, int64_t k, void* y, int y_dtype, int64_t ldy, void* stream, int gated);
// The same for an fp32 x already split into bf16 hi / lo (row stride ldx each).
int gemm_w8a16_run_x2(const void* hi, const void* lo, int64_t ldx, const void* packed, const float* scale,
                      const float* bias, int64_t m, int64_t n, int64_t k, void* y, int y_dtype, int64_t ldy, void* stream,
                      int gated);
// Workspace of the fp32 path: hi then lo, [m, k] bf16 each.
size_t split_workspace_bytes(int64_t m, int64_t k);
int split_into_workspace(const void* x, int64_t ldx, int64_t m, int64_t k, void* workspace, size_t workspace_bytes,
                         void** hi, void** lo, void* stream);
}  // namespace sbq

size_t sbq::split_workspace_bytes(int64_t m, int64_t k) { return 2 * align256((size_t)(m * k * 2)); }

int sbq::split_into_workspace(const void* x, int64_t ldx, int64_t m, int64_t k, void* workspace, size_t workspace_bytes,
                              void** hi, void** lo, void* stream) {
    if (!workspace) return set_error(SBQ_ERR_INVALID_ARGUMENT, "fp32 activations need a workspace");
    if (reinterpret_cast<uintptr_t>(workspace) % 256) return set_error(SBQ_ERR_ALIGNMENT, "workspace must be 256-byte aligned");
    const size_t need = split_workspace_bytes(m, k);
    if (workspace_bytes < need) return set_error(SBQ_ERR_WORKSPACE, "workspace needs %zu bytes", need);
    *hi = workspace;
    *lo = static_cast<uint8_t*>(workspace) + need / 2;
    return launch_split(static_cast<const float*>(x), ldx, m, k, *hi, *lo, k, static_cast<cudaStream_t>(stream));
}

extern "C" int sbq_gemm_w8a16(const void* x, int x_dtype, int64_t ldx, const void* packed, const float* scale,
                              const float* bias, int64_t m, int64_t n, int64_t k, void* y, int y_dtype, int64_t ldy,
                              void* stream) {
    return gemm_w8a16_run(x, x_dtype, ldx, packed, scale, bias, m, n, k, y, y_dtype, ldy, stream, 0);
}

int sbq::gemm_w8a16_run(const void* x, int x_dtype, int64_t ldx, const void* packed, const float* scale,
                        const float* bias, int64_t m, int64_t n, int64_t k, void* y, int y_dtype, int64_t ldy,
                        void* stream, int gated) {
    int st = check_linear_args(x, x_dtype, ldx, packed, scale, m, n, k, y, y_dtype, ldy);
    if (st) return st;
    if (x_dtype == SBQ_F16)
        return gemm_run_ak<kAF16>(x, nullptr, ldx, packed, scale, bias, m, n, k, y, y_dtype, ldy, stream, gated);
    if (x_dtype == SBQ_BF16)
        return gemm_run_ak<kABF16>(x, nullptr, ldx, packed, scale, bias, m, n, k, y, y_dtype, ldy, stream, gated);
    return set_error(SBQ_ERR_UNSUPPORTED,
                     "sbq_gemm_w8a16 takes fp16 or bf16 activations (fp32: sbq_gemm_w8a16_x2 or sbq_linear_w8_ws)");
}

int sbq::gemm_w8a16_run_x2(const void* hi, const void* lo, int64_t ldx, const void* packed, const float* scale,
                           const float* bias, int64_t m, int64_t n, int64_t k, void* y, int y_dtype, int64_t ldy,
                           void* stream, int gated) {
    int st = check_linear_args(hi, SBQ_BF16, ldx, packed, scale, m, n, k, y, y_dtype, ldy);
    if (st) return st;
    if (!lo) return set_error(SBQ_ERR_INVALID_ARGUMENT, "null low part");
    if (reinterpret_cast<uintptr_t>(lo) % 16) return set_error(SBQ_ERR_ALIGNMENT, "activation rows must be 16-byte aligned");
    return gemm_run_ak<kABF16x2>(hi, lo, ldx, packed, scale, bias, m, n, k, y, y_dtype, ldy, stream, gated);
}

extern "C" int sbq_split_f32_bf16x2(const float* x, int64_t ldx, int64_t m, int64_t k, void* hi, void* lo,
                                    int64_t ldo, void* stream) {
    if (!x || !hi || !lo) return set_error(SBQ_ERR_INVALID_ARGUMENT, "null pointer");
    if (m <= 0 || k <= 0) return set_error(SBQ_ERR_INVALID_ARGUMENT, "m and k must be positive");
    if (k % 8) return set_error(SBQ_ERR_UNSUPPORTED, "k must be a multiple of 8 (k=%lld)", (long long)k);
    if (ldx < k || ldo < k) return set_error(SBQ_ERR_INVALID_ARGUMENT, "row stride smaller than the row");
    if (reinterpret_cast<uintptr_t>(x) % 16 || (ldx * 4) % 16 || reinterpret_cast<uintptr_t>(hi) % 16 ||
        reinterpret_cast<uintptr_t>(lo) % 16 || (ldo * 2) % 16)
        return set_error(SBQ_ERR_ALIGNMENT, "rows must be 16-byte aligned");
    return launch_split(x, ldx, m, k, hi, lo, ldo, static_cast<cudaStream_t>(stream));
}

extern "C" int sbq_gemm_w8a16_x2(const void* x_hi, const void* x_lo, int64_t ldx, const void* packed, const float* scale,
                                 const float* bias, int64_t m, int64_t n, int64_t k, void* y, int y_dtype, int64_t ldy,
                                 void* stream) {
    return gemm_w8a16_run_x2(x_hi, x_lo, ldx, packed, scale, bias, m, n, k, y, y_dtype, ldy, stream, 0);
}
