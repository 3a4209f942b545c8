// Decode GEMV for the int8 weight-only format (and the fused gate/up SwiGLU half of the MLP).
//
// Reference: Int8Linear.forward (spikingbrain_cpu/quant.py:41-53) at decode shapes (one token per
// call, engine.py:104-106) and GatedMLP.forward (model.py:239-240).  The reference dequantises
// each 128-row block of the weight to fp32 and runs an fp32 sgemm, then multiplies by the
// per-row scale.  Here the weight is streamed from HBM exactly once per launch:
//
//   * each CTA owns a run of consecutive 16-row tiles of one weight (sized so a launch has about
//     three CTAs per SM, each moving a similar number of bytes); a producer warp streams that
//     contiguous byte range with cp.async.bulk copies into a 40 KiB shared-memory ring (8 KiB
//     chunks, mbarrier transaction counts), across tile boundaries without pausing;
//   * the consumers copy x into shared memory once (when m * k fits in 26 KiB), so the chunk
//     loop reads its activation fragments from shared memory instead of waiting on L2;
//   * eight consumer warps (or four on gate and four on up) take one 1 KiB tile of each chunk:
//     two conflict-free 16-byte shared loads per lane, int8 -> fp16 (or bf16) in registers (exact), m16n8k16 tensor-core MMAs with
//     fp32 accumulation and the activation rows as the n dimension (8 or 16 tokens per pass);
//   * at the end of each tile the warps' partial sums are reduced through shared memory in a fixed
//     order, then the fp32 per-row scale (and bias, or the SiLU(gate) * up product) is applied
//     before one store, while the producer keeps streaming the next tile;
//   * one launch can carry several independent projections ("jobs": e.g. q|k|v|delta_in and
//     gate/up of one layer, which read the same x); each CTA finds its job from its block index;
//   * programmatic dependent launch: the weights never depend on the previous kernel, so the
//     producer starts streaming at once; only the consumers wait (griddepcontrol.wait) before
//     reading x, and each CTA releases the next launch as soon as it starts.
//
// fp32 activations are split into a bf16 high and low part (two MMAs, ~16 mantissa bits kept);
// the dot product of int8 weights and fp16/bf16 activations is exact up to fp32 accumulation.
#include <cmath>
#include <vector>

#include "tc.cuh"

namespace sbq {

enum XKind { kXF16 = 0, kXBF16 = 1, kXF32 = 2 };

// One projection of a launch.
struct GemvJob {
    const void* x;     // activation [m, k], 16-byte aligned rows
    int64_t ldx;
    const int8_t* w0;  // packed weight (gate for a fused gate/up job)
    const float* s0;
    const int8_t* w1;  // packed up weight (fused job only, else null)
    const float* s1;
    const float* bias;
    void* y;
    int64_t ldy;
    int m;             // rows of x handled by this launch (<= 8 * MT)
    int n;
    int k;
    int kt_total;      // ceil(k / 64)
    int chunk_tiles;   // tiles per chunk and matrix: the largest of 8 (4 for gate/up), 4, 2, 1 dividing kt_total
    int out_f16;       // 1: fp16 output, 0: fp32
    int n_tiles;       // 16-row tiles of the weight
    int tiles_per_cta; // consecutive tiles one CTA streams
    int cta_begin;     // first block index of this job in the grid
};

constexpr int kMaxJobs = 8;

struct GemvGroup {
    GemvJob job[kMaxJobs];
    int njobs;
};

// Output-channel shards on several GPUs of one node (sbq_gemv_w8_group_peer).  Every rank computes
// its slice of each job's output and stores it straight into every rank's full-width buffer over
// NVLink (peer pointers).  The CTAs of a launch count themselves out on a local counter; the last
// one adds 1 to this launch's signal on every rank.  A launch that reads such outputs first waits
// (bounded) until its local copy of the producing launch's signal has received one increment per
// rank for this step.  Signals are kept in kSignalCopies copies 128 bytes apart (the last CTA's
// warp writes all of them at once) so that the CTAs of the waiting launch poll different L2 lines.
constexpr int kMaxPeers = 8;
constexpr int kSignalCopies = SBQ_PEER_SIGNAL_COPIES;
constexpr int kSignalStride = 32;  // u32 words between copies
static_assert(kSignalCopies == 32, "one warp writes the signal copies");

struct PeerSync {
    void* y[kMaxJobs][kMaxPeers];  // job j's output slice as mapped on rank p (same ldy as the job)
    unsigned* signal[kMaxPeers];   // this launch's signal copies on rank p
    unsigned* done;                // local: CTAs of this launch that have published their stores
    const unsigned* wait_count;    // local signal copies of the launch whose outputs x comes from, or null
    unsigned* wait_state;          // [generation, arrivals] of this launch's wait (local)
    unsigned wait_expected;        // increments a signal copy receives per step (one per rank)
    int nranks;
};

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_add_sys(unsigned* p, unsigned v) {
    asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// One thread per CTA: waits until its copy of the signal has received this step's `expected`
// increments (targets grow by `expected` per step; state[0] counts completed steps of this
// waiter), then records the CTA's arrival; the last CTA of the grid advances the generation for
// the next step.  Bounded (ranks may drift apart on the host by up to kPeerWaitLimitNs): on expiry
// the error word is set and the kernel carries on (its outputs are then invalid, the host sees
// SBQ_ERR_TIMEOUT); after an earlier failure it does not wait at all.
constexpr uint64_t kPeerWaitLimitNs = 10000000000ull;

__device__ __forceinline__ void peer_wait(const unsigned* signal, unsigned* state, unsigned expected) {
    const unsigned* count = signal + (blockIdx.x % kSignalCopies) * kSignalStride;
    const unsigned gen = *reinterpret_cast<volatile unsigned*>(state);
    const unsigned target = (gen + 1u) * expected;
    if (*reinterpret_cast<volatile int*>(&g_device_error) == 0 && (int)(ld_acquire_sys(count) - target) < 0) {
        const uint64_t t0 = tc::now_ns();
        for (uint32_t i = 1; (int)(ld_acquire_sys(count) - target) < 0; ++i) {
            __nanosleep(64);
            if ((i & 63) == 0 && tc::now_ns() - t0 > kPeerWaitLimitNs) {
                tc::raise_error(SBQ_ERR_TIMEOUT);
                break;
            }
        }
    }
    if (atomicAdd(state + 1, 1u) == gridDim.x - 1) {
        state[1] = 0;
        __threadfence();
        atomicAdd(state, 1u);
    }
}

// Warp 0 of every CTA, after the consumers' barrier that follows their last output stores.
// Ordering: the barrier orders every consumer's (local and peer) output stores before lane 0's
// GPU-scope release (fence + count-out); the last CTA's count-out reads the whole release sequence,
// and its system-scope fence is cumulative, so all CTAs' stores are ordered before the signal the
// other ranks acquire.  One system-scope fence per launch: a per-CTA system fence measured about
// 8 us per launch on B200.
__device__ __forceinline__ void peer_publish(const PeerSync& ps, int lane) {
    unsigned last = 0;
    if (lane == 0) {
        __threadfence();
        last = atomicAdd(ps.done, 1u) == gridDim.x - 1;
        if (last) *ps.done = 0;  // next used by this launch position of the next step
    }
    __syncwarp();
    last = __shfl_sync(0xffffffffu, last, 0);
    if (last) {
        __threadfence_system();
        for (int p = 0; p < ps.nranks; ++p) red_add_sys(ps.signal[p] + lane * kSignalStride, 1u);
    }
}

constexpr int kGemvWarps = 8;  // consumer warps

template <int XK>
struct XFrag {
    uint32_t b[4][2];      // fp16 / bf16 main part
    uint32_t blo[4][2];    // bf16 low part (fp32 input only)
};

// Loads the 16 activation values lane (g, c) needs for k0 .. k0 + 15 of row `row` as MMA B fragments
// b[s][0..1] (s = the four k16 steps).  Rows beyond m (or spans beyond k) read as zero.
// `coh`: x is in global memory and was written by other GPUs during this launch (L2-only loads).
template <int XK>
__device__ __forceinline__ void load_x(XFrag<XK>& f, const void* xv, int64_t ldx, int row, int m, int64_t k0, int k,
                                       bool coh = false) {
    const uint8_t* x = static_cast<const uint8_t*>(xv);
    const bool ok = row < m && k0 < k;
    if (XK == kXF16 || XK == kXBF16) {
        uint4 v0 = make_uint4(0, 0, 0, 0), v1 = v0;
        if (ok) {
            const uint4* q = reinterpret_cast<const uint4*>(x + ((int64_t)row * ldx + k0) * 2);
            v0 = coh ? __ldcg(q) : q[0];
            v1 = coh ? __ldcg(q + 1) : q[1];
        }
        f.b[0][0] = v0.x; f.b[0][1] = v0.y; f.b[1][0] = v0.z; f.b[1][1] = v0.w;
        f.b[2][0] = v1.x; f.b[2][1] = v1.y; f.b[3][0] = v1.z; f.b[3][1] = v1.w;
    } else {
        float v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = 0.0f;
        if (ok) {
            const uint4* q = reinterpret_cast<const uint4*>(x + ((int64_t)row * ldx + k0) * 4);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint4 t = coh ? __ldcg(q + i) : q[i];
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

constexpr int kGemvThreads = (kGemvWarps + 1) * 32;  // 8 consumer warps + 1 producer warp
constexpr int kChunkTiles = 8;                         // tiles (KiB) per chunk and matrix, at most
constexpr int kRingBytes = 40 * 1024;                  // 5 stages of 8 KiB (8 tiles, or 4 gate + 4 up tiles)
constexpr int kMaxStages = 5;
constexpr int kXBytes = 25 * 1024 + 512;               // x staged in shared memory when it fits (m * (k + 8) * es)
template <int MT>
struct GemvSmemSize {
    static constexpr int kRed = kGemvWarps * MT * 16 * 9 * 4;  // per-warp partial sums of one tile
    static constexpr int kBytes = kRingBytes + kXBytes + kRed + 2 * kMaxStages * 8;  // 3 CTAs per SM at MT = 1
};
constexpr int kCtasPerSm = 3;  // CTAs a launch is sized for (three fit per SM)

// Named barrier 1 over the consumer warps.
__device__ __forceinline__ void consumers_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kGemvWarps * 32) : "memory");
}

// Named barrier 1 over the consumer warps with an AND of `v` across them.
__device__ __forceinline__ int consumers_sync_and(int v) {
    int r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.s32 p, %1, 0;\n\t"
        "bar.red.and.pred q, 1, %2, p;\n\t"
        "selp.s32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(v), "n"(kGemvWarps * 32)
        : "memory");
    return r;
}

// A CTA's work on one job is a run of consecutive 16-row tiles [t0, t1): a contiguous byte range of
// the packed weight (and of the up weight when NMAT = 2).  A chunk holds C tiles of each matrix; the
// consumer warps are split evenly over the matrices (8 over one, or 4 on gate and 4 on up), each
// warp taking one tile of its matrix per chunk.  `ci` counts chunks through the ring across runs,
// so a CTA can stream several runs back to back (the decode program kernel does).

// Producer (one thread): streams the run's chunks.  False if a wait timed out.
template <int NMAT>
__device__ __forceinline__ bool produce_run(const GemvJob& jb, int t0, int t1, uint8_t* ring, uint64_t* full,
                                            uint64_t* empty, uint32_t& ci) {
    constexpr int S = kMaxStages;
    constexpr int kStageBytes = kChunkTiles * kTileBytes;
    const int C = jb.chunk_tiles;
    const int nchunks = (t1 - t0) * (jb.kt_total / C);
    const uint32_t bytes = (uint32_t)C * kTileBytes;
    const int8_t* src0 = jb.w0 + (int64_t)t0 * jb.kt_total * kTileBytes;
    const int8_t* src1 = NMAT == 2 ? jb.w1 + (int64_t)t0 * jb.kt_total * kTileBytes : nullptr;
    for (int i = 0; i < nchunks; ++i, ++ci) {
        const int s = ci % S;
        if (!tc::mbar_wait(&empty[s], ((ci / S) & 1) ^ 1)) return false;
        uint8_t* dst = ring + s * kStageBytes;
        tc::mbar_arrive_expect_tx(&full[s], bytes * NMAT);
        tc::bulk_load(dst, src0 + (int64_t)i * bytes, bytes, &full[s]);
        if (NMAT == 2) tc::bulk_load(dst + bytes, src1 + (int64_t)i * bytes, bytes, &full[s]);
    }
    return true;
}

// Consumers: copy x into shared memory when it fits (m * (k + 8) elements), else read it in place.
// `coherent` loads bypass L1 (x written earlier in the same kernel by other SMs).
template <int XK>
__device__ __forceinline__ void stage_x(const GemvJob& jb, uint8_t* xs, bool coherent, const void*& xsrc,
                                        int64_t& xld) {
    constexpr int es = XK == kXF32 ? 4 : 2;
    const int xrow = jb.k * es + 16;  // bytes per staged row (+16 against bank conflicts)
    xsrc = jb.x;
    xld = jb.ldx;
    if (jb.m * xrow <= kXBytes) {
        const int vpr = jb.k * es / 16;
        for (int v = threadIdx.x; v < jb.m * vpr; v += kGemvWarps * 32) {
            const int r = v / vpr, cc = v - r * vpr;
            const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(jb.x) +
                                                              (int64_t)r * jb.ldx * es + cc * 16);
            *reinterpret_cast<uint4*>(xs + r * xrow + cc * 16) = coherent ? __ldcg(src) : *src;
        }
        consumers_sync();
        xsrc = xs;
        xld = xrow / es;
    }
}

// Consumers (8 warps): the run's chunks, a fixed-order reduction and the epilogue per tile.
// Returns false (warp-uniformly) if a wait timed out.
// PEER: every output is stored to each rank's copy (ps->y[jidx][p]) instead of jb.y.
template <int XK, int MT, int NMAT, bool PEER = false>
__device__ __forceinline__ bool consume_run(const GemvJob& jb, int t0, int t1, const void* xsrc, int64_t xld,
                                            uint8_t* ring, float* red, uint64_t* full, uint64_t* empty,
                                            uint32_t& ci, const PeerSync* ps = nullptr, int jidx = 0,
                                            bool xcoh = false) {
    constexpr int S = kMaxStages;
    constexpr int kStageBytes = kChunkTiles * kTileBytes;  // 8 KiB: C tiles of each of the NMAT matrices
    constexpr int WPM = kGemvWarps / NMAT;                   // warps per matrix
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int C = jb.chunk_tiles;                            // tiles per chunk and matrix (<= WPM)
    const int cpt = jb.kt_total / C;                         // chunks per tile
    const int nchunks = (t1 - t0) * cpt;
    const int g = lane >> 2, c = lane & 3;
    const int mat = warp / WPM, slot = warp % WPM;  // this warp's matrix and tile within a chunk
    const bool mine = slot < C;
    const int mat_off = mat * C * kTileBytes;
    float acc[MT][4];
    for (int i = 0, j = 0; i < nchunks; ++i, ++ci) {
        if (j == 0) {
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[mt][e] = 0.0f;
        }
        const int s = ci % S;
        XFrag<XK> xf[MT];
        if (mine) {
            const int64_t k0 = (int64_t)(j * C + slot) * kTileCols + 16 * c;
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) load_x<XK>(xf[mt], xsrc, xld, 8 * mt + g, jb.m, k0, jb.k, xcoh);
        }
        // warp-uniform wait (the __syncwarp below must see every lane)
        if (!__all_sync(0xffffffffu, tc::mbar_wait(&full[s], (ci / S) & 1))) return false;
        if (mine) {
            const uint8_t* t = ring + s * kStageBytes + mat_off + slot * kTileBytes + lane * 16;
            const uint4 wa = *reinterpret_cast<const uint4*>(t);
            const uint4 wb = *reinterpret_cast<const uint4*>(t + 512);
            tile_mma<XK, MT>(acc, wa, wb, xf);
        }
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&empty[s]);
        if (++j < cpt) continue;
        j = 0;

        // ---- tile complete: reduce the warps' partial sums (fixed order), scale, store
        const int nt = t0 + i / cpt;
#define SBQ_RED(w, mt, r, col) red[(((w) * MT + (mt)) * 16 + (r)) * 9 + (col)]
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            SBQ_RED(warp, mt, g, 2 * c) = acc[mt][0];
            SBQ_RED(warp, mt, g, 2 * c + 1) = acc[mt][1];
            SBQ_RED(warp, mt, g + 8, 2 * c) = acc[mt][2];
            SBQ_RED(warp, mt, g + 8, 2 * c + 1) = acc[mt][3];
        }
        consumers_sync();
        for (int t = threadIdx.x; t < MT * 8 * 16; t += kGemvWarps * 32) {
            const int r = t & 15, tok = t >> 4, mt = tok >> 3, col = tok & 7;
            const int n = nt * 16 + r;
            if (n >= jb.n || tok >= jb.m) continue;
            float v[NMAT];
#pragma unroll
            for (int a = 0; a < NMAT; ++a) {
                float sum = 0.0f;
#pragma unroll
                for (int w = 0; w < WPM; ++w) sum += SBQ_RED(a * WPM + w, mt, r, col);
                v[a] = sum;
            }
            float out;
            if (NMAT == 1) {
                out = v[0] * jb.s0[n];
                if (jb.bias) out += jb.bias[n];
            } else {
                const float gv = v[0] * jb.s0[n];
                const float uv = v[1] * jb.s1[n];
                out = gv / (1.0f + expf(-gv)) * uv;
            }
            const int64_t idx = (int64_t)tok * jb.ldy + n;
            if (PEER) {
                // consecutive threads store consecutive rows: one coalesced NVLink write per rank
                for (int p = 0; p < ps->nranks; ++p) {
                    if (jb.out_f16)
                        static_cast<__half*>(ps->y[jidx][p])[idx] = __float2half_rn(out);
                    else
                        static_cast<float*>(ps->y[jidx][p])[idx] = out;
                }
            } else if (jb.out_f16) {
                static_cast<__half*>(jb.y)[idx] = __float2half_rn(out);
            } else {
                static_cast<float*>(jb.y)[idx] = out;
            }
        }
#undef SBQ_RED
        consumers_sync();  // red is rewritten by the next tile
    }
    return true;
}

template <int XK, int MT, int NMAT, bool PEER>
__device__ __forceinline__ void gemv_tiles(const GemvJob& jb, int t0, int t1, uint8_t* ring, uint8_t* xs, float* red,
                                           uint64_t* full, uint64_t* empty, const PeerSync& ps, int jidx) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint32_t ci = 0;
    if (warp == kGemvWarps) {
        if (lane == 0) produce_run<NMAT>(jb, t0, t1, ring, full, empty, ci);
        return;
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");  // x is the previous kernel's output
    if (PEER && ps.wait_count) {
        // x also holds the other ranks' slices, stored by their previous launch
        if (threadIdx.x == 0) peer_wait(ps.wait_count, ps.wait_state, ps.wait_expected);
        consumers_sync();
    }
    const void* xsrc;
    int64_t xld;
    stage_x<XK>(jb, xs, PEER, xsrc, xld);
    const bool staged = xsrc != jb.x;
    const bool ok =
        consume_run<XK, MT, NMAT, PEER>(jb, t0, t1, xsrc, xld, ring, red, full, empty, ci, &ps, jidx, PEER && !staged);
    if (!consumers_sync_and(ok) && threadIdx.x == 0) tc::raise_error(SBQ_ERR_TIMEOUT);
    if (PEER) {
        // publish (also after a timeout, so that the other ranks do not wait in vain)
        consumers_sync();
        if (warp == 0) peer_publish(ps, lane);
    }
}

template <int XK, int MT, bool PEER>
__global__ void __launch_bounds__(kGemvThreads, MT == 1 ? 3 : 2)
    gemv_w8_kernel(const __grid_constant__ GemvGroup grp, const __grid_constant__ PeerSync ps) {
    extern __shared__ __align__(128) uint8_t ring[];
    uint8_t* xs = ring + kRingBytes;
    float* red = reinterpret_cast<float*>(xs + kXBytes);
    uint64_t* full = reinterpret_cast<uint64_t*>(xs + kXBytes + GemvSmemSize<MT>::kRed);
    uint64_t* empty = full + kMaxStages;
    int j = 0;
    while (j + 1 < grp.njobs && (int)blockIdx.x >= grp.job[j + 1].cta_begin) ++j;
    const GemvJob& jb = grp.job[j];
    const int nmat = jb.w1 ? 2 : 1;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kMaxStages; ++i) {
            tc::mbar_init(&full[i], 1);
            tc::mbar_init(&empty[i], kGemvWarps);
        }
        tc::fence_mbar_init();
    }
    __syncthreads();
    // the next launch may start its own weight stream now (it waits for this grid before reading x)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int t0 = ((int)blockIdx.x - jb.cta_begin) * jb.tiles_per_cta;
    const int t1 = min(t0 + jb.tiles_per_cta, jb.n_tiles);
    if (nmat == 2)
        gemv_tiles<XK, MT, 2, PEER>(jb, t0, t1, ring, xs, red, full, empty, ps, j);
    else
        gemv_tiles<XK, MT, 1, PEER>(jb, t0, t1, ring, xs, red, full, empty, ps, j);
}

// Waits (one CTA) for a peer launch's outputs: the end of a sharded decode step, before the host
// or another stream reads the gathered result.
__global__ void peer_wait_kernel(const unsigned* count, unsigned* state, unsigned expected) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (threadIdx.x == 0) peer_wait(count, state, expected);
}

// ---------------------------------------------------------------------------------------------
// Decode program: a whole sequence of grouped stages in one persistent cooperative launch.
//
// Stage s may read what stages < s wrote.  Every CTA owns at most one run per stage; when its
// consumers finish that run (or have none) they publish with a fence and an atomic increment of
// counters[s]; before stage s + 1 a CTA's consumers wait until counters[s] equals the grid size.
// The producer never waits on a stage: it streams the next stages' weights (which depend on
// nothing) as fast as the ring drains, so HBM stays busy across the barriers.  All CTAs are
// co-resident (cooperative launch), every wait is bounded, and activations are read with L2-only
// loads (they were written during this launch by other SMs).
// ---------------------------------------------------------------------------------------------
struct ProgItem {
    int job;
    int t0;
    int t1;
};

struct ProgStage {
    GemvJob job[kMaxJobs];
    int njobs;
    int pad;
};

struct ProgParams {
    const ProgStage* stages;
    const ProgItem* items;  // [stage][cta]
    int nstages;
    int* counters;          // [stage], zero at launch
};

__device__ __forceinline__ int ld_acquire(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

template <int XK>
__global__ void __launch_bounds__(kGemvThreads, 3) gemv_program_kernel(const ProgParams p) {
    constexpr int MT = 1;
    extern __shared__ __align__(128) uint8_t ring[];
    uint8_t* xs = ring + kRingBytes;
    float* red = reinterpret_cast<float*>(xs + kXBytes);
    uint64_t* full = reinterpret_cast<uint64_t*>(xs + kXBytes + GemvSmemSize<MT>::kRed);
    uint64_t* empty = full + kMaxStages;
    __shared__ int abort_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nctas = gridDim.x, cta = blockIdx.x;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kMaxStages; ++i) {
            tc::mbar_init(&full[i], 1);
            tc::mbar_init(&empty[i], kGemvWarps);
        }
        tc::fence_mbar_init();
        abort_flag = 0;
    }
    __syncthreads();
    uint32_t ci = 0;
    if (warp == kGemvWarps) {
        if (lane == 0) {
            for (int st = 0; st < p.nstages; ++st) {
                const ProgItem it = p.items[(int64_t)st * nctas + cta];
                if (it.t1 <= it.t0) continue;
                const GemvJob jb = p.stages[st].job[it.job];
                const bool ok = jb.w1 ? produce_run<2>(jb, it.t0, it.t1, ring, full, empty, ci)
                                      : produce_run<1>(jb, it.t0, it.t1, ring, full, empty, ci);
                if (!ok) break;
            }
        }
        return;
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");  // the first stage's x comes from the previous kernel
    for (int st = 0; st < p.nstages; ++st) {
        if (st > 0) {
            if (threadIdx.x == 0) {
                const int* ctr = p.counters + (st - 1);
                if (ld_acquire(ctr) < nctas) {
                    const uint64_t t0 = tc::now_ns();
                    for (uint32_t i = 1; ld_acquire(ctr) < nctas; ++i) {
                        if ((i & 63) == 0 && tc::now_ns() - t0 > tc::kWaitLimitNs) {
                            tc::raise_error(SBQ_ERR_TIMEOUT);
                            abort_flag = 1;
                            break;
                        }
                    }
                }
            }
            consumers_sync();
            if (abort_flag) return;
        }
        const ProgItem it = p.items[(int64_t)st * nctas + cta];
        if (it.t1 > it.t0) {
            const GemvJob jb = p.stages[st].job[it.job];
            const void* xsrc;
            int64_t xld;
            stage_x<XK>(jb, xs, true, xsrc, xld);
            const bool ok = jb.w1 ? consume_run<XK, MT, 2>(jb, it.t0, it.t1, xsrc, xld, ring, red, full, empty, ci)
                                  : consume_run<XK, MT, 1>(jb, it.t0, it.t1, xsrc, xld, ring, red, full, empty, ci);
            if (!ok) {
                if (lane == 0) tc::raise_error(SBQ_ERR_TIMEOUT);
                abort_flag = 1;
            }
        }
        // publish this CTA's part of stage st: every consumer's stores precede the barrier, the fence
        // of the publishing thread orders them before its increment
        consumers_sync();
        if (abort_flag) return;
        if (threadIdx.x == 0) {
            __threadfence();
            atomicAdd(p.counters + st, 1);
        }
    }
}

template <int XK, int MT, bool PEER>
static void launch_group(const GemvGroup& grp, const PeerSync& ps, int total_ctas, cudaStream_t s) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)total_ctas);
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = GemvSmemSize<MT>::kBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaFuncSetAttribute(gemv_w8_kernel<XK, MT, PEER>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         GemvSmemSize<MT>::kBytes);
    cudaLaunchKernelEx(&cfg, gemv_w8_kernel<XK, MT, PEER>, grp, ps);
}

static int sm_count() {
    static int count[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!count[dev]) {
        int c = 0;
        cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev);
        count[dev] = c > 0 ? c : 148;
    }
    return count[dev];
}

// Splits every job into runs of consecutive tiles so that the launch has about kCtasPerSm CTAs per
// SM, each streaming a similar number of weight bytes.  Returns the number of CTAs.
static int plan_group(GemvGroup& grp) {
    double total = 0.0;
    for (int i = 0; i < grp.njobs; ++i) {
        GemvJob& j = grp.job[i];
        j.n_tiles = (int)ceil_div(j.n, 16);
        total += (double)j.n_tiles * (j.w1 ? 2 : 1) * j.kt_total * kTileBytes;
    }
    const double target = total / (double)(kCtasPerSm * sm_count());
    int ctas = 0;
    for (int i = 0; i < grp.njobs; ++i) {
        GemvJob& j = grp.job[i];
        const double tile_bytes = (double)(j.w1 ? 2 : 1) * j.kt_total * kTileBytes;
        int t = (int)(target / tile_bytes + 0.5);
        j.tiles_per_cta = t < 1 ? 1 : (t > j.n_tiles ? j.n_tiles : t);
        j.cta_begin = ctas;
        ctas += (int)ceil_div(j.n_tiles, j.tiles_per_cta);
    }
    return ctas;
}

template <bool PEER>
static void dispatch_group_t(GemvGroup& grp, const PeerSync& ps, int xk, int mt, cudaStream_t s) {
    const int ctas = plan_group(grp);
    switch (xk) {
        case kXF16:
            mt == 2 ? launch_group<kXF16, 2, PEER>(grp, ps, ctas, s) : launch_group<kXF16, 1, PEER>(grp, ps, ctas, s);
            break;
        case kXBF16:
            mt == 2 ? launch_group<kXBF16, 2, PEER>(grp, ps, ctas, s) : launch_group<kXBF16, 1, PEER>(grp, ps, ctas, s);
            break;
        default:
            mt == 2 ? launch_group<kXF32, 2, PEER>(grp, ps, ctas, s) : launch_group<kXF32, 1, PEER>(grp, ps, ctas, s);
            break;
    }
}

static void dispatch_group(GemvGroup& grp, int xk, int mt, cudaStream_t s) {
    const PeerSync none{};
    dispatch_group_t<false>(grp, none, xk, mt, s);
}

SBQ_DEFINE_ERROR_POLL(poll_error_gemv)

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

static void fill_job(GemvJob& jb, const void* x, int64_t ldx, const void* w0, const float* s0, const void* w1,
                     const float* s1, const float* bias, int64_t n, int64_t k, void* y, int y_dtype, int64_t ldy) {
    jb = GemvJob{};
    jb.x = x;
    jb.ldx = ldx;
    jb.w0 = static_cast<const int8_t*>(w0);
    jb.s0 = s0;
    jb.w1 = static_cast<const int8_t*>(w1);
    jb.s1 = s1;
    jb.bias = bias;
    jb.y = y;
    jb.ldy = ldy;
    jb.n = (int)n;
    jb.k = (int)k;
    jb.kt_total = (int)ceil_div(k, kTileCols);
    const int cmax = w1 ? 4 : 8;  // a chunk is 8 KiB: 8 tiles of one matrix or 4 of each of two
    jb.chunk_tiles = jb.kt_total % cmax == 0 ? cmax : jb.kt_total % 4 == 0 ? 4 : jb.kt_total % 2 == 0 ? 2 : 1;
    jb.out_f16 = y_dtype == SBQ_F16;
}

// One job over all rows of x, in passes of 16 rows (each pass streams the weight once).
static int run_single(GemvJob jb, int64_t m, int x_dtype, int y_dtype, cudaStream_t s, const char* what) {
    const int xs = elem_size(x_dtype), ys = y_dtype == SBQ_F32 ? 4 : 2;
    GemvGroup grp{};
    grp.njobs = 1;
    for (int64_t m0 = 0; m0 < m; m0 += 16) {
        GemvJob q = jb;
        q.m = (int)(m - m0 < 16 ? m - m0 : 16);
        q.x = static_cast<const char*>(jb.x) + m0 * jb.ldx * xs;
        q.y = static_cast<char*>(jb.y) + m0 * jb.ldy * ys;
        grp.job[0] = q;
        dispatch_group(grp, x_kind(x_dtype), q.m > 8 ? 2 : 1, s);
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
    GemvJob jb;
    fill_job(jb, x, ldx, packed, scale, nullptr, nullptr, bias, n, k, y, y_dtype, ldy);
    return run_single(jb, m, x_dtype, y_dtype, static_cast<cudaStream_t>(stream), "gemv_w8");
}

extern "C" int sbq_mlp_gateup_w8(const void* x, int x_dtype, int64_t ldx, const void* packed_gate,
                                 const float* scale_gate, const void* packed_up, const float* scale_up, int64_t m,
                                 int64_t n, int64_t k, void* h, int h_dtype, int64_t ldh, void* stream) {
    int st = check_linear_args(x, x_dtype, ldx, packed_gate, scale_gate, m, n, k, h, h_dtype, ldh);
    if (st) return st;
    if (!packed_up || !scale_up) return set_error(SBQ_ERR_INVALID_ARGUMENT, "null up-projection pointer");
    if (reinterpret_cast<uintptr_t>(packed_up) % 256) return set_error(SBQ_ERR_ALIGNMENT, "packed weight must be 256-byte aligned");
    GemvJob jb;
    fill_job(jb, x, ldx, packed_gate, scale_gate, packed_up, scale_up, nullptr, n, k, h, h_dtype, ldh);
    return run_single(jb, m, x_dtype, h_dtype, static_cast<cudaStream_t>(stream), "mlp_gateup_w8");
}

extern "C" int sbq_gemv_w8_group(const sbq_gemv_job* jobs, int njobs, int x_dtype, int64_t m, void* stream) {
    if (!jobs || njobs < 1 || njobs > kMaxJobs)
        return set_error(SBQ_ERR_INVALID_ARGUMENT, "njobs must be 1..%d", kMaxJobs);
    if (m < 1 || m > 16) return set_error(SBQ_ERR_UNSUPPORTED, "a grouped launch takes 1..16 rows of x (m=%lld)", (long long)m);
    GemvGroup grp{};
    grp.njobs = njobs;
    for (int i = 0; i < njobs; ++i) {
        const sbq_gemv_job& j = jobs[i];
        int st = check_linear_args(j.x, x_dtype, j.ldx, j.packed, j.scale, m, j.n, j.k, j.y, j.y_dtype, j.ldy);
        if (st) return set_error(st, "job %d: %s", i, sbq_last_error());
        if (j.packed_up) {
            if (!j.scale_up) return set_error(SBQ_ERR_INVALID_ARGUMENT, "job %d: null up-projection scale", i);
            if (reinterpret_cast<uintptr_t>(j.packed_up) % 256)
                return set_error(SBQ_ERR_ALIGNMENT, "job %d: packed weight must be 256-byte aligned", i);
            if (j.bias) return set_error(SBQ_ERR_UNSUPPORTED, "job %d: a fused gate/up job takes no bias", i);
        }
        fill_job(grp.job[i], j.x, j.ldx, j.packed, j.scale, j.packed_up, j.scale_up, j.bias, j.n, j.k, j.y, j.y_dtype,
                 j.ldy);
        grp.job[i].m = (int)m;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    dispatch_group(grp, x_kind(x_dtype), m > 8 ? 2 : 1, s);
    return check_launch("gemv_w8_group");
}

extern "C" int sbq_gemv_w8_group_peer(const sbq_gemv_job* jobs, int njobs, int x_dtype, int64_t m,
                                      const sbq_peer_group* peers, void* stream) {
    if (!peers) return set_error(SBQ_ERR_INVALID_ARGUMENT, "null peer description");
    if (!jobs || njobs < 1 || njobs > kMaxJobs)
        return set_error(SBQ_ERR_INVALID_ARGUMENT, "njobs must be 1..%d", kMaxJobs);
    if (m < 1 || m > 16) return set_error(SBQ_ERR_UNSUPPORTED, "a grouped launch takes 1..16 rows of x (m=%lld)", (long long)m);
    const sbq_peer_group& pg = *peers;
    if (pg.nranks < 1 || pg.nranks > kMaxPeers)
        return set_error(SBQ_ERR_INVALID_ARGUMENT, "nranks must be 1..%d (got %d)", kMaxPeers, pg.nranks);
    if (pg.wait_count && (!pg.wait_state || pg.wait_expected == 0))
        return set_error(SBQ_ERR_INVALID_ARGUMENT, "a wait needs wait_state and a positive wait_expected");
    if (reinterpret_cast<uintptr_t>(pg.wait_count) % 128 || reinterpret_cast<uintptr_t>(pg.wait_state) % 8)
        return set_error(SBQ_ERR_ALIGNMENT, "wait signal must be 128-byte and wait state 8-byte aligned");
    if (!pg.done || reinterpret_cast<uintptr_t>(pg.done) % 4)
        return set_error(SBQ_ERR_INVALID_ARGUMENT, "done must be a 4-byte aligned device pointer");
    PeerSync ps{};
    ps.nranks = pg.nranks;
    ps.done = pg.done;
    ps.wait_count = pg.wait_count;
    ps.wait_state = pg.wait_state;
    ps.wait_expected = pg.wait_expected;
    for (int p = 0; p < pg.nranks; ++p) {
        if (!pg.signal[p] || reinterpret_cast<uintptr_t>(pg.signal[p]) % 128)
            return set_error(SBQ_ERR_INVALID_ARGUMENT, "signal[%d] must be a 128-byte aligned device pointer", p);
        ps.signal[p] = pg.signal[p];
    }
    GemvGroup grp{};
    grp.njobs = njobs;
    for (int i = 0; i < njobs; ++i) {
        const sbq_gemv_job& j = jobs[i];
        int st = check_linear_args(j.x, x_dtype, j.ldx, j.packed, j.scale, m, j.n, j.k, j.y, j.y_dtype, j.ldy);
        if (st) return set_error(st, "job %d: %s", i, sbq_last_error());
        if (j.packed_up) {
            if (!j.scale_up) return set_error(SBQ_ERR_INVALID_ARGUMENT, "job %d: null up-projection scale", i);
            if (reinterpret_cast<uintptr_t>(j.packed_up) % 256)
                return set_error(SBQ_ERR_ALIGNMENT, "job %d: packed weight must be 256-byte aligned", i);
            if (j.bias) return set_error(SBQ_ERR_UNSUPPORTED, "job %d: a fused gate/up job takes no bias", i);
        }
        bool local = false;
        for (int p = 0; p < pg.nranks; ++p) {
            if (!pg.y[i][p]) return set_error(SBQ_ERR_INVALID_ARGUMENT, "job %d: null destination for rank %d", i, p);
            local = local || pg.y[i][p] == j.y;
            ps.y[i][p] = pg.y[i][p];
        }
        if (!local) return set_error(SBQ_ERR_INVALID_ARGUMENT, "job %d: y must be one of its rank destinations", i);
        fill_job(grp.job[i], j.x, j.ldx, j.packed, j.scale, j.packed_up, j.scale_up, j.bias, j.n, j.k, j.y, j.y_dtype,
                 j.ldy);
        grp.job[i].m = (int)m;
    }
    dispatch_group_t<true>(grp, ps, x_kind(x_dtype), m > 8 ? 2 : 1, static_cast<cudaStream_t>(stream));
    return check_launch("gemv_w8_group_peer");
}

extern "C" int sbq_peer_wait(const unsigned* count, unsigned* state, unsigned expected, void* stream) {
    if (!count || !state || expected == 0) return set_error(SBQ_ERR_INVALID_ARGUMENT, "null counter/state or zero expected");
    if (reinterpret_cast<uintptr_t>(count) % 128 || reinterpret_cast<uintptr_t>(state) % 8)
        return set_error(SBQ_ERR_ALIGNMENT, "signal must be 128-byte and state 8-byte aligned");
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(32);
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, peer_wait_kernel, count, state, expected);
    return check_launch("peer_wait");
}

// ---- decode program: build (once, synchronous) and run (per step, capturable) ---------------------
static int program_ctas() { return kCtasPerSm * sm_count(); }

static size_t program_bytes_for(int nstages, int nctas) {
    return 256 + (size_t)nstages * sizeof(ProgStage) + (size_t)nstages * nctas * sizeof(ProgItem);
}

extern "C" size_t sbq_gemv_program_bytes(int nstages) {
    if (nstages < 1) return 0;
    return program_bytes_for(nstages, program_ctas());
}

extern "C" int sbq_gemv_program_build(const sbq_gemv_job* jobs, const int* job_stage, int njobs, int x_dtype, int64_t m,
                                      void* program, size_t program_bytes) {
    if (!jobs || !job_stage || njobs < 1 || !program) return set_error(SBQ_ERR_INVALID_ARGUMENT, "null argument");
    if (x_kind(x_dtype) < 0) return set_error(SBQ_ERR_UNSUPPORTED, "activation dtype %d", x_dtype);
    if (reinterpret_cast<uintptr_t>(program) % 256) return set_error(SBQ_ERR_ALIGNMENT, "program must be 256-byte aligned");
    int nstages = 0;
    for (int i = 0; i < njobs; ++i) {
        if (job_stage[i] < 0 || (i > 0 && job_stage[i] < job_stage[i - 1]))
            return set_error(SBQ_ERR_INVALID_ARGUMENT, "job stages must be non-negative and non-decreasing");
        if (job_stage[i] + 1 > nstages) nstages = job_stage[i] + 1;
    }
    const int nctas = program_ctas();
    if (program_bytes < program_bytes_for(nstages, nctas))
        return set_error(SBQ_ERR_WORKSPACE, "program needs %zu bytes", program_bytes_for(nstages, nctas));
    const int es = elem_size(x_dtype);
    std::vector<uint8_t> host(program_bytes_for(nstages, nctas), 0);
    ProgStage* stages = reinterpret_cast<ProgStage*>(host.data() + 256);
    ProgItem* items = reinterpret_cast<ProgItem*>(host.data() + 256 + (size_t)nstages * sizeof(ProgStage));
    for (int i = 0; i < njobs; ++i) {
        const sbq_gemv_job& j = jobs[i];
        int st = check_linear_args(j.x, x_dtype, j.ldx, j.packed, j.scale, m, j.n, j.k, j.y, j.y_dtype, j.ldy);
        if (st) return set_error(st, "job %d: %s", i, sbq_last_error());
        if (m > 8 || m * (j.k * es + 16) > kXBytes)
            return set_error(SBQ_ERR_UNSUPPORTED, "job %d: a program needs m * (k + 8) activation elements to fit in "
                             "%d bytes (m=%lld k=%lld)", i, kXBytes, (long long)m, (long long)j.k);
        if (j.packed_up && (!j.scale_up || j.bias))
            return set_error(SBQ_ERR_INVALID_ARGUMENT, "job %d: fused gate/up job needs scale_up and no bias", i);
        ProgStage& ps = stages[job_stage[i]];
        if (ps.njobs >= kMaxJobs) return set_error(SBQ_ERR_UNSUPPORTED, "more than %d jobs in one stage", kMaxJobs);
        GemvJob& jb = ps.job[ps.njobs++];
        fill_job(jb, j.x, j.ldx, j.packed, j.scale, j.packed_up, j.scale_up, j.bias, j.n, j.k, j.y, j.y_dtype, j.ldy);
        jb.m = (int)m;
        jb.n_tiles = (int)ceil_div(j.n, 16);
    }
    // per stage: CTAs in proportion to each job's weight bytes, consecutive tiles per CTA
    for (int st = 0; st < nstages; ++st) {
        ProgStage& ps = stages[st];
        ProgItem* row = items + (size_t)st * nctas;
        for (int c = 0; c < nctas; ++c) row[c] = ProgItem{0, 0, 0};
        if (ps.njobs == 0) continue;
        double total = 0.0;
        for (int i = 0; i < ps.njobs; ++i)
            total += (double)ps.job[i].n_tiles * (ps.job[i].w1 ? 2 : 1) * ps.job[i].kt_total;
        const double per_cta = total / nctas;
        int c = 0;
        for (int i = 0; i < ps.njobs && c < nctas; ++i) {
            GemvJob& jb = ps.job[i];
            const double tile_cost = (double)(jb.w1 ? 2 : 1) * jb.kt_total;
            int t = (int)std::ceil(per_cta / tile_cost - 1e-9);
            if (t < 1) t = 1;
            // leave at least one CTA for every later job
            const int later = ps.njobs - 1 - i;
            while ((int)ceil_div(jb.n_tiles, t) > nctas - c - later) ++t;
            jb.tiles_per_cta = t;
            for (int t0 = 0; t0 < jb.n_tiles && c < nctas; t0 += t, ++c)
                row[c] = ProgItem{i, t0, t0 + t < jb.n_tiles ? t0 + t : jb.n_tiles};
        }
    }
    int* header = reinterpret_cast<int*>(host.data());
    header[0] = nstages;
    header[1] = nctas;
    header[2] = x_dtype;
    header[3] = (int)m;
    if (cudaMemcpy(program, host.data(), host.size(), cudaMemcpyHostToDevice) != cudaSuccess)
        return check_launch("copy decode program");
    return SBQ_OK;
}

extern "C" int sbq_gemv_program_run(const void* program, int nstages, int x_dtype, int* counters, void* stream) {
    if (!program || !counters || nstages < 1) return set_error(SBQ_ERR_INVALID_ARGUMENT, "null argument");
    const int xk = x_kind(x_dtype);
    if (xk < 0) return set_error(SBQ_ERR_UNSUPPORTED, "activation dtype %d", x_dtype);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (cudaMemsetAsync(counters, 0, sizeof(int) * nstages, s) != cudaSuccess) return check_launch("clear counters");
    ProgParams pp{};
    const uint8_t* base = static_cast<const uint8_t*>(program);
    const int nctas = program_ctas();
    pp.stages = reinterpret_cast<const ProgStage*>(base + 256);
    pp.items = reinterpret_cast<const ProgItem*>(base + 256 + (size_t)nstages * sizeof(ProgStage));
    pp.nstages = nstages;
    pp.counters = counters;
    const int smem = GemvSmemSize<1>::kBytes;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)nctas);
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // every CTA co-resident: the stage barriers rely on it
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e;
    switch (xk) {
        case kXF16:
            cudaFuncSetAttribute(gemv_program_kernel<kXF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            e = cudaLaunchKernelEx(&cfg, gemv_program_kernel<kXF16>, pp);
            break;
        case kXBF16:
            cudaFuncSetAttribute(gemv_program_kernel<kXBF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            e = cudaLaunchKernelEx(&cfg, gemv_program_kernel<kXBF16>, pp);
            break;
        default:
            cudaFuncSetAttribute(gemv_program_kernel<kXF32>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            e = cudaLaunchKernelEx(&cfg, gemv_program_kernel<kXF32>, pp);
            break;
    }
    if (e != cudaSuccess) return set_error(SBQ_ERR_CUDA, "decode program launch: %s", cudaGetErrorString(e));
    return check_launch("gemv_program");
}
