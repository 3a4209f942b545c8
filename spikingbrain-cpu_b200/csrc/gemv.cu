// Decode GEMV for the int8 weight-only format (and the fused gate/up SwiGLU half of the MLP).
//
// Reference: Int8Linear.forward (spikingbrain_cpu/quant.py:41-53) at decode shapes (one token per
// call, engine.py:104-106) and GatedMLP.forward (model.py:239-240).  The reference dequantises
// each 128-row block of the weight to fp32 and runs an fp32 sgemm, then multiplies by the
// per-row scale.  Here the weight is streamed from HBM exactly once per launch:
//
//   * a launch's work is a list of units - one 16-row tile of one job (its contiguous K strip in
//     the packed layout), or one K part of such a tile when the tiles are too few for the GPU -
//     and every CTA slot of the GPU (three per SM) runs one CTA; each CTA's producer thread takes
//     its first unit by block index and claims the next ones from a per-launch counter, largest
//     units first, and streams them with cp.async.bulk copies into a 48 KiB shared-memory ring
//     (16 KiB chunks, mbarrier transaction counts; each chunk's unit described beside it);
//   * eight consumer warps (or four on gate and four on up) take two 1 KiB tiles of each chunk
//     (one chunk's waits and bookkeeping per two tiles): per tile two conflict-free 16-byte shared
//     loads per lane, int8 -> fp16 (or bf16) in registers
//     (exact), m16n8k16 tensor-core MMAs with fp32 accumulation and the activation rows as the n
//     dimension (8 or 16 tokens per pass); activation fragments are read in place (L1-cached)
//     before waiting for the chunk, so the load overlaps the wait;
//   * at the end of each unit the warps' partial sums go to a double-buffered shared-memory area
//     and one rotating warp reduces them in a fixed order and applies the fp32 per-row scale (and
//     bias, or the SiLU(gate) * up product) while the others continue; K parts are added in part
//     order by the CTA that completes a tile's last part (deterministic);
//   * one launch can carry several independent projections ("jobs": e.g. q|k|v|delta_in and
//     gate/up of one layer, which read the same x);
//   * programmatic dependent launch: the weights never depend on the previous kernel, so the
//     producer starts streaming at once; only the consumers wait (griddepcontrol.wait, or the
//     peer signal of a sharded step) before reading x, and each CTA releases the next launch once
//     its consumers have passed that wait;
//   * ready jobs (inputs written two or more launches back) are ordered first and their units run
//     before the wait, which the consumers take at their first unit of another job.
//
// fp32 activations are split into a bf16 high and low part (two MMAs, ~16 mantissa bits kept);
// the dot product of int8 weights and fp16/bf16 activations is exact up to fp32 accumulation.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <mutex>
#include <queue>
#include <unordered_map>
#include <unordered_set>
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
    int chunk_tiles;   // tiles per chunk and matrix: the largest of 16 (8 for gate/up), 8, 4, 2, 1 dividing kt_total
    int out_f16;       // 1: fp16 output, 0: fp32
    int n_tiles;       // 16-row tiles of the weight
};

constexpr int kMaxJobs = 8;

struct GemvGroup {
    GemvJob job[kMaxJobs];
    int njobs;
    int n_ready;                     // jobs [0, n_ready) are ready: their x is not the previous kernel's output
    int spread;                      // > 1: CTAs per SM of the grid; first units dealt across SMs (see produce_units)
    int total_units;                 // units of all jobs (a unit = one K part of one 16-row tile)
    int unit_begin[kMaxJobs + 1];    // first unit of each job
    int parts[kMaxJobs];             // K parts per tile of each job (1: a tile is one unit)
    int split_base[kMaxJobs];        // first split-tile counter of each job (jobs with parts > 1)
    int64_t split_fbase[kMaxJobs];   // first scratch float of each job: [tile][part][split_stride]
    int split_stride;                // floats per part partial (entries x matrices)
    unsigned* claim;                 // this launch's work counter pair (g_claim slot)
    float* split_scratch;            // part partials [split tile][part][split_stride]
    unsigned* split_count;           // parts completed per split tile (reset by the combining CTA)
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
    unsigned long long wait_limit_ns;  // bound of the wait
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
// the next step.  Bounded (by default ranks may drift apart on the host by up to kPeerWaitLimitNs): on expiry
// the error word is set and the kernel carries on (its outputs are then invalid, the host sees
// SBQ_ERR_TIMEOUT); after an earlier failure it does not wait at all.
constexpr uint64_t kPeerWaitLimitNs = 10000000000ull;

__device__ __forceinline__ void peer_wait(const unsigned* signal, unsigned* state, unsigned expected,
                                          unsigned long long limit_ns) {
    const unsigned* count = signal + (blockIdx.x % kSignalCopies) * kSignalStride;
    const unsigned gen = *reinterpret_cast<volatile unsigned*>(state);
    const unsigned target = (gen + 1u) * expected;
    if (*reinterpret_cast<volatile int*>(&g_device_error) == 0 && (int)(ld_acquire_sys(count) - target) < 0) {
        const uint64_t t0 = tc::now_ns();
        for (uint32_t i = 1; (int)(ld_acquire_sys(count) - target) < 0; ++i) {
            __nanosleep(64);
            if ((i & 63) == 0 && tc::now_ns() - t0 > limit_ns) {
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
// x written earlier in the same launch (or by other GPUs) is read with these ordinary loads too: the
// reading CTA has passed an acquire (one thread) and a CTA barrier since, the grid-barrier pattern.
template <int XK>
__device__ __forceinline__ void load_x(XFrag<XK>& f, const void* xv, int64_t ldx, int row, int m, int64_t k0, int k) {
    const uint8_t* x = static_cast<const uint8_t*>(xv);
    const bool ok = row < m && k0 < k;
    if (XK == kXF16 || XK == kXBF16) {
        uint4 v0 = make_uint4(0, 0, 0, 0), v1 = v0;
        if (ok) {
            const uint4* q = reinterpret_cast<const uint4*>(x + ((int64_t)row * ldx + k0) * 2);
            v0 = q[0];
            v1 = q[1];
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
                const uint4 t = q[i];
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


constexpr int kGemvThreads = (kGemvWarps + 1) * 32;  // 8 consumer warps + 1 producer warp
constexpr int kChunkTiles = 16;                        // tiles (KiB) per chunk and matrix, at most
#ifndef SBQ_GEMV_STAGES
#define SBQ_GEMV_STAGES 3
#endif
constexpr int kMaxStages = SBQ_GEMV_STAGES;            // ring stages of 16 KiB (16 tiles, or 8 gate + 8 up tiles)
constexpr int kRingBytes = kMaxStages * 16 * 1024;
template <int MT>
struct GemvSmemSize {
    static constexpr int kRed = 2 * kGemvWarps * MT * 16 * 9 * 4;  // per-warp partial sums of two tiles
    static constexpr int kBytes = kRingBytes + kRed + 2 * kMaxStages * 8;  // 3 CTAs per SM at MT = 1
};
#ifndef SBQ_GEMV_CTAS_PER_SM
#define SBQ_GEMV_CTAS_PER_SM 3
#endif
constexpr int kCtasPerSm = SBQ_GEMV_CTAS_PER_SM;  // CTAs a launch is sized for (three fit per SM)
// The same for 9..16 rows (twice the accumulators).  Measured: three per SM (72 registers) runs the
// 36-layer step at 9 / 12 / 16 rows in 2.38 / 2.44 / 2.53 ms against 2.30 / 2.52 / 2.71 ms with two,
// but the fused MLP alone at 16 rows (configuration 1) in 60 us against 52-54 us; two are kept.
#ifndef SBQ_GEMV_CTAS_PER_SM_16
#define SBQ_GEMV_CTAS_PER_SM_16 2
#endif
constexpr int kCtasPerSm16 = SBQ_GEMV_CTAS_PER_SM_16;
// Launches with at least one unit per SM take the whole grid with their first units dealt across the
// SMs (GemvGroup::spread).  Measured on the 36-layer step: batch 1 1.643 -> 1.63 ms, batch 8 1.95 ->
// 1.88 ms; a 4096 x 4096 launch alone 6.17 -> 6.28 us at one row, 6.81 -> 6.57 us at eight.
#ifndef SBQ_GEMV_SPREAD
#define SBQ_GEMV_SPREAD 1
#endif

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

// ---------------------------------------------------------------------------------------------
// Grouped launch with dynamic work: the units of a launch are the 16-row tiles of all its jobs
// (largest tiles first), claimed one at a time from a per-launch counter by each CTA's producer.
// A CTA that runs ahead (the warp schedulers favour some CTAs of an SM over others) simply takes
// more units, so every CTA slot stays busy until the work runs out and the launch ends within about
// one unit of its ideal time.  Each ring stage carries its unit's (job, tile, chunk, chunks) in
// shared memory; x is read in place, so a CTA may take units of different jobs.
// ---------------------------------------------------------------------------------------------
//
// Work counters and split-K scratch are device arrays of this library, divided into lanes so that
// launches on different streams never share them: each stream (per device) is given one of kLanes
// lanes the first time it launches a grouped GEMV, and launches take their counter and scratch from
// their stream's lane only (decode programs have a lane of their own).  Up to kLanes streams per
// device can therefore run grouped GEMVs concurrently; a CUDA graph keeps the lane of the stream it
// was captured on.
constexpr int kLanes = kStreamLanes;       // stream lanes for grouped launches
constexpr int kProgramLane = kLanes;       // the decode programs' lane
constexpr int kLaneCount = kLanes + 1;
constexpr int kClaimSlots = 128;           // per lane: per-launch counters, used round-robin
static __device__ unsigned g_claim[kLaneCount][kClaimSlots][2];  // [next unit, unused]; reset by the launch's last claimer
// (every claiming CTA makes exactly one failing claim, so the values handed out are 0 .. units - 1;
// the producer that gets units - 1 resets the counter, early and off the CTAs' exit path)

// Split-K scratch: when a launch has too few tiles to keep every CTA busy (a sharded step on several
// GPUs), tiles are cut into K parts; each part's partial sums go here and the CTA that completes a
// tile's last part adds them in part order (deterministic).  Two regions per lane, used alternately
// by consecutive launches of the lane: with programmatic dependent launch a launch may overlap the
// one before it on its stream, but its consumers start only after that one has completed, which
// itself waited for the one before, so a region is never used by two launches at once.
constexpr int kSplitRegions = 2;
constexpr int kSplitFloats = 512 * 1024;  // per region (2 MiB)
constexpr int kSplitTiles = 8192;         // split tiles per region
static __device__ float g_split[kLaneCount][kSplitRegions][kSplitFloats];
static __device__ unsigned g_split_count[kLaneCount][kSplitRegions][kSplitTiles];

// Producer (one thread).  Claims the next unit while the last ring-full of the current one is
// still to be issued, so the claim's latency is hidden; the producer that makes the launch's last
// claim resets the counter.  False if a wait timed out (after the CTA's remaining claims, so that
// the reset still happens).  `claim`: the work counter pair; `ci`: ring position (continues across calls, the decode program
// streams one group per stage through the same ring).  The end marker takes a ring slot too.
__device__ __forceinline__ bool produce_units(const GemvGroup& grp, unsigned* claim, uint8_t* ring, uint64_t* full,
                                              uint64_t* empty, int4* meta, uint32_t& ci) {
    constexpr int S = kMaxStages;
    constexpr int kStageBytes = kChunkTiles * kTileBytes;
    // the first unit of every CTA is its own, later ones are claimed.  With `spread` (a grid of
    // `spread` CTAs per SM) block b takes unit (b % spread) * (grid / spread) + b / spread: a
    // permutation of the grid that deals the first units across the SMs however the blocks are
    // placed (consecutive blocks share an SM or not), so a launch with fewer units than CTA slots
    // does not crowd them onto a third of the SMs
    int u = blockIdx.x;
    if (grp.spread > 1) u = (int)(blockIdx.x % grp.spread) * (int)(gridDim.x / grp.spread) + (int)(blockIdx.x / grp.spread);
    for (;;) {
        if (u >= grp.total_units) {
            const int s = ci % S;
            if (!tc::mbar_wait(&empty[s], ((ci / S) & 1) ^ 1)) return false;
            meta[s] = make_int4(-1, 0, 0, 0);
            tc::mbar_arrive(&full[s]);  // the end marker: a phase with no bytes
            ++ci;
            return true;
        }
        int j = 0;
        while (j + 1 < grp.njobs && u >= grp.unit_begin[j + 1]) ++j;
        const GemvJob& jb = grp.job[j];
        const int P = grp.parts[j];
        const int tile = (u - grp.unit_begin[j]) / P, part = (u - grp.unit_begin[j]) % P;
        const int C = jb.chunk_tiles, cpt = jb.kt_total / C, nmat = jb.w1 ? 2 : 1;
        const int i0 = part * cpt / P, i1 = (part + 1) * cpt / P;  // this part's chunks
        const uint32_t bytes = (uint32_t)C * kTileBytes;
        const int8_t* src0 = jb.w0 + (int64_t)tile * jb.kt_total * kTileBytes;
        const int8_t* src1 = jb.w1 ? jb.w1 + (int64_t)tile * jb.kt_total * kTileBytes : nullptr;
        const int claim_at = i1 - i0 > S ? i1 - S : i0;
        unsigned v = 0;
        for (int i = i0; i < i1; ++i, ++ci) {
            if (i == claim_at) v = atomicAdd(claim, 1u);
            const int s = ci % S;
            if (!tc::mbar_wait(&empty[s], ((ci / S) & 1) ^ 1)) {
                // keep the count: claim (and drop) until this CTA's one failing claim
                if (i < claim_at) v = atomicAdd(claim, 1u);
                while ((int)(gridDim.x + v) < grp.total_units) v = atomicAdd(claim, 1u);
                if (v == (unsigned)grp.total_units - 1u) claim[0] = 0;
                return false;
            }
            meta[s] = make_int4(j | (part << 8), tile, i, i1 - i0);
            uint8_t* dst = ring + s * kStageBytes;
            tc::mbar_arrive_expect_tx(&full[s], bytes * nmat);
            tc::bulk_load(dst, src0 + (int64_t)i * bytes, bytes, &full[s]);
            if (nmat == 2) tc::bulk_load(dst + bytes, src1 + (int64_t)i * bytes, bytes, &full[s]);
        }
        // every claiming CTA makes exactly one failing claim, so the values handed out are
        // 0 .. total_units - 1 and the one that gets the last has made the launch's last claim
        if (v == (unsigned)grp.total_units - 1u) claim[0] = 0;
        u = (int)(gridDim.x + v);
    }
}

// The consumers' wait for the producer of x when it is deferred past the ready jobs' units: the
// previous grid (griddepcontrol.wait, every thread), or in a sharded launch the producing launch's
// signal on every rank - thread 0 waits (peer_wait: once per CTA, it also records the CTA's arrival)
// and releases the other consumer warps through a shared flag, which they poll with a bound (a warp
// that gave up after a timeout elsewhere cannot hold them at a barrier).  Then the CTA lets the next
// launch begin.
template <bool PEER>
__device__ __forceinline__ void deferred_wait(const PeerSync& ps, int* s_flag) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (PEER && ps.wait_count) {
        if (lane == 0) {
            if (warp == 0) {
                peer_wait(ps.wait_count, ps.wait_state, ps.wait_expected, ps.wait_limit_ns);
                asm volatile("st.release.cta.shared.u32 [%0], %1;" ::"r"(tc::smem_u32(s_flag)), "r"(1u) : "memory");
            } else {
                const uint64_t t0 = tc::now_ns();
                for (uint32_t i = 1;; ++i) {
                    unsigned v;
                    asm volatile("ld.acquire.cta.shared.u32 %0, [%1];" : "=r"(v) : "r"(tc::smem_u32(s_flag)) : "memory");
                    if (v) break;
                    __nanosleep(32);
                    if ((i & 63) == 0 && tc::now_ns() - t0 > ps.wait_limit_ns + 1000000000ull) {
                        tc::raise_error(SBQ_ERR_TIMEOUT);
                        break;
                    }
                }
            }
        }
        __syncwarp();
    } else {
        asm volatile("griddepcontrol.wait;" ::: "memory");
    }
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Consumers (8 warps): per unit, its chunks (each warp takes tiles slot and slot + 8 of each chunk,
// or slot and slot + 4 of each matrix of a gate/up chunk - the same tiles, in the same order, as one
// tile per warp of chunks half the size; per tile two conflict-free 16-byte shared loads per lane,
// int8 -> fp16/bf16 in registers, m16n8k16 MMAs with the activation rows as the n dimension), then
// the fixed-order reduction and the epilogue.  The
// job and the warp split are read once per unit from the first chunk's stage.
// False (warp-uniformly) on a timeout.
// `ci` / `units`: ring position and units done so far (both continue across calls).
// `waited`: null when the consumers have waited for the previous kernel already; else the flag of a
// deferred wait (deferred_wait), taken before the first unit of a job that is not ready.
template <int XK, int MT, bool PEER>
__device__ __forceinline__ bool consume_units(const GemvGroup& grp, uint8_t* ring, float* red, uint64_t* full,
                                              uint64_t* empty, const int4* meta, const PeerSync& ps,
                                              uint32_t& ci, int& units, bool* waited = nullptr,
                                              int* s_flag = nullptr) {
    constexpr int S = kMaxStages;
    constexpr int kStageBytes = kChunkTiles * kTileBytes;
    constexpr int kEntries = MT * 8 * 16;
    constexpr int kRedFloats = kGemvWarps * MT * 16 * 9;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, c = lane & 3;
    for (;; ++units) {
        int s = ci % S;
        if (!__all_sync(0xffffffffu, tc::mbar_wait(&full[s], (ci / S) & 1))) return false;
        const int4 md = meta[s];
        if (md.x < 0) {
            // the end marker: release its slot (the producer may go on with another group)
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&empty[s]);
            ++ci;
            break;
        }
        const int j = md.x & 0xff, part = md.x >> 8, tile = md.y, i0 = md.z, cpt = md.w;
        const GemvJob& jb = grp.job[j];
        if (waited && !*waited && j >= grp.n_ready) {
            // the first unit whose x is the previous launch's output (see gemv_w8_kernel)
            deferred_wait<PEER>(ps, s_flag);
            *waited = true;
        }
        const bool two = jb.w1 != nullptr;
        const int C = jb.chunk_tiles;
        const int mat = two ? warp >> 2 : 0, slot = two ? warp & 3 : warp;
        const bool mine = slot < C;
        const int W2 = two ? 4 : 8;
        const bool mine2 = slot + W2 < C;
        const void* xj = jb.x;
        const int64_t ldx = jb.ldx;
        const int xm = jb.m, xk = jb.k;
        const uint32_t toff = (uint32_t)((mat * C + slot) * kTileBytes + lane * 16);
        const uint32_t toff2 = toff + W2 * kTileBytes;
        float acc[MT][4];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[mt][e] = 0.0f;
        // this unit's epilogue runs on warp (unit % 8) onwards: its threads fetch the scales now
        const int vt = (threadIdx.x + kGemvWarps * 32 - (units % kGemvWarps) * 32) % (kGemvWarps * 32);
        float sc0 = 0.0f, sc1 = 0.0f, bz = 0.0f;
        {
            const int n = tile * 16 + (vt & 15);
            if (vt < kEntries && n < jb.n) {
                sc0 = jb.s0[n];
                if (two) sc1 = jb.s1[n];
                else if (jb.bias) bz = jb.bias[n];
            }
        }
        XFrag<XK> xf[MT], xf2[MT];
        if (mine) {
            const int64_t k0 = (int64_t)(i0 * C + slot) * kTileCols + 16 * c;
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) load_x<XK>(xf[mt], xj, ldx, 8 * mt + g, xm, k0, xk);
        }
        if (mine2) {
            const int64_t k0 = (int64_t)(i0 * C + slot + W2) * kTileCols + 16 * c;
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) load_x<XK>(xf2[mt], xj, ldx, 8 * mt + g, xm, k0, xk);
        }
        for (int i = 0;;) {
            if (mine) {
                const uint8_t* t = ring + s * kStageBytes + toff;
                const uint4 wa = *reinterpret_cast<const uint4*>(t);
                const uint4 wb = *reinterpret_cast<const uint4*>(t + 512);
                tile_mma<XK, MT>(acc, wa, wb, xf);
            }
            if (mine2) {
                const uint8_t* t = ring + s * kStageBytes + toff2;
                const uint4 wa = *reinterpret_cast<const uint4*>(t);
                const uint4 wb = *reinterpret_cast<const uint4*>(t + 512);
                tile_mma<XK, MT>(acc, wa, wb, xf2);
            }
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&empty[s]);
            ++ci;
            if (++i == cpt) break;
            // the next chunk of this unit: load its x, then wait for its weights (loading x a whole
            // chunk ahead instead measured slower)
            if (mine) {
                const int64_t k0 = (int64_t)((i0 + i) * C + slot) * kTileCols + 16 * c;
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) load_x<XK>(xf[mt], xj, ldx, 8 * mt + g, xm, k0, xk);
            }
            if (mine2) {
                const int64_t k0 = (int64_t)((i0 + i) * C + slot + W2) * kTileCols + 16 * c;
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) load_x<XK>(xf2[mt], xj, ldx, 8 * mt + g, xm, k0, xk);
            }
            s = ci % S;
            if (!__all_sync(0xffffffffu, tc::mbar_wait(&full[s], (ci / S) & 1))) return false;
        }

        // ---- unit complete: partial sums to a double-buffered area, one barrier, then the unit's
        // epilogue threads reduce (fixed order), scale and store while the other warps go on
        float* rb = red + (units & 1) * kRedFloats;
#define SBQ_RED(w, mt, r, col) rb[(((w) * MT + (mt)) * 16 + (r)) * 9 + (col)]
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            SBQ_RED(warp, mt, g, 2 * c) = acc[mt][0];
            SBQ_RED(warp, mt, g, 2 * c + 1) = acc[mt][1];
            SBQ_RED(warp, mt, g + 8, 2 * c) = acc[mt][2];
            SBQ_RED(warp, mt, g + 8, 2 * c + 1) = acc[mt][3];
        }
        consumers_sync();
        const int P = grp.parts[j];
        if (P > 1) {
            // a K part of a split tile: one warp writes the part's partial sums to the scratch; the
            // CTA completing the tile's last part sums the parts in order and runs the epilogue
            if (warp == units % kGemvWarps) {
                const int st = grp.split_base[j] + tile;
                const int stride = grp.split_stride;
                float* const tp = grp.split_scratch + grp.split_fbase[j] + (int64_t)tile * P * stride;
                float* mp = tp + (int64_t)part * stride;
                for (int e = lane; e < kEntries; e += 32) {
                    const int r = e & 15, tok = e >> 4, mt = tok >> 3, col = tok & 7;
                    float v0 = 0.0f, v1 = 0.0f;
                    if (!two) {
#pragma unroll
                        for (int w = 0; w < 8; ++w) v0 += SBQ_RED(w, mt, r, col);
                    } else {
#pragma unroll
                        for (int w = 0; w < 4; ++w) v0 += SBQ_RED(w, mt, r, col);
#pragma unroll
                        for (int w = 0; w < 4; ++w) v1 += SBQ_RED(4 + w, mt, r, col);
                        mp[kEntries + e] = v1;
                    }
                    mp[e] = v0;
                }
                __syncwarp();
                unsigned last = 0;
                if (lane == 0) {
                    __threadfence();  // this part's partial before the count
                    last = atomicAdd(grp.split_count + st, 1u) == (unsigned)(P - 1);
                    if (last) {
                        grp.split_count[st] = 0;  // for the next launch that uses this slot
                        __threadfence();          // every part's partial before the reads below
                    }
                }
                __syncwarp();
                last = __shfl_sync(0xffffffffu, last, 0);
                if (last) {
                    const float* base = tp;
                    for (int e = lane; e < kEntries; e += 32) {
                        const int r = e & 15, tok = e >> 4;
                        const int n = tile * 16 + r;
                        if (n >= jb.n || tok >= xm) continue;
                        float v0 = 0.0f, v1 = 0.0f;
                        for (int q = 0; q < P; ++q) {
                            v0 += __ldcg(base + (int64_t)q * stride + e);
                            if (two) v1 += __ldcg(base + (int64_t)q * stride + kEntries + e);
                        }
                        float out;
                        if (!two) {
                            out = v0 * jb.s0[n];
                            if (jb.bias) out += jb.bias[n];
                        } else {
                            const float gv = v0 * jb.s0[n];
                            const float uv = v1 * jb.s1[n];
                            out = gv / (1.0f + expf(-gv)) * uv;
                        }
                        const int64_t idx = (int64_t)tok * jb.ldy + n;
                        if (PEER) {
                            for (int p = 0; p < ps.nranks; ++p) {
                                if (jb.out_f16)
                                    static_cast<__half*>(ps.y[j][p])[idx] = __float2half_rn(out);
                                else
                                    static_cast<float*>(ps.y[j][p])[idx] = out;
                            }
                        } else if (jb.out_f16) {
                            static_cast<__half*>(jb.y)[idx] = __float2half_rn(out);
                        } else {
                            static_cast<float*>(jb.y)[idx] = out;
                        }
                    }
                }
            }
        } else if (vt < kEntries) {
            const int r = vt & 15, tok = vt >> 4, mt = tok >> 3, col = tok & 7;
            const int n = tile * 16 + r;
            if (n < jb.n && tok < xm) {
                float out;
                if (!two) {
                    float v0 = 0.0f;
#pragma unroll
                    for (int w = 0; w < 8; ++w) v0 += SBQ_RED(w, mt, r, col);
                    out = v0 * sc0;
                    if (jb.bias) out += bz;
                } else {
                    float v0 = 0.0f, v1 = 0.0f;
#pragma unroll
                    for (int w = 0; w < 4; ++w) v0 += SBQ_RED(w, mt, r, col);
#pragma unroll
                    for (int w = 0; w < 4; ++w) v1 += SBQ_RED(4 + w, mt, r, col);
                    const float gv = v0 * sc0;
                    const float uv = v1 * sc1;
                    out = gv / (1.0f + expf(-gv)) * uv;
                }
                const int64_t idx = (int64_t)tok * jb.ldy + n;
                if (PEER) {
                    // consecutive threads store consecutive rows: one coalesced NVLink write per rank
                    for (int p = 0; p < ps.nranks; ++p) {
                        if (jb.out_f16)
                            static_cast<__half*>(ps.y[j][p])[idx] = __float2half_rn(out);
                        else
                            static_cast<float*>(ps.y[j][p])[idx] = out;
                    }
                } else if (jb.out_f16) {
                    static_cast<__half*>(jb.y)[idx] = __float2half_rn(out);
                } else {
                    static_cast<float*>(jb.y)[idx] = out;
                }
            }
        }
#undef SBQ_RED
    }
    consumers_sync();  // the last epilogue is done
    return true;
}

template <int XK, int MT, bool PEER>
__global__ void __launch_bounds__(kGemvThreads, MT == 1 ? kCtasPerSm : kCtasPerSm16)
    gemv_w8_kernel(const __grid_constant__ GemvGroup grp, const __grid_constant__ PeerSync ps) {
    extern __shared__ __align__(128) uint8_t ring[];
    float* red = reinterpret_cast<float*>(ring + kRingBytes);
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + kRingBytes + GemvSmemSize<MT>::kRed);
    uint64_t* empty = full + kMaxStages;
    __shared__ int4 meta[kMaxStages];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kMaxStages; ++i) {
            tc::mbar_init(&full[i], 1);
            tc::mbar_init(&empty[i], kGemvWarps);
        }
        tc::fence_mbar_init();
    }
    __syncthreads();
    // Programmatic dependent launch.  The weights never depend on the previous kernel, so the
    // producer streams at once; the consumers wait for the previous kernel (or, sharded, for the
    // producing launch's signal on every rank) before reading x.  The next launch may begin once
    // every CTA here has passed that wait: the ready jobs of the next launch read outputs of the
    // launch before this one, which has then completed (on every rank).  Ready jobs' units come
    // first and run before the wait, which the consumers take at their first unit of another job
    // (or at the end).
    __shared__ int s_flag;
    if (threadIdx.x == 0) s_flag = 0;
    __syncthreads();
    if (warp == kGemvWarps) {
        uint32_t pci = 0;
        if (lane == 0 && !produce_units(grp, grp.claim, ring, full, empty, meta, pci)) tc::raise_error(SBQ_ERR_TIMEOUT);
        return;
    }
    bool waited = grp.n_ready == 0;
    if (waited) {
        if (PEER && ps.wait_count) {
            // x is the previous launch's output on every rank (this one included): its signal, not
            // the end of the previous grid, is what the consumers need, so they start as soon as the
            // last rank's last CTA has published (the release/acquire pair orders every store before)
            if (threadIdx.x == 0) peer_wait(ps.wait_count, ps.wait_state, ps.wait_expected, ps.wait_limit_ns);
            consumers_sync();
        } else {
            asm volatile("griddepcontrol.wait;" ::: "memory");  // x is the previous kernel's output
        }
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    }
    uint32_t ci = 0;
    int units = 0;
    const bool ok = consume_units<XK, MT, PEER>(grp, ring, red, full, empty, meta, ps, ci, units, &waited, &s_flag);
    if (!waited) deferred_wait<PEER>(ps, &s_flag);  // this warp ran ready units only
    if (!consumers_sync_and(ok) && threadIdx.x == 0) tc::raise_error(SBQ_ERR_TIMEOUT);
    if (PEER && warp == 0) peer_publish(ps, lane);  // also after a timeout, so that the other ranks do not wait in vain
}

// Waits (one CTA) for a peer launch's outputs: the end of a sharded decode step, before the host
// or another stream reads the gathered result.
__global__ void peer_wait_kernel(const unsigned* count, unsigned* state, unsigned expected,
                                 unsigned long long limit_ns) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (threadIdx.x == 0) peer_wait(count, state, expected, limit_ns);
}

// ---------------------------------------------------------------------------------------------
// Decode program: a whole sequence of grouped stages in one persistent cooperative launch.
//
// Stage s may read what stages < s wrote (on this rank and, in a sharded program, on every rank).
// Each stage is a grouped launch's work (dynamic units, K parts), streamed through the CTA's ring
// by its producer, which moves on to the next stage's units as soon as the current stage's are all
// claimed: the weight stream never waits for a stage barrier.  When its consumers have finished
// the stage's units (its end marker), the CTA counts itself in on the stage's arrival counter
// (GPU-scope fence + 64-bit atomic; the counters only grow, so a run's epoch E is the first return
// value / grid size); the last CTA of the stage on each rank resets the stage's claim counter and
// adds 1 to the stage's flag on every rank, in 32 copies on separate L2 lines.  Before stage s + 1
// a CTA's consumers poll their copy (with backoff) until it reaches (E + 1) * ranks.  All CTAs are
// co-resident (cooperative launch) and every wait is bounded.
// ---------------------------------------------------------------------------------------------
struct ProgStage {
    GemvGroup grp;  // the stage's jobs, planned as a grouped launch (claim counter: in the sync region)
    PeerSync peer;  // sharded program: output destinations on every rank (y, nranks)
};

// Synchronisation region per stage: the arrival counter, 32 lines of flag copies, the claim pair.
constexpr int kSyncFlagOff = 128;
constexpr int kSyncClaimOff = 128 + kSignalCopies * 128;
constexpr int kSyncStageBytes = kSyncClaimOff + 128;

// Header at the start of a program buffer (256 bytes).
struct ProgHeader {
    int nstages;
    int nctas;
    int x_dtype;
    int m;
    int nranks;                        // 1: single GPU; > 1: sharded program
    int pad[3];
    uint8_t* peer_sync[kMaxPeers];     // every rank's synchronisation region as mapped here
};
static_assert(sizeof(ProgHeader) <= 256, "program header");

struct ProgParams {
    const ProgHeader* hdr;
    const ProgStage* stages;
    int nstages;
    uint8_t* sync;                     // this rank's synchronisation region
};

__device__ __forceinline__ unsigned* prog_flag(uint8_t* sync, int st, int copy) {
    return reinterpret_cast<unsigned*>(sync + (size_t)st * kSyncStageBytes + kSyncFlagOff + copy * 128);
}

__device__ __forceinline__ unsigned* prog_claim(uint8_t* sync, int st) {
    return reinterpret_cast<unsigned*>(sync + (size_t)st * kSyncStageBytes + kSyncClaimOff);
}

template <int XK, bool PEER>
__global__ void __launch_bounds__(kGemvThreads, kCtasPerSm) gemv_program_kernel(const __grid_constant__ ProgParams p) {
    constexpr int MT = 1;
    extern __shared__ __align__(128) uint8_t ring[];
    float* red = reinterpret_cast<float*>(ring + kRingBytes);
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + kRingBytes + GemvSmemSize<MT>::kRed);
    uint64_t* empty = full + kMaxStages;
    __shared__ int4 meta[kMaxStages];
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
    if (warp == kGemvWarps) {
        if (lane == 0) {
            uint32_t pci = 0;
            for (int st = 0; st < p.nstages; ++st)
                if (!produce_units(p.stages[st].grp, prog_claim(p.sync, st), ring, full, empty, meta, pci)) {
                    tc::raise_error(SBQ_ERR_TIMEOUT);
                    break;
                }
        }
        return;
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");  // the first stage's x comes from the previous kernel
    const int nranks = PEER ? p.hdr->nranks : 1;
    const uint64_t limit = PEER ? kPeerWaitLimitNs : tc::kWaitLimitNs;
    unsigned long long epoch = 0;  // thread 0: this run's epoch, from its first arrival
    uint32_t ci = 0;
    int units = 0;
    for (int st = 0; st <= p.nstages; ++st) {
        if (st > 0 && (st < p.nstages || (PEER && cta == 0))) {
            // wait for stage st - 1 on every rank (after the last stage: one CTA, so that the
            // kernel ends only when every rank's final outputs have arrived)
            if (threadIdx.x == 0) {
                const unsigned* flag = prog_flag(p.sync, st - 1, cta % kSignalCopies);
                const unsigned target = (unsigned)(epoch + 1) * (unsigned)nranks;
                if ((int)(ld_acquire_sys(flag) - target) < 0) {
                    const uint64_t t0 = tc::now_ns();
                    for (uint32_t i = 1; (int)(ld_acquire_sys(flag) - target) < 0; ++i) {
                        __nanosleep(32);
                        if ((i & 63) == 0 && tc::now_ns() - t0 > limit) {
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
        if (st == p.nstages) break;
        const ProgStage& ps = p.stages[st];
        if (!consume_units<XK, MT, PEER>(ps.grp, ring, red, full, empty, meta, ps.peer, ci, units)) {
            if (lane == 0) tc::raise_error(SBQ_ERR_TIMEOUT);
            abort_flag = 1;
        }
        // count in: every consumer's stores precede the barrier, the fence of the counting thread
        // orders them before its increment (and the last one's system fence before the flags)
        consumers_sync();
        if (abort_flag) return;
        if (warp == 0) {
            unsigned last = 0;
            if (lane == 0) {
                __threadfence();
                unsigned long long* ctr = reinterpret_cast<unsigned long long*>(p.sync + (size_t)st * kSyncStageBytes);
                const unsigned long long old = atomicAdd(ctr, 1ull);
                if (st == 0) epoch = old / (unsigned long long)nctas;
                last = old + 1 == (epoch + 1) * (unsigned long long)nctas;
                if (last) {
                    // every producer has made its last claim of this stage (before the end marker
                    // its consumers have seen): the claim counter starts over for the next run
                    unsigned* claim = prog_claim(p.sync, st);
                    claim[0] = 0;
                    claim[1] = 0;
                }
            }
            __syncwarp();
            last = __shfl_sync(0xffffffffu, last, 0);
            if (last) {
                if (PEER) {
                    __threadfence_system();
                    for (int r = 0; r < nranks; ++r) red_add_sys(prog_flag(p.hdr->peer_sync[r], st, lane), 1u);
                } else {
                    __threadfence();
                    atomicAdd(prog_flag(p.sync, st, lane), 1u);
                }
            }
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

// SMs of the current device, cached per device (atomics: first calls may come from several threads)
static int sm_count() {
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

// Device addresses of this device's claim counters and split scratch (cached per device).
struct UnitBuffers {
    unsigned* claim = nullptr;        // [kLaneCount][kClaimSlots][2]
    float* split = nullptr;           // [kLaneCount][kSplitRegions][kSplitFloats]
    unsigned* split_count = nullptr;  // [kLaneCount][kSplitRegions][kSplitTiles]
};

static const UnitBuffers* unit_buffers() {
    static UnitBuffers per_dev[64];
    static std::mutex mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    UnitBuffers& b = per_dev[dev];
    if (!b.claim) {
        void *c = nullptr, *sp = nullptr, *sc = nullptr;
        if (cudaGetSymbolAddress(&c, g_claim) != cudaSuccess || cudaGetSymbolAddress(&sp, g_split) != cudaSuccess ||
            cudaGetSymbolAddress(&sc, g_split_count) != cudaSuccess)
            return nullptr;
        b.split = static_cast<float*>(sp);
        b.split_count = static_cast<unsigned*>(sc);
        b.claim = static_cast<unsigned*>(c);
    }
    return &b;
}

// The lane of a stream on the current device (assigned round-robin on first use) and the lane's
// launch count.  The per-thread default stream is one stream per host thread, so it is keyed by
// thread too.  The table is bounded: past 4096 entries it starts afresh.
struct LaneKey {
    int dev;
    const void* stream;
    size_t thread;
    bool operator==(const LaneKey& o) const { return dev == o.dev && stream == o.stream && thread == o.thread; }
};
struct LaneKeyHash {
    size_t operator()(const LaneKey& k) const {
        return std::hash<const void*>()(k.stream) ^ ((size_t)k.dev * 0x9E3779B97F4A7C15ull) ^ (k.thread * 1099511628211ull);
    }
};
static std::atomic<unsigned> g_lane_launches[64][kLaneCount];

int stream_lane(cudaStream_t s, int dev) {
    static std::mutex mu;
    static std::unordered_map<LaneKey, int, LaneKeyHash> lanes;
    static unsigned next[64] = {};
    static thread_local char thread_tag;
    LaneKey key{dev, static_cast<const void*>(s),
                s == cudaStreamPerThread ? reinterpret_cast<size_t>(&thread_tag) : size_t(0)};
    std::lock_guard<std::mutex> lock(mu);
    auto it = lanes.find(key);
    if (it != lanes.end()) return it->second;
    if (lanes.size() >= 4096) lanes.clear();
    const int lane = (int)(next[dev]++ % kLanes);
    lanes.emplace(key, lane);
    return lane;
}

// Launch time of units claimed greedily by `slots` equally fast CTAs, in bytes per CTA: the units
// are taken in order, each by the CTA that is free first.
static double greedy_makespan(const std::vector<double>& unit_bytes, int slots) {
    std::priority_queue<double, std::vector<double>, std::greater<double>> free_at;
    for (int i = 0; i < slots; ++i) free_at.push(0.0);
    double end = 0.0;
    for (double b : unit_bytes) {
        const double t = free_at.top() + b;
        free_at.pop();
        free_at.push(t);
        end = std::max(end, t);
    }
    return end;
}

// K parts per tile for a launch shape.  Launch time model: the larger of the GPU's streaming time
// (all bytes at the HBM rate) and the busiest CTA's bytes at one CTA's own rate (a CTA streams
// about 1/kCtaShare of the HBM rate: its ring holds a fixed number of bytes in flight), with units
// claimed greedily.  Tiles are cut into K parts (at least 32 KiB and whole chunks each, partial sums
// added in part order) only while that lowers the modelled time by more than 2 %: a sharded step
// on several GPUs, whose launches have few tiles, cuts its large tiles; a one-GPU launch does not.
// Cached per shape: eager callers plan each shape once.
#ifndef SBQ_GEMV_CTA_SHARE
#define SBQ_GEMV_CTA_SHARE 200.0
#endif
constexpr double kCtaShare = SBQ_GEMV_CTA_SHARE;
struct PartsKey {
    int slots, m, nj;
    int64_t shape[kMaxJobs][3];  // tiles, tile bytes, chunks per tile
    bool operator==(const PartsKey& o) const {
        if (slots != o.slots || m != o.m || nj != o.nj) return false;
        for (int i = 0; i < nj; ++i)
            for (int f = 0; f < 3; ++f)
                if (shape[i][f] != o.shape[i][f]) return false;
        return true;
    }
};
struct PartsKeyHash {
    size_t operator()(const PartsKey& k) const {
        size_t h = (size_t)k.slots * 1000003u ^ (size_t)k.m * 7919u ^ (size_t)k.nj;
        for (int i = 0; i < k.nj; ++i)
            for (int f = 0; f < 3; ++f) h = h * 1099511628211ull ^ (size_t)k.shape[i][f];
        return h;
    }
};

// Job order of a launch: the ready jobs (the first n_ready) before the others, each class by
// decreasing unit bytes (stable).
static void unit_order(int nj, const int64_t* tile_bytes, const int* parts, int* perm, int n_ready = 0) {
    for (int i = 0; i < nj; ++i) perm[i] = i;
    auto before = [&](int a, int b) {
        const bool ra = a < n_ready, rb = b < n_ready;
        if (ra != rb) return ra;
        return tile_bytes[a] * parts[b] > tile_bytes[b] * parts[a];
    };
    for (int i = 1; i < nj; ++i)  // stable insertion sort
        for (int k = i; k > 0 && before(perm[k], perm[k - 1]); --k) std::swap(perm[k], perm[k - 1]);
}

static void choose_parts(const PartsKey& key, int* parts_out) {
    static std::mutex mu;
    static std::unordered_map<PartsKey, std::vector<int>, PartsKeyHash> cache;
    {
        std::lock_guard<std::mutex> lock(mu);
        auto it = cache.find(key);
        if (it != cache.end()) {
            for (int i = 0; i < key.nj; ++i) parts_out[i] = it->second[i];
            return;
        }
    }
    const int nj = key.nj;
    int tiles[kMaxJobs], parts[kMaxJobs], max_parts[kMaxJobs];
    int64_t tile_bytes[kMaxJobs];
    double total = 0.0;
    for (int i = 0; i < nj; ++i) {
        tiles[i] = (int)key.shape[i][0];
        tile_bytes[i] = key.shape[i][1];
        max_parts[i] = std::max(1, (int)std::min<int64_t>(std::min<int64_t>(8, key.shape[i][2]), tile_bytes[i] >> 15));
        parts[i] = 1;
        total += (double)tiles[i] * tile_bytes[i];
    }
    const int stride = 2 * (key.m > 8 ? 2 : 1) * 128;
    auto makespan = [&]() {
        int perm[kMaxJobs];
        unit_order(nj, tile_bytes, parts, perm);
        std::vector<double> ub;
        for (int i = 0; i < nj; ++i)
            for (int t = 0; t < tiles[perm[i]] * parts[perm[i]]; ++t) ub.push_back((double)tile_bytes[perm[i]] / parts[perm[i]]);
        return greedy_makespan(ub, key.slots);
    };
    auto scratch_ok = [&]() {
        int64_t f = 0, t = 0;
        for (int i = 0; i < nj; ++i)
            if (parts[i] > 1) f += (int64_t)tiles[i] * parts[i] * stride, t += tiles[i];
        return f <= kSplitFloats && t <= kSplitTiles;
    };
    const double stream = total / kCtaShare;  // the streaming time, in bytes of one CTA
    auto model = [&]() { return std::max(stream, makespan()); };
    double best_t = model();
    int best[kMaxJobs];
    for (int i = 0; i < nj; ++i) best[i] = parts[i];
    for (;;) {
        int cut = -1;  // the job with the largest units that can still be cut
        for (int i = 0; i < nj; ++i)
            if (parts[i] < max_parts[i] && (cut < 0 || tile_bytes[i] * parts[cut] > tile_bytes[cut] * parts[i])) cut = i;
        if (cut < 0) break;
        ++parts[cut];
        if (!scratch_ok()) break;
        const double t = model();
        if (t < 0.98 * best_t) {
            best_t = t;
            for (int i = 0; i < nj; ++i) best[i] = parts[i];
        }
    }
    std::lock_guard<std::mutex> lock(mu);
    cache.emplace(key, std::vector<int>(best, best + nj));
    for (int i = 0; i < nj; ++i) parts_out[i] = best[i];
}

// Plans a grouped launch: K parts per tile (choose_parts), jobs ordered by unit size (largest
// first, so that the last units claimed are the small ones; the peer destinations are permuted
// alike), unit numbering, this launch's counter and scratch.  Returns the grid size (every CTA slot,
// or one CTA per unit if there are fewer), 0 if the device buffers are unavailable.
static int plan_units(GemvGroup& grp, PeerSync& ps, int slots, int m, int lane) {
    const int nj = grp.njobs;
    int parts[kMaxJobs] = {}, tiles[kMaxJobs] = {};
    int64_t tile_bytes[kMaxJobs] = {};
    PartsKey key{};
    key.slots = slots;
    key.m = m;
    key.nj = nj;
    for (int i = 0; i < nj; ++i) {
        const GemvJob& jb = grp.job[i];
        tiles[i] = (int)ceil_div(jb.n, 16);
        tile_bytes[i] = (int64_t)jb.kt_total * (jb.w1 ? 2 : 1) * kTileBytes;
        key.shape[i][0] = tiles[i];
        key.shape[i][1] = tile_bytes[i];
        key.shape[i][2] = jb.kt_total / jb.chunk_tiles;
    }
    choose_parts(key, parts);
    const int stride = 2 * (m > 8 ? 2 : 1) * 128;  // floats per part partial (entries of both matrices)
    int perm[kMaxJobs];
    unit_order(nj, tile_bytes, parts, perm, grp.n_ready);
    GemvGroup sorted = grp;
    PeerSync pss = ps;
    int units = 0, split_tiles = 0;
    int64_t split_floats = 0;
    for (int i = 0; i < nj; ++i) {
        const int q = perm[i];
        sorted.job[i] = grp.job[q];
        for (int p = 0; p < kMaxPeers; ++p) pss.y[i][p] = ps.y[q][p];
        sorted.job[i].n_tiles = tiles[q];
        sorted.parts[i] = parts[q];
        sorted.split_base[i] = split_tiles;
        sorted.split_fbase[i] = split_floats;
        if (parts[q] > 1) {
            split_tiles += tiles[q];
            split_floats += (int64_t)tiles[q] * parts[q] * stride;
        }
        sorted.unit_begin[i] = units;
        units += tiles[q] * parts[q];
    }
    sorted.unit_begin[nj] = units;
    sorted.total_units = units;
    sorted.split_stride = stride;
    const UnitBuffers* ub = unit_buffers();
    if (!ub) return 0;
    int dev = 0;
    cudaGetDevice(&dev);
    const unsigned slot = g_lane_launches[dev & 63][lane].fetch_add(1);
    const size_t region = (size_t)lane * kSplitRegions + slot % kSplitRegions;
    sorted.claim = ub->claim + 2 * ((size_t)lane * kClaimSlots + slot % kClaimSlots);
    sorted.split_scratch = ub->split + region * kSplitFloats;
    sorted.split_count = ub->split_count + region * kSplitTiles;
    grp = sorted;
    ps = pss;
    if (SBQ_GEMV_SPREAD && units >= sm_count()) {
        // at least one unit per SM: the whole grid, first units dealt across the SMs
        grp.spread = slots / sm_count();
        return slots;
    }
    return units < slots ? units : slots;
}

template <bool PEER>
static int dispatch_group_t(GemvGroup& grp, PeerSync ps, int xk, int mt, cudaStream_t s) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return check_launch("cudaGetDevice");
    const int ctas = plan_units(grp, ps, (mt == 2 ? kCtasPerSm16 : kCtasPerSm) * sm_count(), grp.job[0].m,
                                stream_lane(s, dev));
    if (ctas <= 0) return set_error(SBQ_ERR_CUDA, "grouped GEMV: no work counter on this device");
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
    return SBQ_OK;
}

static int dispatch_group(GemvGroup& grp, int xk, int mt, cudaStream_t s) {
    const PeerSync none{};
    return dispatch_group_t<false>(grp, none, xk, mt, s);
}

SBQ_DEFINE_ERROR_POLL(poll_error_gemv)

// ---------------------------------------------------------------------------------------------
// Fused rank-r pair of projections y = B(A(x)) (the LoRA pairs lora_q_proj / lora_k_proj of the
// hybrid block, model.py:287-288: Linear(hidden -> 128) then Linear(128 -> heads * head_dim)), at
// decode sizes in one launch.  A cluster of 8 CTAs computes t = A(x) once: CTA c owns rows
// 16 c .. 16 c + 15 of A (its eight warps split the K range; partial sums added in warp order, the
// fp32 per-row scale applied after the dot product as in Int8Linear), and every CTA then gathers all
// of t [m, r] from the cluster's shared memory (distributed shared memory) - t never leaves the SMs.
// Each cluster then streams its share of B's 16-row tiles, one tile per warp, with t as an fp32
// activation (split into bf16 high + low parts, as the GEMV does for fp32 x).  Several clusters
// cover B; each recomputes t (A is small: r x hidden bytes, from L2).
constexpr int kLoraCluster = 8;
constexpr int kLoraMaxR = 16 * kLoraCluster;  // 128
constexpr int kLoraThreads = 256;
constexpr int kLoraTPad = kLoraMaxR + 4;      // row stride of the gathered t (floats; 16-byte rows)

struct LoraParams {
    const void* x;
    int64_t ldx;
    int m, k, kt;          // kt = ceil(k / 64)
    const int8_t* wa;      // packed [r, k]
    const float* sa;
    int r, kt_b;           // kt_b = ceil(r / 64)
    const int8_t* wb;      // packed [n, r]
    const float* sb;
    int n, n_tiles, tiles_per_cta;
    void* y;
    int64_t ldy;
    int out_f16;
};

template <int XK, int MT>
__global__ void __launch_bounds__(kLoraThreads, 1) lora_pair_kernel(const LoraParams p) {
    __shared__ float red[kGemvWarps][MT * 8][17];                       // per-warp partials [token][row]
    __shared__ __align__(16) float t_loc[MT * 8][16];                   // this CTA's 16 columns of t
    __shared__ __align__(16) float t_full[MT * 8][kLoraTPad];           // t [token][0, r)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, c = lane & 3;
    const int rank = (int)tc::cluster_ctarank();

    // ---- stage 1: rows 16 rank .. of A, the K tiles split over the warps
    float acc[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[mt][e] = 0.0f;
    if (16 * rank < p.r) {
        for (int kt = warp; kt < p.kt; kt += kGemvWarps) {
            const int8_t* t = p.wa + ((int64_t)rank * p.kt + kt) * kTileBytes + lane * 16;
            const uint4 wa = ld_stream(t), wb = ld_stream(t + 512);
            XFrag<XK> xf[MT];
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) load_x<XK>(xf[mt], p.x, p.ldx, 8 * mt + g, p.m, (int64_t)kt * kTileCols + 16 * c, p.k);
            tile_mma<XK, MT>(acc, wa, wb, xf);
        }
    }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
        red[warp][8 * mt + 2 * c][g] = acc[mt][0];
        red[warp][8 * mt + 2 * c + 1][g] = acc[mt][1];
        red[warp][8 * mt + 2 * c][g + 8] = acc[mt][2];
        red[warp][8 * mt + 2 * c + 1][g + 8] = acc[mt][3];
    }
    __syncthreads();
    if (threadIdx.x < MT * 8 * 16) {
        const int rr = threadIdx.x & 15, tok = threadIdx.x >> 4, ch = 16 * rank + rr;
        float v = 0.0f;
#pragma unroll
        for (int w = 0; w < kGemvWarps; ++w) v += red[w][tok][rr];
        t_loc[tok][rr] = ch < p.r ? __fmul_rn(v, p.sa[ch]) : 0.0f;
    }
    tc::cluster_sync();  // every CTA's 16 columns of t are written
    for (int e = threadIdx.x; e < MT * 8 * (kLoraMaxR / 4); e += kLoraThreads) {
        const int tok = e / (kLoraMaxR / 4), q = e % (kLoraMaxR / 4);  // q: 4-column group
        const int src = q / 4, col = (q % 4) * 4;
        const uint4 v = tc::ld_cluster_v4(tc::cluster_addr(&t_loc[tok][col], (uint32_t)src));
        *reinterpret_cast<uint4*>(&t_full[tok][src * 16 + col]) = v;
    }
    tc::cluster_sync();  // t gathered everywhere (and no CTA leaves while another reads its t_loc)

    // ---- stage 2: this CTA's 16-row tiles of B, one per warp, t as an fp32 activation
    for (int ti = warp; ti < p.tiles_per_cta; ti += kGemvWarps) {
        const int tile = blockIdx.x * p.tiles_per_cta + ti;
        if (tile >= p.n_tiles) break;
        float acc2[MT][4];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc2[mt][e] = 0.0f;
        for (int kt = 0; kt < p.kt_b; ++kt) {
            const int8_t* t = p.wb + ((int64_t)tile * p.kt_b + kt) * kTileBytes + lane * 16;
            const uint4 wa = ld_stream(t), wb = ld_stream(t + 512);
            XFrag<kXF32> xf[MT];
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
                load_x<kXF32>(xf[mt], &t_full[0][0], kLoraTPad, 8 * mt + g, p.m, (int64_t)kt * kTileCols + 16 * c, p.r);
            tile_mma<kXF32, MT>(acc2, wa, wb, xf);
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int rrow = g + (e >> 1) * 8, tok = 8 * mt + 2 * c + (e & 1);
                const int nn = tile * 16 + rrow;
                if (nn >= p.n || tok >= p.m) continue;
                const float v = __fmul_rn(acc2[mt][e], p.sb[nn]);
                if (p.out_f16)
                    static_cast<__half*>(p.y)[(int64_t)tok * p.ldy + nn] = __float2half_rn(v);
                else
                    static_cast<float*>(p.y)[(int64_t)tok * p.ldy + nn] = v;
            }
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
    const int cmax = w1 ? 8 : 16;  // a chunk is 16 KiB: 16 tiles of one matrix or 8 of each of two
    jb.chunk_tiles = jb.kt_total % cmax == 0 ? cmax : jb.kt_total % 8 == 0 ? 8 : jb.kt_total % 4 == 0 ? 4 : jb.kt_total % 2 == 0 ? 2 : 1;
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
        const int st = dispatch_group(grp, x_kind(x_dtype), q.m > 8 ? 2 : 1, s);
        if (st) return st;
    }
    return check_launch(what);
}

}  // namespace sbq

using namespace sbq;

extern "C" int sbq_gemv_plan_parts(const int64_t* shapes, int njobs, int slots, int64_t m, int* parts) {
    if (!shapes || !parts || njobs < 1 || njobs > kMaxJobs || slots < 1 || m < 1 || m > 16)
        return set_error(SBQ_ERR_INVALID_ARGUMENT, "plan: 1..%d jobs, slots >= 1, 1 <= m <= 16", kMaxJobs);
    PartsKey key{};
    key.slots = slots;
    key.m = (int)m;
    key.nj = njobs;
    for (int i = 0; i < njobs; ++i) {
        const int64_t n = shapes[3 * i], k = shapes[3 * i + 1], nmat = shapes[3 * i + 2];
        if (n < 1 || k < 1 || k % 16 || (nmat != 1 && nmat != 2))
            return set_error(SBQ_ERR_INVALID_ARGUMENT, "plan: job %d needs n >= 1, k a positive multiple of 16, "
                             "1 or 2 matrices", i);
        GemvJob jb;
        fill_job(jb, nullptr, k, nullptr, nullptr, nmat == 2 ? reinterpret_cast<const void*>(1) : nullptr, nullptr,
                 nullptr, n, k, nullptr, SBQ_F32, n);
        key.shape[i][0] = ceil_div(n, 16);
        key.shape[i][1] = (int64_t)jb.kt_total * nmat * kTileBytes;
        key.shape[i][2] = jb.kt_total / jb.chunk_tiles;
    }
    choose_parts(key, parts);
    return SBQ_OK;
}

extern "C" int sbq_gemv_w8(const void* x, int x_dtype, int64_t ldx, const void* packed, const float* scale,
                           const float* bias, int64_t m, int64_t n, int64_t k, void* y, int y_dtype, int64_t ldy,
                           void* stream) {
    int st = check_linear_args(x, x_dtype, ldx, packed, scale, m, n, k, y, y_dtype, ldy);
    if (st) return st;
    GemvJob jb;
    fill_job(jb, x, ldx, packed, scale, nullptr, nullptr, bias, n, k, y, y_dtype, ldy);
    return run_single(jb, m, x_dtype, y_dtype, static_cast<cudaStream_t>(stream), "gemv_w8");
}

namespace sbq {
int gemm_w8a16_run(const void* x, int x_dtype, int64_t ldx, const void* packed, const float* scale, const float* bias,
                   int64_t m, int64_t n, int64_t k, void* y, int y_dtype, int64_t ldy, void* stream, int gated);
int gemm_w8a16_run_x2(const void* hi, const void* lo, int64_t ldx, const void* packed, const float* scale,
                      const float* bias, int64_t m, int64_t n, int64_t k, void* y, int y_dtype, int64_t ldy, void* stream,
                      int gated);
int split_into_workspace(const void* x, int64_t ldx, int64_t m, int64_t k, void* workspace, size_t workspace_bytes,
                         void** hi, void** lo, void* stream);
}

// Above kGemmMinRows rows of x the gate/up pair runs as two tensor-memory GEMMs (the gate projection
// into h, then the up projection whose epilogue turns h into silu(gate) * up) instead of the fused GEMV.
constexpr int64_t kGateUpGemmMinRows = kGemmMinRows;

extern "C" int sbq_mlp_gateup_w8(const void* x, int x_dtype, int64_t ldx, const void* packed_gate,
                                 const float* scale_gate, const void* packed_up, const float* scale_up, int64_t m,
                                 int64_t n, int64_t k, void* h, int h_dtype, int64_t ldh, void* stream) {
    int st = check_linear_args(x, x_dtype, ldx, packed_gate, scale_gate, m, n, k, h, h_dtype, ldh);
    if (st) return st;
    if (!packed_up || !scale_up) return set_error(SBQ_ERR_INVALID_ARGUMENT, "null up-projection pointer");
    if (reinterpret_cast<uintptr_t>(packed_up) % 256) return set_error(SBQ_ERR_ALIGNMENT, "packed weight must be 256-byte aligned");
    if (m > kGateUpGemmMinRows && (x_dtype == SBQ_F16 || x_dtype == SBQ_BF16)) {
        st = gemm_w8a16_run(x, x_dtype, ldx, packed_gate, scale_gate, nullptr, m, n, k, h, h_dtype, ldh, stream, 0);
        if (st) return st;
        return gemm_w8a16_run(x, x_dtype, ldx, packed_up, scale_up, nullptr, m, n, k, h, h_dtype, ldh, stream, 1);
    }
    GemvJob jb;
    fill_job(jb, x, ldx, packed_gate, scale_gate, packed_up, scale_up, nullptr, n, k, h, h_dtype, ldh);
    return run_single(jb, m, x_dtype, h_dtype, static_cast<cudaStream_t>(stream), "mlp_gateup_w8");
}

extern "C" int sbq_mlp_gateup_w8_ws(const void* x, int x_dtype, int64_t ldx, const void* packed_gate,
                                    const float* scale_gate, const void* packed_up, const float* scale_up, int64_t m,
                                    int64_t n, int64_t k, void* h, int h_dtype, int64_t ldh, void* workspace,
                                    size_t workspace_bytes, void* stream) {
    if (m > kGateUpGemmMinRows && x_dtype == SBQ_F32) {
        int st = check_linear_args(x, x_dtype, ldx, packed_gate, scale_gate, m, n, k, h, h_dtype, ldh);
        if (st) return st;
        if (!packed_up || !scale_up) return set_error(SBQ_ERR_INVALID_ARGUMENT, "null up-projection pointer");
        if (reinterpret_cast<uintptr_t>(packed_up) % 256) return set_error(SBQ_ERR_ALIGNMENT, "packed weight must be 256-byte aligned");
        void *hi = nullptr, *lo = nullptr;
        st = split_into_workspace(x, ldx, m, k, workspace, workspace_bytes, &hi, &lo, stream);
        if (st) return st;
        st = gemm_w8a16_run_x2(hi, lo, k, packed_gate, scale_gate, nullptr, m, n, k, h, h_dtype, ldh, stream, 0);
        if (st) return st;
        return gemm_w8a16_run_x2(hi, lo, k, packed_up, scale_up, nullptr, m, n, k, h, h_dtype, ldh, stream, 1);
    }
    return sbq_mlp_gateup_w8(x, x_dtype, ldx, packed_gate, scale_gate, packed_up, scale_up, m, n, k, h, h_dtype, ldh,
                             stream);
}

template <int XK, int MT>
static cudaError_t launch_lora(const LoraParams& lp, int clusters, cudaStream_t s) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)(kLoraCluster * clusters));
    cfg.blockDim = dim3(kLoraThreads);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kLoraCluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, lora_pair_kernel<XK, MT>, lp);
}

extern "C" int sbq_lora_pair_w8(const void* x, int x_dtype, int64_t ldx, const void* packed_a, const float* scale_a,
                                const void* packed_b, const float* scale_b, int64_t m, int64_t r, int64_t n, int64_t k,
                                void* y, int y_dtype, int64_t ldy, void* stream) {
    int st = check_linear_args(x, x_dtype, ldx, packed_a, scale_a, m, r, k, y, y_dtype, ldy);
    if (st) return st;
    if (!packed_b || !scale_b) return set_error(SBQ_ERR_INVALID_ARGUMENT, "null second-stage pointer");
    if (reinterpret_cast<uintptr_t>(packed_b) % 256) return set_error(SBQ_ERR_ALIGNMENT, "packed weight must be 256-byte aligned");
    if (m > 16) return set_error(SBQ_ERR_UNSUPPORTED, "the fused pair takes 1..16 rows of x (m=%lld)", (long long)m);
    if (r % 16 || r > kLoraMaxR)
        return set_error(SBQ_ERR_UNSUPPORTED, "the pair's inner size must be a multiple of 16 up to %d (r=%lld)", kLoraMaxR,
                         (long long)r);
    if (n <= 0 || n >= (int64_t(1) << 31) || ldy < n) return set_error(SBQ_ERR_INVALID_ARGUMENT, "bad output size or stride");
    LoraParams lp{};
    lp.x = x;
    lp.ldx = ldx;
    lp.m = (int)m;
    lp.k = (int)k;
    lp.kt = (int)ceil_div(k, kTileCols);
    lp.wa = static_cast<const int8_t*>(packed_a);
    lp.sa = scale_a;
    lp.r = (int)r;
    lp.kt_b = (int)ceil_div(r, kTileCols);
    lp.wb = static_cast<const int8_t*>(packed_b);
    lp.sb = scale_b;
    lp.n = (int)n;
    lp.n_tiles = (int)ceil_div(n, 16);
    // one B tile per warp: 64 tiles per cluster of 8 CTAs
    const int clusters = (int)ceil_div(lp.n_tiles, kLoraCluster * kGemvWarps);
    lp.tiles_per_cta = (int)ceil_div(lp.n_tiles, kLoraCluster * clusters);
    lp.y = y;
    lp.ldy = ldy;
    lp.out_f16 = y_dtype == SBQ_F16;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool two = m > 8;
    cudaError_t e;
    switch (x_kind(x_dtype)) {
        case kXF16: e = two ? launch_lora<kXF16, 2>(lp, clusters, s) : launch_lora<kXF16, 1>(lp, clusters, s); break;
        case kXBF16: e = two ? launch_lora<kXBF16, 2>(lp, clusters, s) : launch_lora<kXBF16, 1>(lp, clusters, s); break;
        default: e = two ? launch_lora<kXF32, 2>(lp, clusters, s) : launch_lora<kXF32, 1>(lp, clusters, s); break;
    }
    if (e != cudaSuccess) return set_error(SBQ_ERR_CUDA, "lora pair launch: %s", cudaGetErrorString(e));
    return check_launch("lora_pair_w8");
}

extern "C" int sbq_gemv_w8_group_ready(const sbq_gemv_job* jobs, int njobs, int n_ready, int x_dtype, int64_t m,
                                       void* stream) {
    if (!jobs || njobs < 1 || njobs > kMaxJobs)
        return set_error(SBQ_ERR_INVALID_ARGUMENT, "njobs must be 1..%d", kMaxJobs);
    if (n_ready < 0 || n_ready > njobs) return set_error(SBQ_ERR_INVALID_ARGUMENT, "n_ready must be 0..njobs");
    if (m < 1 || m > 16) return set_error(SBQ_ERR_UNSUPPORTED, "a grouped launch takes 1..16 rows of x (m=%lld)", (long long)m);
    GemvGroup grp{};
    grp.njobs = njobs;
    grp.n_ready = n_ready;
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
    const int st = dispatch_group(grp, x_kind(x_dtype), m > 8 ? 2 : 1, s);
    if (st) return st;
    return check_launch("gemv_w8_group");
}

extern "C" int sbq_gemv_w8_group(const sbq_gemv_job* jobs, int njobs, int x_dtype, int64_t m, void* stream) {
    return sbq_gemv_w8_group_ready(jobs, njobs, 0, x_dtype, m, stream);
}

extern "C" int sbq_gemv_w8_group_peer_ready(const sbq_gemv_job* jobs, int njobs, int n_ready, int x_dtype, int64_t m,
                                            const sbq_peer_group* peers, void* stream) {
    if (!peers) return set_error(SBQ_ERR_INVALID_ARGUMENT, "null peer description");
    if (!jobs || njobs < 1 || njobs > kMaxJobs)
        return set_error(SBQ_ERR_INVALID_ARGUMENT, "njobs must be 1..%d", kMaxJobs);
    if (n_ready < 0 || n_ready > njobs) return set_error(SBQ_ERR_INVALID_ARGUMENT, "n_ready must be 0..njobs");
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
    ps.wait_limit_ns = pg.wait_limit_ns ? pg.wait_limit_ns : kPeerWaitLimitNs;
    for (int p = 0; p < pg.nranks; ++p) {
        if (!pg.signal[p] || reinterpret_cast<uintptr_t>(pg.signal[p]) % 128)
            return set_error(SBQ_ERR_INVALID_ARGUMENT, "signal[%d] must be a 128-byte aligned device pointer", p);
        ps.signal[p] = pg.signal[p];
    }
    GemvGroup grp{};
    grp.njobs = njobs;
    grp.n_ready = n_ready;
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
    const int st = dispatch_group_t<true>(grp, ps, x_kind(x_dtype), m > 8 ? 2 : 1, static_cast<cudaStream_t>(stream));
    if (st) return st;
    return check_launch("gemv_w8_group_peer");
}

extern "C" int sbq_gemv_w8_group_peer(const sbq_gemv_job* jobs, int njobs, int x_dtype, int64_t m,
                                      const sbq_peer_group* peers, void* stream) {
    return sbq_gemv_w8_group_peer_ready(jobs, njobs, 0, x_dtype, m, peers, stream);
}

extern "C" int sbq_peer_wait(const unsigned* count, unsigned* state, unsigned expected, unsigned long long limit_ns,
                             void* stream) {
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
    cudaLaunchKernelEx(&cfg, peer_wait_kernel, count, state, expected, limit_ns ? limit_ns : kPeerWaitLimitNs);
    return check_launch("peer_wait");
}

// ---- decode program: build (once, synchronous) and run (per step, capturable) ---------------------
static int program_ctas() { return kCtasPerSm * sm_count(); }

static size_t program_bytes_for(int nstages) { return 256 + (size_t)nstages * sizeof(ProgStage); }

extern "C" size_t sbq_gemv_program_bytes(int nstages) {
    if (nstages < 1) return 0;
    return program_bytes_for(nstages);
}

extern "C" size_t sbq_gemv_program_sync_bytes(int nstages) {
    if (nstages < 1) return 0;
    return (size_t)nstages * kSyncStageBytes;
}

// Programs built by sbq_gemv_program_build_peer (the run picks the sharded kernel for them).
static std::mutex g_peer_programs_mu;
static std::unordered_set<const void*> g_peer_programs;

// Shared by the single-GPU and the sharded build.  ydest: null, or [njobs][nranks] destinations.
static int program_build(const sbq_gemv_job* jobs, const int* job_stage, int njobs, int x_dtype, int64_t m,
                         void* const* ydest, int nranks, void* const* peer_sync, void* program, size_t program_bytes) {
    if (!jobs || !job_stage || njobs < 1 || !program) return set_error(SBQ_ERR_INVALID_ARGUMENT, "null argument");
    if (x_kind(x_dtype) < 0) return set_error(SBQ_ERR_UNSUPPORTED, "activation dtype %d", x_dtype);
    if (reinterpret_cast<uintptr_t>(program) % 256) return set_error(SBQ_ERR_ALIGNMENT, "program must be 256-byte aligned");
    if (m < 1 || m > 8) return set_error(SBQ_ERR_UNSUPPORTED, "a program takes 1..8 rows of x (m=%lld)", (long long)m);
    int nstages = 0;
    for (int i = 0; i < njobs; ++i) {
        if (job_stage[i] < 0 || (i > 0 && job_stage[i] < job_stage[i - 1]))
            return set_error(SBQ_ERR_INVALID_ARGUMENT, "job stages must be non-negative and non-decreasing");
        if (job_stage[i] + 1 > nstages) nstages = job_stage[i] + 1;
    }
    if (program_bytes < program_bytes_for(nstages))
        return set_error(SBQ_ERR_WORKSPACE, "program needs %zu bytes", program_bytes_for(nstages));
    const int nctas = program_ctas();
    std::vector<uint8_t> host(program_bytes_for(nstages), 0);
    ProgHeader* hdr = reinterpret_cast<ProgHeader*>(host.data());
    std::vector<ProgStage> stages(nstages);
    for (auto& ps : stages) {
        ps.grp = GemvGroup{};
        ps.peer = PeerSync{};
        ps.peer.nranks = nranks;
    }
    for (int i = 0; i < njobs; ++i) {
        const sbq_gemv_job& j = jobs[i];
        int st = check_linear_args(j.x, x_dtype, j.ldx, j.packed, j.scale, m, j.n, j.k, j.y, j.y_dtype, j.ldy);
        if (st) return set_error(st, "job %d: %s", i, sbq_last_error());
        if (j.packed_up && (!j.scale_up || j.bias))
            return set_error(SBQ_ERR_INVALID_ARGUMENT, "job %d: fused gate/up job needs scale_up and no bias", i);
        ProgStage& ps = stages[job_stage[i]];
        if (ps.grp.njobs >= kMaxJobs) return set_error(SBQ_ERR_UNSUPPORTED, "more than %d jobs in one stage", kMaxJobs);
        const int jj = ps.grp.njobs++;
        fill_job(ps.grp.job[jj], j.x, j.ldx, j.packed, j.scale, j.packed_up, j.scale_up, j.bias, j.n, j.k, j.y,
                 j.y_dtype, j.ldy);
        ps.grp.job[jj].m = (int)m;
        if (ydest) {
            bool local = false;
            for (int r = 0; r < nranks; ++r) {
                void* d = ydest[(size_t)i * nranks + r];
                if (!d) return set_error(SBQ_ERR_INVALID_ARGUMENT, "job %d: null destination for rank %d", i, r);
                local = local || d == j.y;
                ps.peer.y[jj][r] = d;
            }
            if (!local) return set_error(SBQ_ERR_INVALID_ARGUMENT, "job %d: y must be one of its rank destinations", i);
        }
    }
    // each stage is planned as a grouped launch over the program's grid (units, K parts, largest
    // first); its split scratch alternates between the two regions stage by stage (stage s + 2
    // starts only after stage s + 1's barrier, so after every use of stage s's region)
    const UnitBuffers* ub = unit_buffers();
    if (!ub) return set_error(SBQ_ERR_CUDA, "decode program: no device work buffers");
    for (int st = 0; st < nstages; ++st) {
        ProgStage& ps = stages[st];
        if (ps.grp.njobs == 0) continue;
        if (plan_units(ps.grp, ps.peer, nctas, (int)m, kProgramLane) <= 0) return set_error(SBQ_ERR_CUDA, "decode program plan");
        ps.grp.claim = nullptr;  // the stage's claim pair lives in the run's sync region
        const size_t region = (size_t)kProgramLane * kSplitRegions + st % kSplitRegions;
        ps.grp.split_scratch = ub->split + region * kSplitFloats;
        ps.grp.split_count = ub->split_count + region * kSplitTiles;
    }
    std::memcpy(host.data() + 256, stages.data(), (size_t)nstages * sizeof(ProgStage));
    hdr->nstages = nstages;
    hdr->nctas = nctas;
    hdr->x_dtype = x_dtype;
    hdr->m = (int)m;
    hdr->nranks = nranks;
    for (int r = 0; r < nranks && peer_sync; ++r) hdr->peer_sync[r] = static_cast<uint8_t*>(peer_sync[r]);
    if (cudaMemcpy(program, host.data(), host.size(), cudaMemcpyHostToDevice) != cudaSuccess)
        return check_launch("copy decode program");
    std::lock_guard<std::mutex> lock(g_peer_programs_mu);
    if (nranks > 1)
        g_peer_programs.insert(program);
    else
        g_peer_programs.erase(program);
    return SBQ_OK;
}

extern "C" int sbq_gemv_program_build(const sbq_gemv_job* jobs, const int* job_stage, int njobs, int x_dtype, int64_t m,
                                      void* program, size_t program_bytes) {
    return program_build(jobs, job_stage, njobs, x_dtype, m, nullptr, 1, nullptr, program, program_bytes);
}

extern "C" int sbq_gemv_program_build_peer(const sbq_gemv_job* jobs, const int* job_stage, int njobs, int x_dtype,
                                           int64_t m, void* const* ydest, int nranks, void* const* peer_sync,
                                           void* program, size_t program_bytes) {
    if (!ydest || !peer_sync) return set_error(SBQ_ERR_INVALID_ARGUMENT, "null destination or sync table");
    if (nranks < 2 || nranks > kMaxPeers)
        return set_error(SBQ_ERR_INVALID_ARGUMENT, "a sharded program has 2..%d ranks (got %d)", kMaxPeers, nranks);
    for (int r = 0; r < nranks; ++r)
        if (!peer_sync[r] || reinterpret_cast<uintptr_t>(peer_sync[r]) % 128)
            return set_error(SBQ_ERR_ALIGNMENT, "sync region of rank %d must be 128-byte aligned", r);
    return program_build(jobs, job_stage, njobs, x_dtype, m, ydest, nranks, peer_sync, program, program_bytes);
}

template <int XK, bool PEER>
static cudaError_t launch_program(const cudaLaunchConfig_t& cfg, const ProgParams& pp) {
    cudaFuncSetAttribute(gemv_program_kernel<XK, PEER>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)cfg.dynamicSmemBytes);
    return cudaLaunchKernelEx(&cfg, gemv_program_kernel<XK, PEER>, pp);
}

extern "C" int sbq_gemv_program_run(const void* program, int nstages, int x_dtype, void* sync, void* stream) {
    if (!program || !sync || nstages < 1) return set_error(SBQ_ERR_INVALID_ARGUMENT, "null argument");
    if (reinterpret_cast<uintptr_t>(sync) % 128) return set_error(SBQ_ERR_ALIGNMENT, "sync region must be 128-byte aligned");
    const int xk = x_kind(x_dtype);
    if (xk < 0) return set_error(SBQ_ERR_UNSUPPORTED, "activation dtype %d", x_dtype);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    ProgParams pp{};
    const uint8_t* base = static_cast<const uint8_t*>(program);
    const int nctas = program_ctas();
    pp.hdr = reinterpret_cast<const ProgHeader*>(base);
    pp.stages = reinterpret_cast<const ProgStage*>(base + 256);
    pp.nstages = nstages;
    pp.sync = static_cast<uint8_t*>(sync);
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
    bool peer;
    {
        std::lock_guard<std::mutex> lock(g_peer_programs_mu);
        peer = g_peer_programs.count(program) != 0;
    }
    cudaError_t e;
    switch (xk) {
        case kXF16: e = peer ? launch_program<kXF16, true>(cfg, pp) : launch_program<kXF16, false>(cfg, pp); break;
        case kXBF16: e = peer ? launch_program<kXBF16, true>(cfg, pp) : launch_program<kXBF16, false>(cfg, pp); break;
        default: e = peer ? launch_program<kXF32, true>(cfg, pp) : launch_program<kXF32, false>(cfg, pp); break;
    }
    if (e != cudaSuccess) return set_error(SBQ_ERR_CUDA, "decode program launch: %s", cudaGetErrorString(e));
    return check_launch("gemv_program");
}
