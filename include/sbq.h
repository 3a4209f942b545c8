/*
 * sbq.h - C ABI of the B200 (sm_100a) int8 / int8-dyn quantised-linear library (libsbq.so).
 *
 * Every entry point takes plain device pointers, element counts and a CUDA stream handle
 * (cudaStream_t passed as void*; NULL = the legacy default stream), launches asynchronously on
 * that stream and returns an int status (SBQ_OK = 0).  Nothing here synchronises the device or
 * allocates memory.  Argument errors are detected on the host before any launch.  The last error
 * message of the calling host thread is available from sbq_last_error().
 *
 * Matrices are row-major.  "ld*" arguments are row strides in elements.  Weights are [n, k]
 * (output channels x input features), activations [m, k], outputs [m, n] - the shapes of the
 * reference's nn.Linear replacements.
 *
 * Streams and host threads: the entry points may be called from several host threads and launch on
 * any streams.  The decode GEMV (sbq_linear_w8 up to 16 rows, sbq_gemv_w8, sbq_mlp_gateup_w8,
 * sbq_gemv_w8_group[_peer]) takes a work counter and, for launches whose tiles are cut into K parts,
 * a split-K scratch region from device arrays of the library.  These are divided into 8 lanes per
 * device and each stream is given one lane on first use, so launches on up to 8 distinct streams of
 * a device may run concurrently; a ninth stream shares a lane with an earlier one and must not run
 * GEMV launches at the same time as it.  A CUDA graph keeps the lane of the stream it was captured
 * on: graphs captured on one stream must not be replayed concurrently with each other.  Decode
 * programs (sbq_gemv_program_*) share one further lane: run them on one stream at a time.
 *
 * Packed weights: an int8 [n, k] matrix stored as 16 x 64 tiles of 1 KiB, tile (nt, kt) at byte
 * (nt * ceil(k/64) + kt) * 1024, rows row-major inside the tile, padding zero-filled.  Its size is
 * sbq_packed_bytes(n, k); it must be 256-byte aligned.
 *
 * Reference interfaces replaced (paths inside the reference project, spikingbrain_cpu/):
 *   quant.py:25-29   quantize_per_channel             -> sbq_quantize_pack
 *   quant.py:35-37   Int8Linear qweight/scale buffers  -> sbq_pack_int8 / sbq_unpack_int8
 *   quant.py:41-53   Int8Linear.forward               -> sbq_linear_w8 / sbq_linear_w8_ws
 *                    (sbq_gemv_w8 / sbq_gemm_w8a16 / sbq_split_f32_bf16x2 + sbq_gemm_w8a16_x2)
 *   model.py:239-240 GatedMLP.forward (gate, up, SiLU) -> sbq_mlp_gateup_w8
 *   model.py:287-288 lora_q_proj / lora_k_proj pairs   -> sbq_lora_pair_w8
 *   quant.py:57-61   DynamicInt8Linear packing         -> sbq_quantize_pack (+ row sums)
 *   quant.py:63-66   DynamicInt8Linear.forward        -> sbq_linear_dyn
 *                    (= sbq_quant_act_per_tensor + sbq_gemm_w8a8)
 */
#ifndef SBQ_H_
#define SBQ_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SBQ_API __attribute__((visibility("default")))
#else
#define SBQ_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------------------------- */
#define SBQ_OK 0
#define SBQ_ERR_INVALID_ARGUMENT 1 /* null pointer, negative or inconsistent size, bad stride */
#define SBQ_ERR_ALIGNMENT 2        /* pointer or stride not aligned as the kernel requires    */
#define SBQ_ERR_UNSUPPORTED 3      /* dtype / shape combination this build does not handle    */
#define SBQ_ERR_CUDA 4             /* a CUDA runtime call or kernel launch failed             */
#define SBQ_ERR_TIMEOUT 5          /* a bounded device-side wait expired (error flag set)     */
#define SBQ_ERR_DEVICE 6           /* no device, or not an sm_100 device                      */
#define SBQ_ERR_WORKSPACE 7        /* the workspace passed in is too small                    */

/* ---- element types --------------------------------------------------------------------- */
#define SBQ_F32 0
#define SBQ_F16 1
#define SBQ_BF16 2
#define SBQ_I8 3
#define SBQ_U8 4
#define SBQ_I32 5

/* ---- activation quantisation modes for the int8-dyn path ------------------------------- */
#define SBQ_ACT_PER_TENSOR 0 /* the reference's mode: one uint8 scale + zero point per call */
#define SBQ_ACT_PER_TOKEN 1  /* symmetric int8, one scale per row (no reference counterpart) */

/* ---- library ---------------------------------------------------------------------------- */
SBQ_API int sbq_version(void);                     /* MAJOR * 10000 + MINOR * 100 + PATCH */
SBQ_API const char* sbq_last_error(void);          /* last message of this host thread ("" if none) */
SBQ_API const char* sbq_status_string(int status); /* static name of a status code */

/* Synchronises the current device, then returns (and clears) the error a kernel recorded on the
 * device: SBQ_ERR_TIMEOUT if one of its bounded waits expired, else SBQ_OK.  Diagnostic call; the
 * launch entry points never synchronise. */
SBQ_API int sbq_check_device_error(void);

/* Bytes of the packed layout of an [n, k] int8 weight. */
SBQ_API size_t sbq_packed_bytes(int64_t n, int64_t k);

/* ---- weight preparation (once per weight, at load) -------------------------------------- */

/* quant.py:25-29 on the device: scale[r] = max(max_c |w[r,c]|, 1e-8) / 127 (fp32),
 * q = clamp(rint(w / scale), -127, 127), written in the packed layout.  Bit-identical to the
 * reference.  w is [n, k] with row stride ldw, dtype SBQ_F32, SBQ_BF16 or SBQ_F16.  rowsum (may be
 * NULL) receives sum_c q[r, c] as int32 (used by the int8-dyn zero-point correction). */
SBQ_API int sbq_quantize_pack(const void* w, int w_dtype, int64_t n, int64_t k, int64_t ldw, void* packed,
                      float* scale, int32_t* rowsum, void* stream);

/* Already-quantised int8 [n, k] (row stride ldq) -> packed layout (+ optional row sums).
 * The state-dict load path of the qweight buffer (quant.py:36). */
SBQ_API int sbq_pack_int8(const int8_t* q, int64_t n, int64_t k, int64_t ldq, void* packed, int32_t* rowsum,
                  void* stream);

/* Packed layout -> row-major int8 [n, k] (row stride ldq).  The state-dict save path. */
SBQ_API int sbq_unpack_int8(const void* packed, int64_t n, int64_t k, int8_t* q, int64_t ldq, void* stream);

/* ---- int8 weight-only linear (format "int8") --------------------------------------------- */

/* Int8Linear.forward (quant.py:41-53): y[m, n] = (x[m, :] . q[n, :]) * scale[n] (+ bias[n]).
 * x dtype SBQ_F16, SBQ_BF16 or SBQ_F32 (fp32 is split into two bf16 terms, ~17 significant bits);
 * y dtype SBQ_F32 (the reference's output type) or SBQ_F16.  bias may be NULL.  Chooses the
 * decode GEMV up to 16 rows and the tensor-memory GEMM above for fp16 / bf16 x; fp32 x always
 * takes the GEMV here (its GEMM path needs a workspace: sbq_linear_w8_ws). */
SBQ_API int sbq_linear_w8(const void* x, int x_dtype, int64_t ldx, const void* packed, const float* scale,
                  const float* bias, int64_t m, int64_t n, int64_t k, void* y, int y_dtype, int64_t ldy,
                  void* stream);

/* Bytes of workspace sbq_linear_w8_ws / sbq_mlp_gateup_w8_ws need for x [m, k] of x_dtype: nonzero
 * only for fp32 x above 16 rows (the bf16 high / low parts of x, 4 * m * k bytes rounded up). */
SBQ_API size_t sbq_linear_w8_workspace_bytes(int64_t m, int64_t k, int x_dtype);

/* sbq_linear_w8 with a caller workspace (sbq_linear_w8_workspace_bytes bytes, 256-byte aligned; NULL
 * when that is 0), which puts fp32 activations above 16 rows - the reference's own prefill, fp32
 * x in chunks of up to 512 tokens (model.py:439-441, quant.py:47) - on the tensor-memory GEMM:
 * sbq_split_f32_bf16x2 into the workspace, then sbq_gemm_w8a16_x2.  Other calls behave exactly as
 * sbq_linear_w8. */
SBQ_API int sbq_linear_w8_ws(const void* x, int x_dtype, int64_t ldx, const void* packed, const float* scale,
                             const float* bias, int64_t m, int64_t n, int64_t k, void* y, int y_dtype, int64_t ldy,
                             void* workspace, size_t workspace_bytes, void* stream);

/* The decode GEMV alone (any m >= 1; streams the weight once per 16 rows of x). */
SBQ_API int sbq_gemv_w8(const void* x, int x_dtype, int64_t ldx, const void* packed, const float* scale,
                const float* bias, int64_t m, int64_t n, int64_t k, void* y, int y_dtype, int64_t ldy,
                void* stream);

/* The tensor-memory GEMM alone: TMA-fed, int8 rows converted to x's 16-bit type straight into tensor
 * memory (the MMA's A operand), tcgen05 MMA with fp32 accumulators in tensor memory, scale epilogue.
 * Up to 128 rows of x: 64-token tiles, with the K range split over a thread-block cluster when the
 * tiles are too few for the GPU (partials added through distributed shared memory in part order);
 * more rows: 256-token tiles.  x must be SBQ_F16 or SBQ_BF16. */
SBQ_API int sbq_gemm_w8a16(const void* x, int x_dtype, int64_t ldx, const void* packed, const float* scale,
                   const float* bias, int64_t m, int64_t n, int64_t k, void* y, int y_dtype, int64_t ldy,
                   void* stream);

/* fp32 x [m, k] (row stride ldx) -> bf16 hi = round(x), lo = round(x - hi), [m, k] each with row
 * stride ldo (x - hi is exact, so hi + lo carries ~17 significant bits and fp32's range).  k a
 * multiple of 8; rows 16-byte aligned. */
SBQ_API int sbq_split_f32_bf16x2(const float* x, int64_t ldx, int64_t m, int64_t k, void* hi, void* lo,
                                 int64_t ldo, void* stream);

/* sbq_gemm_w8a16 on an fp32 activation given as its bf16 high and low parts (same row stride ldx):
 * each k-step runs one MMA per part into the same fp32 accumulators against the same converted
 * weight operand - twice the tensor work of a 16-bit x, the GEMV's fp32 accuracy. */
SBQ_API int sbq_gemm_w8a16_x2(const void* x_hi, const void* x_lo, int64_t ldx, const void* packed, const float* scale,
                              const float* bias, int64_t m, int64_t n, int64_t k, void* y, int y_dtype, int64_t ldy,
                              void* stream);

/* GatedMLP.forward's first half (model.py:239-240): h = silu(x q_gate^T * s_gate) * (x q_up^T * s_up)
 * with h written as h_dtype (SBQ_F16 or SBQ_F32).  Up to 16 rows (or fp32 x): one pass over
 * both weights ([n, k] each) in the decode GEMV.  More fp16 / bf16 rows: the gate projection goes into h
 * (rounded to h_dtype) and the up projection's GEMM epilogue replaces it by silu(gate) * up.  The
 * down projection is a separate sbq_linear_w8 call on h. */
SBQ_API int sbq_mlp_gateup_w8(const void* x, int x_dtype, int64_t ldx, const void* packed_gate,
                      const float* scale_gate, const void* packed_up, const float* scale_up, int64_t m,
                      int64_t n, int64_t k, void* h, int h_dtype, int64_t ldh, void* stream);

/* sbq_mlp_gateup_w8 with a caller workspace (sbq_linear_w8_workspace_bytes(m, k, x_dtype) bytes):
 * fp32 x above 16 rows is split once and both GEMMs read the split (see sbq_linear_w8_ws). */
SBQ_API int sbq_mlp_gateup_w8_ws(const void* x, int x_dtype, int64_t ldx, const void* packed_gate,
                                 const float* scale_gate, const void* packed_up, const float* scale_up, int64_t m,
                                 int64_t n, int64_t k, void* h, int h_dtype, int64_t ldh, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* The rank-r projection pair of the hybrid block's LoRA branches (model.py:287-288: lora_q_proj /
 * lora_k_proj = Linear(k -> r) then Linear(r -> n), each an Int8Linear in the int8 format) at decode
 * sizes in one launch: y = ((x q_a^T) * scale_a) q_b^T * scale_b.  The intermediate t [m, r] stays
 * on the SMs (computed once per 8-CTA cluster, gathered through distributed shared memory) in fp32,
 * and the second stage reads it as an fp32 activation (bf16 high + low parts).  1 <= m <= 16;
 * r a multiple of 16, at most 128; packed_a is [r, k], packed_b is [n, r]; y [m, n] fp32 or fp16
 * (row stride ldy).  x dtype SBQ_F16 / SBQ_BF16 / SBQ_F32. */
SBQ_API int sbq_lora_pair_w8(const void* x, int x_dtype, int64_t ldx, const void* packed_a, const float* scale_a,
                             const void* packed_b, const float* scale_b, int64_t m, int64_t r, int64_t n, int64_t k,
                             void* y, int y_dtype, int64_t ldy, void* stream);

/* One projection of a grouped decode launch (sbq_gemv_w8_group).  A job with packed_up set is a fused
 * gate/up job: y = silu(x q^T * scale) * (x q_up^T * scale_up), no bias. */
typedef struct sbq_gemv_job {
    const void* x;         /* activation [m, k], 16-byte aligned rows */
    int64_t ldx;
    const void* packed;    /* packed weight [n, k] (the gate weight of a fused job) */
    const float* scale;
    const void* packed_up; /* packed up weight [n, k], or NULL */
    const float* scale_up;
    const float* bias;     /* [n] or NULL (plain jobs only) */
    int64_t n;
    int64_t k;
    void* y;               /* output [m, n], SBQ_F32 or SBQ_F16 */
    int y_dtype;
    int64_t ldy;
} sbq_gemv_job;

/* Several independent decode GEMVs in one launch (up to 8 jobs sharing the activation dtype and m,
 * 1 <= m <= 16), e.g. the projections of one layer that read the same x (q|k|v|delta_in and gate/up)
 * or that run between the same two dependencies (o, delta_out, down).  Fewer launches per decode
 * step; each job gives the same result as its own sbq_gemv_w8 / sbq_mlp_gateup_w8 call.  The model's
 * shared-input projections (model.py:317-321 and :363-365, sse_q/k/v and swa_q/k/v of one block) are
 * such a group. */
SBQ_API int sbq_gemv_w8_group(const sbq_gemv_job* jobs, int njobs, int x_dtype, int64_t m, void* stream);

/* sbq_gemv_w8_group with the first n_ready jobs (0 <= n_ready <= njobs) marked ready: their x (and
 * everything they read) was complete before the previous kernel on the stream began its work, i.e.
 * it was written two or more kernels back.  Their units run first and do not wait for the previous
 * kernel to end; the other jobs' units wait for it as in sbq_gemv_w8_group.  So a decode step can
 * stream projections whose inputs are older (side outputs, a layer's later consumers) across the
 * boundary that the other jobs must wait at.  Conditions: the previous kernel on the stream is a
 * grouped GEMV launch of this library (sbq_gemv_w8_group[_ready], sbq_gemv_w8, sbq_mlp_gateup_w8,
 * sbq_linear_w8 at decode sizes) or a kernel launched without programmatic dependent launch - those
 * let the next kernel begin only after their own wait for the kernel before them; and a ready job's
 * y is neither read nor written by the previous kernel.  Results are those of sbq_gemv_w8_group. */
SBQ_API int sbq_gemv_w8_group_ready(const sbq_gemv_job* jobs, int njobs, int n_ready, int x_dtype, int64_t m,
                                    void* stream);

/* The K split a grouped launch would choose (host only, no device call): shapes[3 i .. 3 i + 2] =
 * {n, k, matrices (1, or 2 for a fused gate/up job)} of job i, `slots` = CTAs the launch may use (3
 * per SM at every m).  parts[i] receives the K parts of each of job i's
 * 16-row tiles (1 = unsplit).  Deterministic; the launch uses the same plan for the same shapes. */
SBQ_API int sbq_gemv_plan_parts(const int64_t* shapes, int njobs, int slots, int64_t m, int* parts);

/* A decode program: groups of jobs run as stages of ONE persistent launch, stage s + 1 starting after
 * every output of stage s is written (a grid-wide barrier inside the kernel instead of a kernel
 * boundary); the weight stream continues across the barriers.  jobs[i] belongs to stage job_stage[i]
 * (non-decreasing); later stages may read earlier stages' outputs.  Requirement: 1 <= m <= 8.
 * sbq_gemv_program_build lays the program out in `program` (sbq_gemv_program_bytes(nstages) bytes,
 * device memory, 256-byte aligned) and synchronises (a set-up call; the job pointers are baked in).
 * sbq_gemv_program_run launches it; `sync` is sbq_gemv_program_sync_bytes(nstages) bytes of device
 * memory, 128-byte aligned, zero before the first run and left to the program afterwards (its
 * counters only grow, so no run clears anything).  The run is capturable in a CUDA graph.  The
 * buffers named by the jobs must stay allocated. */
SBQ_API size_t sbq_gemv_program_bytes(int nstages);
SBQ_API size_t sbq_gemv_program_sync_bytes(int nstages);
SBQ_API int sbq_gemv_program_build(const sbq_gemv_job* jobs, const int* job_stage, int njobs, int x_dtype, int64_t m,
                                   void* program, size_t program_bytes);
SBQ_API int sbq_gemv_program_run(const void* program, int nstages, int x_dtype, void* sync, void* stream);

/* ---- output-channel shards across the GPUs of one node (peer memory over NVLink) -------------
 *
 * Replaces the all-gather that follows each sharded projection (the output-channel sharding of
 * the model's projections, quant.py:32-53 run per shard; the reference has no multi-GPU path).
 * Every rank allocates one arena with sbq_peer_alloc, exports it with sbq_peer_handle, and maps
 * the other ranks' arenas with sbq_peer_open (the handles travel over any host channel).  All
 * ranks lay their arenas out identically, so a buffer or counter at offset o is at base_p + o on
 * rank p.  The ranks must be different GPUs of one node with peer access (NVLink). */
SBQ_API int sbq_peer_alloc(size_t bytes, void** ptr);          /* zero-filled device memory */
SBQ_API int sbq_peer_free(void* ptr);
SBQ_API int sbq_peer_handle(const void* ptr, void* handle);      /* SBQ_PEER_HANDLE_BYTES out */
SBQ_API int sbq_peer_open(const void* handle, void** ptr);       /* another process's arena */
SBQ_API int sbq_peer_close(void* ptr);
#define SBQ_PEER_HANDLE_BYTES 64
#define SBQ_MAX_PEERS 8

/* One grouped decode launch of a sharded step (see sbq_gemv_w8_group).  Job j's output slice is
 * stored to y[j][p] on every rank p (this rank's slice inside rank p's full-width buffer, as
 * mapped in this process; row stride = the job's ldy; jobs[j].y must be this rank's own entry).
 * The launch's CTAs count themselves out on `done` (one word of this rank's memory, zero at first
 * use); the last one adds 1 to the launch's signal on every rank (signal[p], as mapped here).  A
 * signal is SBQ_PEER_SIGNAL_COPIES words 128 bytes apart (a 4 KiB region, 128-byte aligned, zero
 * at first use), all incremented together so that waiting CTAs poll different lines.  If
 * wait_count is set (this rank's signal of the launch whose output x is), the launch first waits
 * until that signal has received wait_expected (= the number of ranks) more increments than at its
 * previous step.  wait_state: two zero-initialised words of this rank's memory used only by this
 * launch position.  Every wait is bounded (wait_limit_ns, 10 s by default, so ranks may drift apart
 * on the host by that much; then SBQ_ERR_TIMEOUT through sbq_check_device_error, and later waits
 * are skipped until that error has been read).  Ranks must issue the same launches
 * in the same order. */
#define SBQ_PEER_SIGNAL_COPIES 32
#define SBQ_PEER_SIGNAL_BYTES 4096
typedef struct sbq_peer_group {
    int nranks;
    void* y[8][SBQ_MAX_PEERS];
    unsigned* signal[SBQ_MAX_PEERS];
    unsigned* done;
    const unsigned* wait_count;
    unsigned* wait_state;
    unsigned wait_expected;
    unsigned long long wait_limit_ns; /* bound of the wait; 0 = 10 s */
} sbq_peer_group;
SBQ_API int sbq_gemv_w8_group_peer(const sbq_gemv_job* jobs, int njobs, int x_dtype, int64_t m,
                                   const sbq_peer_group* peers, void* stream);
/* sbq_gemv_w8_group_peer with the first n_ready jobs ready (see sbq_gemv_w8_group_ready): their x
 * was gathered on every rank two or more launches back, so their units run before the launch's wait
 * on wait_count, which the other jobs' units take as usual.  Each CTA lets the next launch begin
 * only after its own wait (in every sharded launch), so the launch before the previous one has then
 * completed on every rank.  The previous launch must be a grouped GEMV launch of this library. */
SBQ_API int sbq_gemv_w8_group_peer_ready(const sbq_gemv_job* jobs, int njobs, int n_ready, int x_dtype, int64_t m,
                                         const sbq_peer_group* peers, void* stream);
/* The same wait as a one-CTA launch: the end of a sharded step, before anything else reads the
 * last launch's gathered output.  limit_ns: bound of the wait (0 = 10 s). */
SBQ_API int sbq_peer_wait(const unsigned* count, unsigned* state, unsigned expected, unsigned long long limit_ns,
                          void* stream);

/* A sharded decode program (see sbq_gemv_program_build): the stages' barriers span every rank, and
 * job i's output slice is stored to ydest[i * nranks + p] on every rank p (as mapped here; jobs[i].y
 * must be this rank's own entry).  peer_sync[p]: rank p's sync region (the `sync` it passes to
 * sbq_gemv_program_run, inside its peer arena), as mapped here.  Every rank builds the same stage
 * structure and runs its program once per step; the launch ends when every rank's last-stage
 * outputs have arrived.  Waits are bounded (10 s). */
SBQ_API int sbq_gemv_program_build_peer(const sbq_gemv_job* jobs, const int* job_stage, int njobs, int x_dtype,
                                        int64_t m, void* const* ydest, int nranks, void* const* peer_sync,
                                        void* program, size_t program_bytes);

/* ---- int8-dyn: dynamic activation quantisation + int8 x int8 -> int32 GEMM ------------- */

/* Bytes of workspace sbq_linear_dyn / sbq_quant_act_* need for an [m, k] activation. */
SBQ_API size_t sbq_dyn_workspace_bytes(int64_t m, int64_t k, int mode);

/* Quantise x [m, k] (SBQ_F32 / SBQ_F16 / SBQ_BF16) the way fbgemm's dynamic linear does:
 * per-tensor min/max (widened to 0), torch's ChooseQuantizationParams (uint8, zero point),
 * xq = clamp(rint(fma(x, 1/s, zp)), 0, 255).  Writes xq (uint8 [m, k], row stride k), s_x (1 fp32)
 * and zp (1 int32).  Bit-identical to the reference. */
SBQ_API int sbq_quant_act_per_tensor(const void* x, int x_dtype, int64_t ldx, int64_t m, int64_t k, uint8_t* xq,
                             float* s_x, int32_t* zp, void* workspace, size_t workspace_bytes,
                             void* stream);

/* Per-token symmetric mode: s_t = max(max|x_t|, 1e-8) / 127, xq = clamp(rint(x / s_t), +-127) int8. */
SBQ_API int sbq_quant_act_per_token(const void* x, int x_dtype, int64_t ldx, int64_t m, int64_t k, int8_t* xq,
                            float* s_tok, void* stream);

/* acc[m, n] = sum_k (xq - zp) * q (per-tensor; xq uint8) or sum_k xq * q (per-token; xq int8),
 * y = float(acc) * (s * scale[n]) (or fma with bias[n]).  rowsum is required for the per-tensor
 * mode (zero-point correction).  acc_out (may be NULL) receives the int32 accumulators (row stride n).
 * y and acc_out need only their element alignment (4 bytes): rows whose base pointer is 16-byte
 * aligned, with ldy and n multiples of 4, are written with vector (or TMA) stores, any other layout
 * element by element.  Launched in plain stream order (every input may be the previous kernel's
 * output). */
SBQ_API int sbq_gemm_w8a8(const void* xq, int mode, const void* packed, const int32_t* rowsum, const float* s_x,
                  const int32_t* zp, const float* scale, const float* bias, int64_t m, int64_t n, int64_t k,
                  float* y, int64_t ldy, int32_t* acc_out, void* stream);

/* DynamicInt8Linear.forward (quant.py:63-66): quantise + GEMM + epilogue.  The quantised activation
 * and its parameters live in the workspace (sbq_dyn_workspace_bytes(m, k, mode) bytes, 256-byte
 * aligned).  The quantisation and the GEMM are chained by programmatic dependent launch (the GEMM's
 * set-up and first weight tiles overlap the quantisation); work the caller queues afterwards on the
 * stream runs after the GEMM as usual.  mode: SBQ_ACT_PER_TENSOR (the reference) or
 * SBQ_ACT_PER_TOKEN.  Every argument (those of the GEMM included) is checked before the first
 * launch: a call that returns an error has launched nothing.  y: as for sbq_gemm_w8a8. */
SBQ_API int sbq_linear_dyn(const void* x, int x_dtype, int64_t ldx, int mode, const void* packed,
                   const int32_t* rowsum, const float* scale, const float* bias, int64_t m, int64_t n,
                   int64_t k, float* y, int64_t ldy, void* workspace, size_t workspace_bytes,
                   void* stream);

/* sbq_linear_dyn for callers that cannot allocate device memory.  No counterpart in the reference.
 * Some hosts of this library are not allowed to call cudaMalloc: a runtime that has already handed
 * every byte of HBM to its own pool, a plain C / FFI caller that holds raw pointers but has no
 * allocator, or a latency-critical decode loop where cudaMalloc / cudaFree would synchronise the
 * device.  This entry point allocates nothing (no cudaMalloc, cudaFree or allocating library call):
 * its scratch is a fixed 4 MiB array in the library's device memory, which every GPU that loads the
 * library holds until the process exits.  The caller still passes x, the weight buffers and y.
 * Limit: sbq_dyn_workspace_bytes(m, k, mode) must be <= 4 MiB (m * k up to about 4.18 million,
 * e.g. up to 1020 rows at k = 4096); larger calls return SBQ_ERR_WORKSPACE without launching.  The first
 * call on a device looks up the array's device address (cudaGetSymbolAddress) with that device
 * current; make that first call before any stream capture.  Every call shares the one array and
 * leaves its contents behind, so calls that overlap on the GPU (other streams, other threads) race;
 * order them on one stream. */
SBQ_API int sbq_linear_dyn_noalloc(const void* x, int x_dtype, int64_t ldx, int mode, const void* packed,
                                   const int32_t* rowsum, const float* scale, const float* bias, int64_t m,
                                   int64_t n, int64_t k, float* y, int64_t ldy, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SBQ_H_ */
