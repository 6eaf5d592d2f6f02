/*
 * fp8gq -- fused FP8 (e4m3) activation group-quant + block-scaled GEMV for
 * NVIDIA B200 (sm_100a).  C ABI: plain pointers, sizes and strides; no torch
 * or CUDA types in the signatures.  Every entry point is asynchronous on the
 * given stream, allocates nothing, and returns FP8GQ_OK or an error status
 * (it never aborts the process).
 *
 * Operand conventions, identical to the reference's
 * (wafik/sglang-triton-fusion, kernels/fused_gemv_quant_tm.py:83-102):
 *   x    bf16  [M, K]    row stride ldx elements (>= K)
 *   w    e4m3  [N, K]    row stride ldw bytes (>= K), one byte per weight
 *   ws   fp32  [N/128, K/128]  row stride ldws elements (sglang's
 *                              weight_scale_inv, one scale per 128x128 block)
 *   out  bf16  [M, N]    row stride ldo elements (>= N)
 *   K % 128 == 0 and N % 128 == 0 (kernels/fused_gemv_quant_tm.py:87).
 * The activation is quantised per row and per 128-column group:
 *   amax = max(max|x|, 1e-10); sx = amax / 448; xq = e4m3_rne(clamp(x / sx))
 * (x * (1/sx) exactly as sglang fp8_kernel.py:170-173 writes it) and
 *   out[m, n] = bf16( sum_b (sum_{k in b} xq[m,k] w[n,k]) * sx[m,b] * ws[n/128,b] ).
 *
 * Optional outputs xq_out (uint8 [M, K], row stride K) and sx_out (fp32
 * [M, K/128], row stride K/128) receive the quantised activation bytes and
 * scales the fused kernel computed internally; pass NULL to skip them.
 *
 * `stream` is a cudaStream_t (NULL = the legacy default stream).
 */
#ifndef FP8GQ_H_
#define FP8GQ_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FP8GQ_VERSION 2

enum fp8gq_status {
    FP8GQ_OK = 0,
    FP8GQ_ERR_NULL_POINTER = 1,  /* a required pointer is NULL                      */
    FP8GQ_ERR_SHAPE = 2,         /* M < 1, or K / N not a positive multiple of 128  */
    FP8GQ_ERR_ALIGNMENT = 3,     /* x / w / gu not 16-byte aligned, or a stride not
                                    a multiple of 16 bytes                          */
    FP8GQ_ERR_STRIDE = 4,        /* a row stride smaller than the row length        */
    FP8GQ_ERR_WORKSPACE = 5,     /* workspace NULL or smaller than required         */
    FP8GQ_ERR_DEVICE = 6,        /* current device is not compute capability 10.x   */
    FP8GQ_ERR_LAUNCH = 7,        /* the CUDA launch failed                          */
    FP8GQ_ERR_UNSUPPORTED = 8,   /* shape outside what the selected kernel handles  */
    FP8GQ_ERR_DEVICE_TIMEOUT = 9, /* a kernel's bounded wait gave up (see
                                    fp8gq_device_error)                             */
    FP8GQ_ERR_SCRATCH_LIMIT = 10 /* the shape needs more scratch than the fixed
                                    device buffer of fp8gq_gemv_quant_tm_noalloc    */
};

typedef void *fp8gq_stream_t;

/* Library version (FP8GQ_VERSION). */
int fp8gq_version(void);

/* Static, human-readable text for a status code. */
const char *fp8gq_status_string(int status);

/* Fused quant + GEMV, routed by M like the reference wrapper
 * fused_gemv_quant (kernels/fused_gemv_quant_tm.py:83-102): M > 1 runs the
 * tensor-core tile kernel (fp8gq_gemv_quant_tm); M == 1 runs the row kernel
 * (fp8gq_gemv_quant_row) when the weight is at most 20 MiB (N * K bytes) and
 * K <= 49152, and the tile kernel otherwise (on B200 it streams large weights
 * faster).  Both produce the same quantised bytes; outputs agree within the
 * accumulation-order tolerance.  `workspace` must hold fp8gq_workspace_bytes(M, N, K)
 * bytes (it may be NULL when that is 0) and be zero-filled before its first
 * use; kernels leave it zero-filled again when they finish.  Calls that share
 * a workspace must not overlap on the GPU. */
int fp8gq_fused_gemv_quant(const void *x, int64_t ldx, const void *w, int64_t ldw,
                           const float *ws, int64_t ldws, void *out, int64_t ldo,
                           int M, int N, int K, uint8_t *xq_out, float *sx_out,
                           void *workspace, size_t workspace_bytes, fp8gq_stream_t stream);

/* Scratch bytes fp8gq_fused_gemv_quant / fp8gq_fused_swiglu_q_gemm need for
 * this shape (0 when the routed kernel -- the row kernel -- needs none).  K is the contraction
 * length (I for the SwiGLU entry point). */
size_t fp8gq_workspace_bytes(int M, int N, int K);

/* M == 1 row kernel: one pass over the weight on CUDA cores, 128-bit bulk
 * copies into a shared-memory ring, warp-shuffle amax, fp32 accumulation.
 * Replaces gemv_quant_row_kernel (kernels/fused_gemv_quant_tm.py:25-46) and
 * its twin gemv_quant_kernel (kernels/fused_gemv_quant.py:21-46).
 * Requires M == 1 and K <= 49152. */
int fp8gq_gemv_quant_row(const void *x, const void *w, int64_t ldw,
                         const float *ws, int64_t ldws, void *out,
                         int N, int K, uint8_t *xq_out, float *sx_out,
                         fp8gq_stream_t stream);

/* Tile kernel for any M >= 1 (tcgen05 FP8 MMA, each weight tile read once
 * for all M rows, M <= 256 per pass).  Replaces gemv_quant_tm_kernel
 * (kernels/fused_gemv_quant_tm.py:49-80). */
int fp8gq_gemv_quant_tm(const void *x, int64_t ldx, const void *w, int64_t ldw,
                        const float *ws, int64_t ldws, void *out, int64_t ldo,
                        int M, int N, int K, uint8_t *xq_out, float *sx_out,
                        void *workspace, size_t workspace_bytes, fp8gq_stream_t stream);

/* Fused SwiGLU + quant + GEMV (down_proj):
 *   act = silu(gu[:, :I]) * gu[:, I:]   (fp32),   out = GEMV(quant(act), w)
 * gu bf16 [M, 2I] row stride ldgu, w e4m3 [N, I], ws [N/128, I/128].
 * Replaces fused_swiglu_q_gemm / swiglu_q_gemm_kernel
 * (kernels/fused_swiglu_quant_gemv.py:26-67).  Routed like
 * fp8gq_fused_gemv_quant (M == 1 and N * I <= 20 MiB: row kernel).  xq_out /
 * sx_out as above, with K = I. */
int fp8gq_fused_swiglu_q_gemm(const void *gu, int64_t ldgu, const void *w, int64_t ldw,
                              const float *ws, int64_t ldws, void *out, int64_t ldo,
                              int M, int N, int I, uint8_t *xq_out, float *sx_out,
                              void *workspace, size_t workspace_bytes, fp8gq_stream_t stream);

/* Activation group quant alone (the same device code the fused kernels
 * run): x bf16 [M, K] -> xq uint8 [M, K] (row stride K), sx fp32 [M, K/128].
 * Mirrors sglang's per-token-group quant as inlined at
 * kernels/fused_gemv_quant.py:35-43. */
int fp8gq_group_quant(const void *x, int64_t ldx, int M, int K,
                      uint8_t *xq, float *sx, fp8gq_stream_t stream);

/* SwiGLU + group quant alone: gu bf16 [M, 2I] -> xq [M, I], sx [M, I/128]
 * (kernels/fused_swiglu_quant_gemv.py:40-46). */
int fp8gq_swiglu_group_quant(const void *gu, int64_t ldgu, int M, int I,
                             uint8_t *xq, float *sx, fp8gq_stream_t stream);

/* N-sharded linears over several GPUs (one process per GPU): each rank runs
 * the fused op on its rows [col0, col0 + N) of the weight, and the kernel
 * writes that output slice into the same columns of every rank's full output
 * buffer itself -- plain stores over NVLink through the peers' mapped
 * pointers -- instead of a separate all-gather.  The last CTA then raises this
 * rank's flag on every rank; a later call with wait_input != 0 (one whose
 * activation is such a gathered output) waits, inside its kernel, until every
 * rank's flag has caught up before it reads the activation.  The waits are
 * bounded (FP8GQ_ERR_DEVICE_TIMEOUT through fp8gq_device_error).
 *
 * Every rank must issue the same sequence of gathered calls.  out[r] and
 * flags[r] are rank r's buffers as mapped into this process (fp8gq_ipc_open;
 * out[rank] and flags[rank] are this rank's own).  counter and seq are this
 * rank's own, zero-filled once before the first call.  No counterpart in the
 * reference (which is single-GPU); it replaces the NCCL all-gather after each
 * linear of an N-sharded decoder. */
#define FP8GQ_MAX_GATHER_RANKS 8
typedef struct fp8gq_gather {
    void *out[FP8GQ_MAX_GATHER_RANKS];       /* bf16 [M, ldo] full output of rank r */
    uint32_t *flags[FP8GQ_MAX_GATHER_RANKS]; /* uint32 [world] flag array of rank r */
    uint32_t *counter;                       /* this rank: one uint32, zero-filled */
    uint32_t *seq;                           /* this rank: one uint32, zero-filled */
    int64_t ldo;                             /* row stride of the full outputs, elements */
    int col0;                                /* first column of this rank's slice */
    int world;                               /* 1 .. FP8GQ_MAX_GATHER_RANKS (1: one GPU) */
    int rank;
    int wait_input;
    int local_out;                           /* 1: only wait; the output stays local
                                                (set by the reduce entry point below) */
    int tagged;                              /* 1: tagged words, see below */
} fp8gq_gather;

/* Tagged words (tagged = 1), the low-latency form of the same gather.  The
 * flags above cost the publishing kernel a system-scope fence -- a wait for
 * every one of its NVLink stores to be acknowledged -- and a second round of
 * peer stores.  With tagged = 1 every stored word carries its own proof of
 * arrival instead: a 64-bit word holds columns 2i and 2i + 1 of a row (bf16,
 * low half first) and, in its high 32 bits, the sequence number of the call
 * that wrote it.  out[r] then points at rank r's words: M x ldo / 2 uint64
 * (ldo and col0 in elements, as above; ldo a multiple of 8, out[r] 16-byte
 * aligned).  A call with wait_input reads its activation as such words (x or
 * gu points at words, ldx / ldgu in elements) and polls each word it reads,
 * bounded, until it carries this rank's last sequence number: the input must
 * be the output of this rank's last publishing call.  A publishing call
 * without wait_input first waits until every rank has finished this rank's
 * previous publishing call (each rank's own slot flags[q][q], raised without a
 * fence).  M <= 16 (one launch per call); no norm prologue; local_out = 0.
 * fp8gq_gather_decode turns a tagged output into bf16. */

/* fp8gq_fused_gemv_quant with the output gathered as above (routing and
 * workspace as fp8gq_fused_gemv_quant; N is this rank's slice width). */
int fp8gq_fused_gemv_quant_gather(const void *x, int64_t ldx, const void *w, int64_t ldw,
                                  const float *ws, int64_t ldws, int M, int N, int K,
                                  const fp8gq_gather *gather, void *workspace, size_t workspace_bytes,
                                  fp8gq_stream_t stream);

/* Waits on `stream` (a one-thread kernel, bounded) until every rank's slice of
 * this rank's last gathered output has arrived -- e.g. before the full output
 * is read by something that is not a gathered call with wait_input set. */
int fp8gq_gather_wait(const fp8gq_gather *gather, fp8gq_stream_t stream);

/* Tagged words: waits on `stream` (bounded) until every word of this rank's
 * full tagged output [M, N] -- gather->out[gather->rank], row stride
 * gather->ldo elements -- carries this rank's last sequence number, and
 * writes the values as bf16 [M, N] into out (row stride ldo elements; out
 * 16-byte aligned, ldo a multiple of 8).  fp8gq_gather_wait is for flags only
 * (FP8GQ_ERR_UNSUPPORTED with tagged = 1). */
int fp8gq_gather_decode(const fp8gq_gather *gather, int M, int N, void *out, int64_t ldo,
                        fp8gq_stream_t stream);

/* Tensor-parallel pairing without a gather in between: a column-parallel
 * (N-sharded) linear keeps its output slice on its rank, where it feeds a
 * row-parallel (K-sharded) linear whose output is a partial sum over its K
 * slice.  Each rank stores that partial [M, N] into slab `rank` of every
 * rank's partial buffer [world][M][N] -- an fp8gq_gather with out[r] = rank
 * r's buffer + rank * M * N elements, col0 = 0, ldo = N -- and the next
 * column-parallel linear adds the slabs in rank order in its prologue
 * (fp8gq_fused_reduce_add_rmsnorm_gemv_quant).  One exchange per block
 * (attention: qkv -> o; MLP: gate_up -> down) instead of an all-gather after
 * every linear.  No counterpart in the reference (single-GPU).
 *
 * fp8gq_fused_swiglu_q_gemm with the output stored through `gather` (the
 * row-parallel down_proj: gu is this rank's [gate | up] slice, I its width). */
int fp8gq_fused_swiglu_q_gemm_gather(const void *gu, int64_t ldgu, const void *w, int64_t ldw,
                                     const float *ws, int64_t ldws, int M, int N, int I,
                                     const fp8gq_gather *gather, void *workspace, size_t workspace_bytes,
                                     fp8gq_stream_t stream);

/* fp8gq_fused_add_rmsnorm_gemv_quant (below) whose x is the sum of nsrc
 * (1 .. FP8GQ_MAX_GATHER_RANKS) bf16 [M, K] sources src_stride elements apart,
 * each with row stride ldx:
 *   s = ((x_0 + x_1) + ... + x_{nsrc-1}) + residual   (fp32, left to right)
 * then the same norm, residual_out = bf16(s), quant and GEMV into `out` on
 * this rank.  With `wait` (a descriptor of the row-parallel calls that stored
 * the sources; wait_input and local_out are implied, out[] is ignored) the
 * kernel first waits, bounded, until every rank's flag has caught up.
 * nsrc = 1 with wait = NULL is fp8gq_fused_add_rmsnorm_gemv_quant. */
int fp8gq_fused_reduce_add_rmsnorm_gemv_quant(const void *x, int nsrc, int64_t src_stride, int64_t ldx,
                                              const void *residual, int64_t ldr, const void *norm_w, float eps,
                                              const void *w, int64_t ldw, const float *ws, int64_t ldws,
                                              void *out, int64_t ldo, void *residual_out, int64_t ldro,
                                              int M, int N, int K, uint8_t *xq_out, float *sx_out,
                                              const fp8gq_gather *wait, void *workspace, size_t workspace_bytes,
                                              fp8gq_stream_t stream);

/* Device-memory mapping between the processes of one node (CUDA IPC).
 * fp8gq_ipc_get: a 64-byte handle of the allocation that holds `ptr`, and
 * ptr's byte offset in it.  fp8gq_ipc_open: map a peer's handle (the current
 * device gets peer access on first use) and return the mapped base and
 * base + offset.  fp8gq_ipc_close: unmap a base returned by fp8gq_ipc_open. */
int fp8gq_ipc_get(const void *ptr, void *handle64, uint64_t *offset);
int fp8gq_ipc_open(const void *handle64, uint64_t offset, void **base, void **ptr);
int fp8gq_ipc_close(void *base);

/* Fused add + RMSNorm (the reference's add_rmsnorm_kernel,
 * kernels/fused_rmsnorm.py:14-27), bf16 x, residual [M, K] and norm weight
 * [K], K % 128 == 0, 16-byte aligned rows:
 *   s = x + residual (fp32);  residual_out = bf16(s)
 *   rstd = 1 / sqrt(sum(s^2) / K + eps)   (IEEE sqrt and division; the sum in a
 *          fixed order: 16-value chunks left to right, the 8 chunks of a
 *          128-group pairwise, the groups left to right)
 *   out = bf16((s * rstd) * w)
 * residual_out may be NULL (not written). */
int fp8gq_add_rmsnorm(const void *x, int64_t ldx, const void *residual, int64_t ldr, const void *norm_w,
                      float eps, void *out, int64_t ldo, void *residual_out, int64_t ldro, int M, int K,
                      fp8gq_stream_t stream);

/* The same add + RMSNorm as the prologue of the fused quant + GEMV: out =
 * GEMV(quant(norm output)) with the norm output never stored -- the norm's
 * launch leaves the decode chain.  Bit-identical to fp8gq_add_rmsnorm followed
 * by fp8gq_fused_gemv_quant on its output.  residual_out (may be NULL) must
 * not overlap residual (other CTAs still read it while it is written).
 * Routing and workspace as fp8gq_fused_gemv_quant; the tile kernel needs its
 * resident activation feed here and returns FP8GQ_ERR_UNSUPPORTED for shapes
 * where that does not fit.  No counterpart in the reference (it runs the norm
 * as its own kernel). */
int fp8gq_fused_add_rmsnorm_gemv_quant(const void *x, int64_t ldx, const void *residual, int64_t ldr,
                                       const void *norm_w, float eps, const void *w, int64_t ldw,
                                       const float *ws, int64_t ldws, void *out, int64_t ldo,
                                       void *residual_out, int64_t ldro, int M, int N, int K,
                                       uint8_t *xq_out, float *sx_out, void *workspace, size_t workspace_bytes,
                                       fp8gq_stream_t stream);

/* Stand-alone SwiGLU writers for any M (the prefill side, M > 16), gate and up
 * as separate bf16 [M, I] operands (row strides ldg, ldu elements, 16-byte
 * aligned), I % 128 == 0:
 *   y = g * sigmoid(g) * u in fp32 (sigmoid(g) = 1 / (1 + exp(-g)));
 * fp8gq_swiglu stores bf16(y) (RNE) to out [M, I] (row stride ldo elements).
 * Replaces fused_swiglu (kernels/fused_swiglu_fp8.py:19-27, :48-53). */
int fp8gq_swiglu(const void *gate, int64_t ldg, const void *up, int64_t ldu, void *out, int64_t ldo,
                 int M, int I, fp8gq_stream_t stream);

/* fp8gq_swiglu_quant quantises y per row and 128-group with that module's own
 * formula (not the GEMV prologue's):
 *   scale = max(amax / 448, 1e-30),  q = e4m3_rne(clamp(y / scale, +-448))
 * (IEEE divisions) into q uint8 [M, I] (row stride ldq bytes, 8-byte
 * aligned) and scale fp32 [M, I/128] (contiguous).  Replaces
 * fused_swiglu_quant / swiglu_quant_kernel (kernels/fused_swiglu_fp8.py:30-45,
 * :56-63). */
int fp8gq_swiglu_quant(const void *gate, int64_t ldg, const void *up, int64_t ldu, uint8_t *q, int64_t ldq,
                       float *scale, int M, int I, fp8gq_stream_t stream);

/* Declares (enable != 0) that weights and their block scales are never written
 * by work queued earlier on the stream of a call -- true in an inference server
 * whose weights are loaded once.  The kernels are launched with programmatic
 * dependent launch, so a call may start while the previous kernel on its
 * stream is still running; with static weights it then already streams its
 * first weight tiles and block scales before waiting for that kernel (the
 * activation, output and workspace are never touched before the wait).  Off by
 * default: leave it off when weights can change between calls (for example an
 * online weight update followed directly by a call).  Process-wide; returns the
 * previous setting.  No counterpart in the reference. */
int fp8gq_set_static_weights(int enable);

/* Tile-kernel strategy switches (fp8gq_gemv_quant_tm and the M > 1 paths),
 * a bit mask; 0 (the default) picks each strategy where it fits:
 *   FP8GQ_TM_STREAM_ACTIVATIONS  never use the resident activation feed (a CTA
 *       quantising the activation of its whole K range into shared memory once,
 *       before its weight stream starts); every K block's activation tile then
 *       travels with its weight tile and is quantised on arrival;
 *   FP8GQ_TM_PREQUANT_ACTIVATIONS  use the pre-quantised feed wherever its
 *       scales fit: one group-quant launch writes the e4m3 activation and its
 *       scales before the tile kernel, whose B tiles then arrive by TMA next to
 *       the weight tiles (by default it is used where the activation cannot
 *       stay resident, or where quantising it in every CTA costs more);
 *   FP8GQ_TM_RESIDENT_ACTIVATIONS  use the resident feed wherever it fits and
 *       the pre-quantised one only where it does not;
 *   FP8GQ_TM_WORKSPACE_SPLITK   never reduce split-K partial sums inside a
 *       thread-block cluster (over distributed shared memory); they go through
 *       the workspace and the last CTA of the row block adds them.
 * At most one of the three activation-feed bits may be set.  Every combination
 * gives bit-identical results (same products, same order of additions); the
 * switches exist for testing and measurement.  Process-wide; returns the
 * previous mask, or -1 for unknown bits or two feed bits.  No counterpart in
 * the reference. */
#define FP8GQ_TM_STREAM_ACTIVATIONS 1
#define FP8GQ_TM_WORKSPACE_SPLITK 2
#define FP8GQ_TM_PREQUANT_ACTIVATIONS 4
#define FP8GQ_TM_RESIDENT_ACTIVATIONS 8
int fp8gq_set_tm_options(int flags);

/* Reads (and with clear != 0 resets) the current device's error word, which
 * a kernel sets when one of its bounded waits gives up.  Synchronous.  0 means
 * no error was recorded. */
int fp8gq_device_error(uint32_t *code, int clear);

/* Sets the current device's limit of the bounded waits in the kernels, in
 * nanoseconds, 1 ms .. 20 s (default 2 s): a gathered call's wait for the
 * peers' flags gives up after it, a wait for work inside the same kernel (a
 * ring, accumulator or split-K wait) after twice it, so that a lost peer is
 * reported by the peer wait.  *previous (may be NULL) receives the old
 * limit.  Synchronous.  A wait
 * that runs out records its site in the device error word and the kernel
 * finishes without hanging -- this is the failure path that replaces the
 * reference's catch-all fallback (patches/patch_fp8_fused_tail.py:16-26):
 * a lost peer or a stuck copy becomes FP8GQ_ERR_DEVICE_TIMEOUT on the host.
 * Lowering the limit lets a test make a wait run out on purpose; leave the
 * default in production.  FP8GQ_ERR_UNSUPPORTED for a limit out of range. */
int fp8gq_set_wait_limit_ns(uint64_t limit_ns, uint64_t *previous);

/* Stack runner: a list of block-FP8 linears -- e.g. the qkv, o, gate_up and
 * down (SwiGLU) linears of every layer of a decode step -- run in list order
 * by ONE persistent, cooperative launch on all SMs.  Each linear is the tile
 * kernel's fused quant + GEMM (the arithmetic of
 * kernels/fused_gemv_quant_tm.py:49-80, and with swiglu set of
 * kernels/fused_swiglu_quant_gemv.py:26-51); its input may be the output of
 * an earlier linear of the list.  Every SM's TMA stream runs on into the
 * next linear's weights while that linear waits for its input, so the
 * per-launch gap of a linear-at-a-time decode step disappears.  A decoder
 * that owns its step calls it once per step.  The reference has no
 * counterpart: it launches one Triton kernel per linear.
 *
 * Per linear: x bf16 [M, K] (swiglu: [M, 2K] = [gate | up], act =
 * silu(gate) * up quantised as in fp8gq_fused_swiglu_q_gemm), w e4m3 [N, K],
 * ws fp32 [N/128, K/128], out bf16 [M, N]; K, N multiples of 128,
 * N <= 524288; x 16-byte aligned with ldx a multiple of 8 elements; all
 * linears share M, 1 <= M <= 16.  Linear l reads x only after every earlier
 * linear whose output overlaps x, or whose x or out overlaps l's out, has
 * been stored completely (fp8gq_stack_dependencies shows the choice); there
 * is no other ordering between linears. */
typedef struct fp8gq_stack_linear {
    const void *x;   int64_t ldx;
    const void *w;   int64_t ldw;
    const float *ws; int64_t ldws;
    void *out;       int64_t ldo;
    int N, K;
    int swiglu;      /* 1: x is [gate | up] with 2K columns */
    int reserved;    /* 0 */
} fp8gq_stack_linear;

/* Host-side record of a prepared list (filled by fp8gq_stack_prepare). */
typedef struct fp8gq_stack_plan {
    void *device;          /* the caller's device memory holding the plan */
    size_t bytes;
    int n, M, device_id, grid, stages, npw;
    int sw, lg_sw, kpb, nacc;
    size_t smem;
    int64_t reserved[4];
} fp8gq_stack_plan;

/* Device bytes a plan of n linears at M tokens needs on the current device
 * (the linear table, counters and the split-K partial sums). */
size_t fp8gq_stack_plan_bytes(int n, int M);

/* For each linear, the index of the earlier linear it waits for (-1: none):
 * the latest one whose output overlaps this linear's input, or whose input
 * or output overlaps this linear's output.  Host only; no GPU needed. */
int fp8gq_stack_dependencies(const fp8gq_stack_linear *lin, int n, int M, int *dep);

/* Validates the list, writes the plan into `device_mem` (bytes >=
 * fp8gq_stack_plan_bytes(n, M), 256-byte aligned) with copies on `stream`
 * (from pageable host memory: not for use during stream capture) and fills
 * *plan.  The plan holds the linears' pointers: re-prepare after any of them
 * changes. */
int fp8gq_stack_prepare(const fp8gq_stack_linear *lin, int n, int M, void *device_mem, size_t bytes,
                        fp8gq_stack_plan *plan, fp8gq_stream_t stream);

/* Runs every linear of a prepared plan: one kernel launch (capturable in a
 * CUDA graph).  Runs that share a plan must not overlap on the GPU.  If a
 * run records a device error (fp8gq_device_error), its outputs are invalid
 * and the plan must be prepared again. */
int fp8gq_stack_run(const fp8gq_stack_plan *plan, fp8gq_stream_t stream);

/* Chain runner: a decode step's M == 1 linears, N-sharded across the ranks of
 * a tagged gather (world 1 .. FP8GQ_MAX_GATHER_RANKS; world 1 is one GPU),
 * in one persistent cooperative launch.  Linear i holds this rank's N rows
 * (columns col0 .. col0 + N of its full output) and stores them as tagged
 * words (see fp8gq_gather) into out[r] of every rank r.  Its input x is
 * either the words of an earlier linear's output (src = that linear's index;
 * x may point at any 16-byte aligned column of that output row, e.g. its
 * first K columns) or, with src = -1, a bf16 row written before the launch.
 * A linear polls the words it reads until they carry linear src's sequence
 * number, so the list runs with no barrier or flag between linears, and the
 * weight stream of later linears continues while a CTA waits for an input.
 * The weights are static (fetched without waiting for earlier work).  The
 * math and its order are the row kernel's (fp8gq_fused_gemv_quant_gather).
 * Limits: M = 1, K <= 12288 (of gate and of up with swiglu), K and N
 * multiples of 128.  After the launch this rank's sequence number has moved
 * past the list (n numbers); fp8gq_gather_decode of the last linear's output
 * reads it.  No counterpart in the reference (single-GPU, one launch per
 * linear). */
typedef struct fp8gq_chain_linear {
    const void *x;                           /* src >= 0: words; src < 0: bf16 [K] (or [2K]) */
    const void *w;   int64_t ldw;            /* e4m3 [N, ldw], this rank's rows */
    const float *ws; int64_t ldws;           /* fp32 [N/128, ldws] */
    int N, K;
    int src;                                 /* the linear whose output x reads, or -1 */
    int swiglu;                              /* 1: x is [gate | up], 2K columns */
    int col0;                                /* this rank's first column in the full output */
    int reserved;                            /* 0 */
    void *out[FP8GQ_MAX_GATHER_RANKS];       /* rank r's output words of this linear */
} fp8gq_chain_linear;

/* Host-side record of a prepared chain (filled by fp8gq_chain_prepare). */
typedef struct fp8gq_chain_plan {
    void *device;                            /* the caller's device memory holding the list */
    size_t bytes;
    int n, device_id, grid, stages, world, rank;
    size_t smem;
    uint32_t *flags[FP8GQ_MAX_GATHER_RANKS];
    uint32_t *counter, *seq;
    int64_t reserved[4];
} fp8gq_chain_plan;

/* Device bytes a chain of n linears needs (its table). */
size_t fp8gq_chain_plan_bytes(int n);

/* Checks the list, copies it into device_mem (fp8gq_chain_plan_bytes(n),
 * 256-byte aligned; a synchronous copy) and fills `plan`.  `gather` gives the
 * tagged gather's flags, counter, seq, world and rank (its out, ldo, col0 and
 * wait_input are not used). */
int fp8gq_chain_prepare(const fp8gq_chain_linear *lin, int n, const fp8gq_gather *gather,
                        void *device_mem, size_t bytes, fp8gq_chain_plan *plan);

/* Launches a prepared chain on `stream` (cooperative: every CTA resident). */
int fp8gq_chain_run(const fp8gq_chain_plan *plan, fp8gq_stream_t stream);

/* Prepared launches.  A decode loop calls the same linears on the same
 * buffers every step; most of a call's host time is spent on work that does
 * not change between steps -- argument checks, routing, tensor-map encoding,
 * grid choice, the kernel parameter block.  fp8gq_prepare_<entry point> takes
 * the arguments of <entry point> (without the stream), does all of that once
 * and stores the resulting kernel launches (one to three) in *plan, launching
 * nothing; fp8gq_launch_plans then issues the launches of n plans, in array
 * order, on `stream`, with no other host work.  The result of launching a plan
 * is the result of the entry point it was prepared from: same kernels, same
 * parameters.  A plan holds raw device pointers (operands, outputs, workspace,
 * peer buffers) and the process-wide switches in force when it was prepared
 * (fp8gq_set_static_weights, fp8gq_set_tm_options): prepare it again after any
 * of them changes.  Plans are plain data: they may be copied byte for byte,
 * e.g. into one array for fp8gq_launch_plans, and are launched on the device
 * that was current when they were prepared (FP8GQ_ERR_DEVICE otherwise).
 * Launches of plans that share a workspace or a gather descriptor's counters
 * must not overlap on the GPU.  fp8gq_launch_plans stops at the first plan that
 * fails and returns its status.  No counterpart in the reference (which pays
 * Triton's launch path on every call, and removes it with CUDA graphs). */
#define FP8GQ_LAUNCH_PLAN_BYTES 4096
typedef struct fp8gq_launch_plan {
    uint64_t opaque[FP8GQ_LAUNCH_PLAN_BYTES / 8];
} fp8gq_launch_plan;

int fp8gq_prepare_fused_gemv_quant(const void *x, int64_t ldx, const void *w, int64_t ldw,
                                   const float *ws, int64_t ldws, void *out, int64_t ldo,
                                   int M, int N, int K, uint8_t *xq_out, float *sx_out,
                                   void *workspace, size_t workspace_bytes, fp8gq_launch_plan *plan);
int fp8gq_prepare_fused_swiglu_q_gemm(const void *gu, int64_t ldgu, const void *w, int64_t ldw,
                                      const float *ws, int64_t ldws, void *out, int64_t ldo,
                                      int M, int N, int I, uint8_t *xq_out, float *sx_out,
                                      void *workspace, size_t workspace_bytes, fp8gq_launch_plan *plan);
int fp8gq_prepare_fused_gemv_quant_gather(const void *x, int64_t ldx, const void *w, int64_t ldw,
                                          const float *ws, int64_t ldws, int M, int N, int K,
                                          const fp8gq_gather *gather, void *workspace, size_t workspace_bytes,
                                          fp8gq_launch_plan *plan);
int fp8gq_prepare_fused_swiglu_q_gemm_gather(const void *gu, int64_t ldgu, const void *w, int64_t ldw,
                                             const float *ws, int64_t ldws, int M, int N, int I,
                                             const fp8gq_gather *gather, void *workspace,
                                             size_t workspace_bytes, fp8gq_launch_plan *plan);
int fp8gq_prepare_fused_reduce_add_rmsnorm_gemv_quant(const void *x, int nsrc, int64_t src_stride, int64_t ldx,
                                                      const void *residual, int64_t ldr, const void *norm_w,
                                                      float eps, const void *w, int64_t ldw, const float *ws,
                                                      int64_t ldws, void *out, int64_t ldo, void *residual_out,
                                                      int64_t ldro, int M, int N, int K, uint8_t *xq_out,
                                                      float *sx_out, const fp8gq_gather *wait, void *workspace,
                                                      size_t workspace_bytes, fp8gq_launch_plan *plan);
int fp8gq_prepare_gather_wait(const fp8gq_gather *gather, fp8gq_launch_plan *plan);
int fp8gq_prepare_gather_decode(const fp8gq_gather *gather, int M, int N, void *out, int64_t ldo,
                                fp8gq_launch_plan *plan);
int fp8gq_launch_plans(const fp8gq_launch_plan *plans, int n, fp8gq_stream_t stream);

/* fp8gq_gemv_quant_tm without a workspace argument.  No counterpart in the
 * reference (its Triton kernels need no scratch).
 *
 * For callers that cannot allocate device memory at the point of the call:
 * inference servers that reserve nearly all of HBM up front for weights and
 * KV cache and hand it out from a pool they do not let kernels draw on,
 * latency-critical decode loops that cannot afford cudaMalloc's implicit
 * device synchronisation, and plain C/FFI callers that have no allocator of
 * their own to size and zero a workspace with.
 * The tile kernel's split-K scratch lives instead in one fixed device array
 * of FP8GQ_NOALLOC_SCRATCH_BYTES (8 MiB) inside libfp8gq, which every GPU
 * that loads the library keeps until the process exits.  That bounds the
 * shapes: a call whose scratch (fp8gq_workspace_bytes of the tile kernel)
 * exceeds the array returns FP8GQ_ERR_SCRATCH_LIMIT; on a 148-SM B200 every
 * M <= 16 with N <= 524288 and K <= 131072 fits.
 *
 * The first call on a device looks up the array's device address (once per
 * device, with that device current) and keeps it for the life of the
 * process; make that first call before any stream capture begins, and do not
 * reset the device (cudaDeviceReset) between calls.  Every call clears the array's split-K counters with an
 * asynchronous memset on `stream` and then reuses the array, which keeps the
 * last call's partial sums: calls whose kernels overlap on the GPU (two
 * streams, two host threads) race on it, so issue them on one stream.
 * Allocates nothing: no cudaMalloc, no cudaFree, no allocating library call.
 */
#define FP8GQ_NOALLOC_SCRATCH_BYTES (8u << 20)
int fp8gq_gemv_quant_tm_noalloc(const void *x, int64_t ldx, const void *w, int64_t ldw,
                                const float *ws, int64_t ldws, void *out, int64_t ldo,
                                int M, int N, int K, uint8_t *xq_out, float *sx_out,
                                fp8gq_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* FP8GQ_H_ */
