/*
 * busfill.h -- C ABI of the B200 (sm_100a) batched dequant-fused 4-bit-weight
 * GEMM.  C[M, N] = A[M, K] * deq(W)[N, K]^T, fp16 activations, fp32
 * accumulation.
 *
 * Conventions for every entry point:
 *   - all array pointers are DEVICE pointers owned by the caller;
 *   - fp16 data is passed as uint16_t (IEEE binary16 bit patterns);
 *   - `stream` is a cudaStream_t (NULL = the legacy default stream);
 *   - calls are asynchronous on `stream` and never synchronize; errors that
 *     can only be seen on the device (a bounded wait that expired) are
 *     reported by busfill_stream_status();
 *   - the return value is BUSFILL_OK (0) or a negative busfill_status code;
 *     nothing aborts the process.
 *
 * Each entry point names the reference interface it replaces
 * (thegliffy/bus-fill, file:line).
 */
#ifndef BUSFILL_H_
#define BUSFILL_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define BUSFILL_API __attribute__((visibility("default")))
#else
#define BUSFILL_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum busfill_status {
  BUSFILL_OK = 0,
  BUSFILL_ERR_INVALID_ARG = -1,        /* NULL pointer or bad option        */
  BUSFILL_ERR_SHAPE = -2,              /* M/N/K out of the supported range  */
  BUSFILL_ERR_ALIGNMENT = -3,          /* pointer not 16-byte aligned       */
  BUSFILL_ERR_UNSUPPORTED_DEVICE = -4, /* current device is not sm_100      */
  BUSFILL_ERR_LAUNCH = -5,             /* kernel launch failed              */
  BUSFILL_ERR_ALLOC = -6,              /* workspace allocation failed       */
  BUSFILL_ERR_DEVICE_TIMEOUT = -7,     /* a bounded device wait expired     */
  BUSFILL_ERR_CUDA = -8                /* other CUDA runtime error          */
} busfill_status;

/* ---------------------------------------------------------------------------
 * GEMMs
 * ------------------------------------------------------------------------- */

/* Q4_0 in the reference's split-plane layout, fp16 output.
 *   wq [N, K/2] u8  : byte j of 32-value block b holds element 32b+2j in its
 *                     low nibble and 32b+2j+1 in its high nibble;
 *   ws [N, K/32] fp16 scales d;  value = (nibble - 8) * d.
 *   a  [M, K] fp16 row-major;  c [M, N] fp16 row-major.
 * Requires K % 256 == 0, M >= 1, N >= 1; wq, ws, a 16-byte aligned.
 * Replaces busfill_q4 (kernels/busfill_v1a.cu:41-46; launch :151-154), with
 * fp16 output, any M (the reference computes only rows < 32) and any N. */
BUSFILL_API int busfill_gemm_q4_0(const uint8_t* wq, const uint16_t* ws, const uint16_t* a, uint16_t* c, int M, int N, int K,
                      void* stream);

/* Q4_K: llama.cpp block_q4_K rows, K/256 blocks of 144 bytes per weight row
 * (fp16 d, fp16 dmin, 12 bytes of packed 6-bit sub-block scales and mins,
 * 128 nibble bytes); value = d*sc*q - dmin*m.  a [M, K] fp16, c [M, N] fp16.
 * The fp16 weight operand is fp16_rn(fp32(d*sc)*q - fp32(dmin*m)), bit for
 * bit the CPU dequant of busfill_dequant_q4k (llama.cpp's order).
 * Requires K % 256 == 0; blocks and a 16-byte aligned.
 * The reference has no Q4_K kernel; this is the Q4_K counterpart of
 * busfill_q4 (kernels/busfill_v1a.cu:41-46) that its docstring announces
 * (kernels/q4k_batched.py:7-8). */
BUSFILL_API int busfill_gemm_q4k(const uint8_t* blocks, const uint16_t* a, uint16_t* c, int M, int N, int K, void* stream);

/* Fused SwiGLU pair of a gated feed-forward layer:
 *   h[M, N] = silu(A deq(w_gate)^T) * (A deq(w_up)^T),  silu(x) = x / (1 + e^-x),
 * with both products accumulated in fp32 and h rounded once to fp16.
 * w_gate and w_up are llama.cpp block_q4_K rows [N, K/256 x 144 B] (the
 * ffn_gate and ffn_up tensors), a [M, K] fp16, h [M, N] fp16. Requires
 * K % 256 == 0; all pointers 16-byte aligned. Up to M = 128 the gate and up
 * tiles of the same 128 rows are computed by the same CTAs, so neither
 * product goes to memory. Above M = 128 (BUSFILL_OPT_PREFILL_PAIR) the pair
 * runs as two CTA-pair GEMMs: the up projection into h (fp16), then the gate
 * with h = fp16(silu(gate) * h), so the up product is rounded to fp16 before
 * the multiplication (within the same accuracy gate; twice as fast as the
 * fused launch there). No reference counterpart: the epilogue BASELINE config 3's layer
 * set puts after the up projection (kernels/q4k_batched.py:7-8 names the
 * Q4_K GEMM it belongs to). */
BUSFILL_API int busfill_gemm_q4k_swiglu(const uint8_t* w_gate, const uint8_t* w_up, const uint16_t* a, uint16_t* h,
                                        int M, int N, int K, void* stream);

/* ---------------------------------------------------------------------------
 * Layer sweep: up to BUSFILL_SWEEP_MAX_OPS small-batch Q4_K GEMMs in one launch
 *
 * Runs a list of GEMMs ("ops") that share the batch M (1..32) as one kernel
 * launch, e.g. a decoder layer's O, QKV, gate/up (SwiGLU) and down
 * projections. Op o computes c[M, N] = a[M, K] deq(w)[N, K]^T, or with w_up
 * the SwiGLU pair c = silu(a deq(w)^T) * (a deq(w_up)^T), from block_q4_K
 * rows as busfill_gemm_q4k takes them, with the same numerics. Every op's
 * units are split evenly over all SMs; a CTA moves on to the next op's weights
 * as soon as it has done its share of one, and an op with dep = j >= 0 reads
 * its activations only once op j's whole output is stored (j < o: its `a` is
 * op j's `c`, or computed from it). Ops with dep = -1 must not read an
 * earlier op's output in this call. Outputs must not overlap inputs.
 * Order matters for speed, not for results: an op that directly follows
 * the op it reads waits for that op's last tile; with an independent op in
 * between, the wait is hidden. Two decoder layers per call (eight ops) in
 * the order O1, O2, QKV1, gate/up1 (dep 0), gate/up2 (dep 1), down1 (dep 3),
 * down2 (dep 4), QKV2 (dep 5) hide every wait.
 * The first call on a stream allocates its workspace (~80 MB: counters and
 * partial tiles; fails with BUSFILL_ERR_ALLOC inside a graph capture); calls
 * on one stream share it in stream order. Failures are read with
 * busfill_stream_status. No reference counterpart: the reference launches
 * one GEMM per kernel (kernels/busfill_v1a.cu:151-154); this is the layer
 * set of its decode benchmark as one launch. */
#define BUSFILL_SWEEP_MAX_OPS 8
typedef struct busfill_sweep_op {
  const uint8_t* w;      /* block_q4_K rows [N][K/256 * 144] (the gate with w_up) */
  const uint8_t* w_up;   /* SwiGLU: the up projection's rows, same shape; else NULL */
  const uint16_t* a;     /* activations [M][K] fp16 */
  uint16_t* c;           /* output [M][N] fp16 */
  int N, K;
  int dep;               /* index of the earlier op whose output `a` is, or -1 */
} busfill_sweep_op;
BUSFILL_API int busfill_gemm_q4k_sweep(const busfill_sweep_op* ops, int nops, int M, void* stream);

/* ---------------------------------------------------------------------------
 * Column-split GEMMs with the all-gather fused into the epilogue
 *
 * Over a group of `npeers` GPUs (one process each, same node), rank r holds
 * rows [col_off, col_off + N) of a weight whose full output has `ldc`
 * columns. Each rank's GEMM writes its [M, N] slice straight into every
 * rank's full output buffer (out[q] is rank q's [M, ldc] buffer, mapped into
 * this process, e.g. with busfill_ipc_open), over NVLink, and adds the number
 * of 128-row output tiles it wrote to flag[q] (a zeroed word in rank q's
 * memory that only this rank adds to; a running total over the call site's
 * calls). A later GEMM whose activations are that gathered output passes the
 * nwait local words it must wait on (`wait`, one per source rank), the tiles
 * each source rank writes per call (`wait_tiles`) and `wait_gen`, two zeroed
 * local words for its own call site; its kernel waits (acquire, bounded by
 * 1 s, else BUSFILL_ERR_DEVICE_TIMEOUT) until word r reaches (calls so far +
 * 1) x wait_tiles[r], counting its calls in wait_gen[0] (wait_gen[1] counts
 * the CTAs of the call in progress, so M and the launch shape may change from
 * call to call). All state lives in
 * device memory, so the calls can be captured in a CUDA graph and replayed.
 * No NCCL call, no host round trip. Every rank must make the same calls in
 * the same order; a rank that owns no rows of a weight (N = 0: fewer 128-row
 * tiles than ranks) makes the call too, and it does nothing (its weight
 * pointers may be NULL; it writes 0 tiles a call). A call site's output buffer is overwritten by the peers'
 * next call of that site: do not call a site again until every rank's
 * consumers of its previous output have finished (a later site's wait that
 * orders the ranks, or a barrier between passes). The reference is
 * single-GPU (no counterpart); this is BASELINE's N-split with its
 * all-gather moved into the GEMM.
 * ------------------------------------------------------------------------- */
#define BUSFILL_MAX_PEERS 8
typedef struct busfill_gather {
  int npeers;                        /* ranks receiving the output (this one included), 1..8 */
  int col_off;                       /* first column of this rank's slice */
  int ldc;                           /* columns of the full outputs */
  uint16_t* out[BUSFILL_MAX_PEERS];  /* each rank's full output [M, ldc] fp16 (device pointers) */
  uint32_t* flag[BUSFILL_MAX_PEERS]; /* per rank q: this rank's tile counter in rank q's memory */
  const uint32_t* wait;              /* optional: nwait local counter words to wait on before reading a */
  uint32_t* wait_gen;                /* with wait: two zeroed local words of this call site */
  int nwait;                         /* source ranks waited on, <= 8 */
  int wait_tiles[BUSFILL_MAX_PEERS]; /* with wait: 128-row tiles source rank r writes per call */
} busfill_gather;

/* busfill_gemm_q4k on this rank's weight rows [N, K/256 x 144 B], output
 * gathered per `g` (g->out[rank] is this rank's own full output). */
BUSFILL_API int busfill_gemm_q4k_gather(const uint8_t* blocks, const uint16_t* a, int M, int N, int K,
                                        const busfill_gather* g, void* stream);
/* busfill_gemm_q4k_swiglu on this rank's gate/up rows, output gathered per `g`. */
BUSFILL_API int busfill_gemm_q4k_swiglu_gather(const uint8_t* w_gate, const uint8_t* w_up, const uint16_t* a, int M,
                                               int N, int K, const busfill_gather* g, void* stream);

/* Make `stream` wait until a gathered output is complete on this rank: one
 * small kernel waits (acquire, bounded by 1 s) until word r of g->wait
 * reaches (g->wait_gen[0] + 1) x g->wait_tiles[r] and then advances
 * g->wait_gen[0] (two zeroed words of its own, not a GEMM's), as a consuming
 * GEMM would. For consumers that are not busfill GEMMs (a copy to the host,
 * another library's kernel). Only the wait fields of `g` are read. */
BUSFILL_API int busfill_gather_wait(const busfill_gather* g, void* stream);

/* CUDA IPC for the peer buffers above: a 64-byte handle of a device
 * allocation (cudaIpcGetMemHandle), its mapping in another process of the
 * same node (cudaIpcOpenMemHandle, peer access enabled lazily), and unmapping. */
BUSFILL_API int busfill_ipc_alloc(size_t bytes, void** dev_ptr); /* cudaMalloc + zero fill, shareable */
BUSFILL_API int busfill_ipc_free(void* dev_ptr);
BUSFILL_API int busfill_ipc_get_handle(const void* dev_ptr, void* handle64);
BUSFILL_API int busfill_ipc_open(const void* handle64, void** dev_ptr);
BUSFILL_API int busfill_ipc_close(void* dev_ptr);

/* Q4_0 as llama.cpp stores it: block_q4_0 rows, K/32 blocks of 18 bytes per
 * weight row (fp16 d, then 16 bytes whose low nibbles are elements 0-15 and
 * high nibbles elements 16-31); value = (q - 8) * d, the same rule as
 * busfill_gemm_q4_0.  a [M, K] fp16, c [M, N] fp16.  Requires K % 256 == 0;
 * blocks and a 16-byte aligned.  No reference counterpart: it is the
 * ggml-native ingest of the Q4_0 weights the reference's kernels take as
 * split planes (kernels/busfill_v1a.cu:41-46; the layout is named at
 * kernels/busfill_v0.cu:18-20), so llama.cpp buffers drop in without a
 * repack. */
BUSFILL_API int busfill_gemm_q4_0_ggml(const uint8_t* blocks, const uint16_t* a, uint16_t* c, int M, int N, int K,
                                       void* stream);

/* Q5_K: llama.cpp block_q5_K rows, K/256 blocks of 176 bytes per weight row
 * (fp16 d, fp16 dmin, the 12 scale/min bytes of Q4_K, 32 bytes qh holding
 * each value's fifth bit, 128 nibble bytes); value = d*sc*q - dmin*m with q
 * in 0..31.  a [M, K] fp16, c [M, N] fp16.  Requires K % 256 == 0; blocks and
 * a 16-byte aligned.  No reference counterpart: one of the K-quant formats
 * that Q4_K_M models mix in; same kernels as busfill_gemm_q4k, and the same
 * exact operand fp16_rn(fp32(d*sc)*q - fp32(dmin*m)). */
BUSFILL_API int busfill_gemm_q5k(const uint8_t* blocks, const uint16_t* a, uint16_t* c, int M, int N, int K, void* stream);

/* Q6_K weights (llama.cpp block_q6_K: 128 B ql, 64 B qh, 16 int8 scales,
 * fp16 d per 256 values), in the layout busfill_repack_q6k writes:
 *   body [N, K/256 * 208] u8  every block's first 208 bytes (ql, qh, scales)
 *   d    [K/256, N] fp16      the blocks' d, block-major
 * A 210-byte block row has a 16-byte row stride (which the kernels'
 * tensor-memory-access copies need) only when K % 2048 == 0, so the blocks
 * are split once at load time; the bytes per weight stay 6.5625 bits.
 * Operand fp16_rn(fp32(d*sc)*(q-32)), the CPU dequant's bits; N % 8 == 0
 * (d's row stride), K % 256 == 0, body/d/a 16-byte aligned.  No reference
 * counterpart: the other K-quant format that Q4_K_M models mix in. */
BUSFILL_API int busfill_gemm_q6k(const uint8_t* body, const uint16_t* d, const uint16_t* a, uint16_t* c, int M, int N,
                                 int K, void* stream);

/* block_q6_K rows [N, K/256 * 210] (2-byte aligned) -> body and d as above.
 * Asynchronous on `stream`; `blocks` and the outputs must not overlap. */
BUSFILL_API int busfill_repack_q6k(const uint8_t* blocks, uint8_t* body, uint16_t* d, int N, int K, void* stream);

/* Q4_K as separate planes, the split-pointer form of the Q4_K weight:
 *   qs       [N, K/2] u8        each 256-value super-block's 128 nibble bytes
 *                               in block_q4_K order (32-byte chunk c: low
 *                               nibbles sub-block 2c, high nibbles 2c+1);
 *   d, dmin  [N, K/256] fp16    the super-blocks' scale and min scale;
 *   scales12 [N, K/256, 12] u8  the packed 6-bit sub-block scales and mins.
 * busfill_repack_q4k_planar moves these bytes into block_q4_K rows [N,
 * K/256 x 144 B] for busfill_gemm_q4k (do it once, when the weights are
 * loaded). busfill_gemm_q4k_planar repacks into a per-stream buffer that the
 * library allocates on first use (and grows; never during a graph capture:
 * BUSFILL_ERR_ALLOC), then runs busfill_gemm_q4k on it, so every call moves
 * the weights three times (read, write, read): prefer the one-time repack.
 * qs, blocks, a 16-byte aligned; d, dmin 2-byte; scales12 4-byte. The
 * reference has no Q4_K code; this is the planar signature of the Q4_K
 * entry its docstring announces (kernels/q4k_batched.py:7-8). */
BUSFILL_API int busfill_repack_q4k_planar(const uint8_t* qs, const uint16_t* d, const uint16_t* dmin,
                                          const uint8_t* scales12, uint8_t* blocks, int N, int K, void* stream);
BUSFILL_API int busfill_gemm_q4k_planar(const uint8_t* qs, const uint16_t* d, const uint16_t* dmin,
                                        const uint8_t* scales12, const uint16_t* a, uint16_t* c, int M, int N, int K,
                                        void* stream);

/* ---------------------------------------------------------------------------
 * ggml mul_mat call site
 *
 * A tensor as ggml describes one: element type (ggml_type numbering), ne[]
 * elements and nb[] byte strides per dimension (index 0 innermost), and its
 * device data. busfill_mul_mat(src0, src1, dst) computes what
 * ggml_mul_mat(ctx, src0, src1) defines: src0 the quantized weight
 * [ne0 = K, ne1 = N, ne2, ne3] (Q4_0 in block_q4_0, Q4_K in block_q4_K, Q5_K
 * in block_q5_K rows), src1 the activations [K, M, ne12, ne13] fp16, dst
 * [N, M, ne12, ne13] fp16 (row m of dst holds the N outputs of activation row
 * m: C[M, N]); src0 is broadcast over src1's batch dimensions (ne12 % ne02
 * == 0, ne13 % ne03 == 0). Rows must be packed (nb[1] = the row's bytes);
 * batch strides nb[2], nb[3] are free. One busfill_gemm_* call per batch
 * slice. Other types (Q6_K, whose rows need busfill_repack_q6k first; fp32
 * activations) return BUSFILL_ERR_INVALID_ARG. No reference counterpart:
 * the reference's next step is wiring its dequant into llama.cpp's batched
 * GEMM (RESULTS.md:235-237), which is reached through this call site.
 * ------------------------------------------------------------------------- */
#define BUSFILL_TYPE_F32 0
#define BUSFILL_TYPE_F16 1
#define BUSFILL_TYPE_Q4_0 2
#define BUSFILL_TYPE_Q4_K 12
#define BUSFILL_TYPE_Q5_K 13
#define BUSFILL_TYPE_Q6_K 14
typedef struct busfill_tensor {
  int32_t type;  /* BUSFILL_TYPE_*: the ggml_type numbering */
  int64_t ne[4]; /* elements per dimension, ne[0] innermost */
  size_t nb[4];  /* bytes per step along each dimension */
  void* data;    /* device pointer */
} busfill_tensor;
BUSFILL_API int busfill_mul_mat(const busfill_tensor* src0, const busfill_tensor* src1, busfill_tensor* dst,
                                void* stream);

/* busfill_gemm_q4k that allocates no device memory.  It has no counterpart
 * in the reference.
 *
 * busfill_gemm_q4k cudaMallocs a small per-stream buffer (the device error
 * words) on first use of each stream.  Some callers can't allow that: a host
 * whose own pool already holds nearly all device memory, where an outside
 * cudaMalloc fails or fragments it; an operator or plugin interface that
 * hands a kernel only its inputs and outputs; a latency-bound loop where
 * cudaMalloc would stall the device.  This entry point keeps its scratch
 * (the error word and the first failure record) in one 256-byte array
 * compiled into the library, which every GPU that loads the library holds
 * until the process exits.  The decode kernel's split-K partial sums live in
 * shared memory, and large batches here take whole work items per SM (no
 * stream-K workspace), so no problem size needs more scratch.  The caller
 * still passes the inputs
 * and the output; arguments, layout and results are those of
 * busfill_gemm_q4k.
 *
 *   - The first call on each device looks up the array's device address
 *     (cudaGetSymbolAddress) with that device current; make that first call
 *     before any stream capture begins.
 *   - Every call on every stream shares the one array, and each call clears
 *     it (a cudaMemsetAsync on `stream`) before its kernels run.  Calls whose
 *     kernels overlap on the GPU (other streams, other host threads) race on
 *     the array: a failure of one can be cleared or misattributed by another.
 *   - A device-side wait that expires is recorded in the array, not in the
 *     per-stream word that busfill_stream_status reads: busfill_noalloc_status
 *     reports it. The output of such a call is undefined. */
BUSFILL_API int busfill_gemm_q4k_noalloc(const uint8_t* blocks, const uint16_t* a, uint16_t* c, int M, int N, int K,
                                         void* stream);

/* Synchronizes `stream`, then reports (and clears) the error word that
 * busfill_gemm_q4k_noalloc calls keep in the library's static array: BUSFILL_OK,
 * BUSFILL_ERR_DEVICE_TIMEOUT or BUSFILL_ERR_CUDA; *bits (if not NULL) gets the
 * role bits as in busfill_stream_status_ex. Allocates nothing. The array is
 * shared by every no-allocation call on the device, so with calls in flight
 * on other streams the word may belong to any of them. No reference
 * counterpart. */
BUSFILL_API int busfill_noalloc_status(void* stream, unsigned* bits);

/* Reference-compatible surface: the arguments and fp32 output of
 * busfill_q4(A, Wq, Ws, C, Bsz, K, N) (kernels/busfill_v1a.cu:41-46) plus a
 * stream, as a host function instead of a <<<N/32, 128>>> launch
 * (kernels/busfill_v1a.cu:151-154). Every row b < Bsz is computed (the
 * reference silently skips rows >= 32). */
BUSFILL_API int busfill_q4(const uint16_t* A, const uint8_t* Wq, const uint16_t* Ws, float* C, int Bsz, int K, int N,
               void* stream);

/* ---------------------------------------------------------------------------
 * Dequantization to fp16 [N, K] row-major (bit-exact)
 * ------------------------------------------------------------------------- */

/* fp16_rn((q - 8) * d): the dequant of kernels/busfill_v0.cu:74-81 (which
 * kernels/busfill_v1a.cu:6-20 reproduces bit for bit). K % 32 == 0. */
BUSFILL_API int busfill_dequant_q4_0(const uint8_t* wq, const uint16_t* ws, uint16_t* out, int N, int K, void* stream);

/* llama.cpp block_q4_0 rows (18-byte blocks), same value rule. K % 32 == 0.
 * No reference counterpart: the layout the reference's comment names
 * (kernels/busfill_v0.cu:18-20). */
BUSFILL_API int busfill_dequant_q4_0_ggml(const uint8_t* blocks, uint16_t* out, int N, int K, void* stream);

/* fp16_rn(fp32(d)*sc*q - fp32(dmin)*m) per llama.cpp block_q4_K. K % 256 == 0.
 * No reference counterpart (the reference has no Q4_K code). */
BUSFILL_API int busfill_dequant_q4k(const uint8_t* blocks, uint16_t* out, int N, int K, void* stream);

/* fp16_rn(fp32(d)*sc*q - fp32(dmin)*m) per llama.cpp block_q5_K. K % 256 == 0.
 * No reference counterpart. */
BUSFILL_API int busfill_dequant_q5k(const uint8_t* blocks, uint16_t* out, int N, int K, void* stream);

/* fp16_rn((fp32(d)*sc)*(q-32)) per llama.cpp block_q6_K, from the repacked
 * layout of busfill_gemm_q6k. K % 256 == 0. No reference counterpart. */
BUSFILL_API int busfill_dequant_q6k(const uint8_t* body, const uint16_t* d, uint16_t* out, int N, int K, void* stream);

/* ---------------------------------------------------------------------------
 * Status, options, diagnostics
 * ------------------------------------------------------------------------- */

/* Synchronizes `stream`, then reports (and clears) the device-side error word
 * of the workspace bound to this stream: BUSFILL_OK, BUSFILL_ERR_DEVICE_TIMEOUT
 * or BUSFILL_ERR_CUDA. The reference has no error reporting at all
 * (kernels/busfill_v1a.cu:155-158 only prints launch/sync strings). */
BUSFILL_API int busfill_stream_status(void* stream);

/* As busfill_stream_status, and also stores the device error word (0 when
 * clean) in *bits if bits is not NULL: one bit per kernel role whose bounded
 * wait expired (1 weight producer, 2 activation producer, 4 MMA issuer,
 * 8 dequant, 16 epilogue, 32 teardown, 64 activation stage). */
BUSFILL_API int busfill_stream_status_ex(void* stream, unsigned* bits);

/* Detail word of the first bounded wait that expired in the last failing
 * call seen by busfill_stream_status_ex (0 if none): bit 31 set, bits 24-30
 * the warp index, bits 12-23 the unit index within that CTA's range, bits
 * 1-11 the barrier slot, bit 0 the awaited phase parity. For diagnostics. */
BUSFILL_API unsigned busfill_last_failure_detail(void);

/* Number of device allocations this library has made on its own so far in
 * the process (per-stream error words and stream-K workspaces; not the
 * buffers of busfill_ipc_alloc). Diagnostic: lets a caller check that a
 * path allocates nothing. No reference counterpart. */
BUSFILL_API unsigned busfill_internal_allocations(void);

/* Human-readable text for a busfill_status value. */
BUSFILL_API const char* busfill_status_string(int status);

/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
BUSFILL_API int busfill_version(void);

/* Options (process-wide).
 *   BUSFILL_OPT_PDL: 1 (default) launches the GEMMs with programmatic
 *     dependent launch so back-to-back calls on one stream overlap the next
 *     call's weight streaming with the previous call's tail; 0 disables.
 *   BUSFILL_OPT_KSPLIT: 0 (default) lets the library choose how many CTAs (a
 *     thread-block cluster of 1..8) split the K range of each 128-row tile;
 *     1..8 forces that split where K/256 allows it (a tuning and test knob).
 *   BUSFILL_OPT_PREFILL_MIN_M: GEMMs with M >= value rows run the large-batch
 *     (prefill) kernel, one pass over the weights for all rows, instead of
 *     the decode kernel's launches of 64 rows (32 for the SwiGLU pairs and
 *     the gathered GEMMs); 0 (default) chooses by shape:
 *     M > 64, or M > 32 when N <= K and K >= 12288, for the plain GEMMs,
 *     whose prefill
 *     kernel splits the units of work evenly over all SMs (stream-K, with a
 *     per-stream workspace of 2 x SMs x 128 KB allocated on first use, never
 *     during a graph capture); M >= 128 and at least 64 work
 *     items of 256 weight rows x 128 batch rows for SwiGLU pairs and
 *     busfill_gemm_q4k_noalloc, which take whole items. A tuning and test
 *     knob; results agree within the accuracy gate.
 *   BUSFILL_OPT_EXACT_KQUANT: accepted (0 or 1) and ignored: every K-quant
 *     GEMM builds the exact operand fp16_rn(fp32 w). Kept so that callers
 *     which set it keep working.
 *   BUSFILL_OPT_PREFILL_BATCH_TILE: batch rows per work item of the prefill
 *     kernel: 0 (default) chooses 256 (one 128-row weight tile, MMA N = 256)
 *     for M >= 256 and 128 (two weight tiles) below; 128 or 256 forces it
 *     (SwiGLU pairs always take 128). A tuning and test knob; results agree
 *     within the accuracy gate.
 *   BUSFILL_OPT_PREFILL_PAIR: 0 (default) runs prefill GEMMs of M > 128 on
 *     CTA pairs (items of 256 weight rows x 256 batch rows, one MMA over the
 *     two SMs of a 2-CTA cluster, each loading half of the batch rows), and
 *     SwiGLU pairs of M > 128 as two such GEMMs; 1 does so for every prefill
 *     GEMM and SwiGLU pair; 2 never.
 *     A tuning and test knob; results agree within the accuracy gate.
 *   BUSFILL_OPT_SWEEP_CTAS: CTAs of a busfill_gemm_q4k_sweep launch; 0
 *     (default) one per SM. A tuning and test knob; results agree within the
 *     accuracy gate (the split of split tiles, so the fp32 summation order,
 *     follows the CTA count).
 *   BUSFILL_OPT_SWEEP_UNMET_DEP: 0 (default); 1 makes every dependent op of a
 *     busfill_gemm_q4k_sweep wait for one tile more than its input op
 *     stores, so that its bounded wait (1 s) runs out: the call's output is
 *     invalid and busfill_stream_status reports BUSFILL_ERR_DEVICE_TIMEOUT
 *     (and clears the stream's words and counters). For failure-detection
 *     tests only.
 * Returns BUSFILL_ERR_INVALID_ARG for an unknown option or value. */
#define BUSFILL_OPT_PDL 1
#define BUSFILL_OPT_KSPLIT 2
#define BUSFILL_OPT_PREFILL_MIN_M 3
#define BUSFILL_OPT_EXACT_KQUANT 4
#define BUSFILL_OPT_PREFILL_BATCH_TILE 5
#define BUSFILL_OPT_PREFILL_PAIR 6
#define BUSFILL_OPT_SWEEP_CTAS 7
#define BUSFILL_OPT_SWEEP_UNMET_DEP 8
BUSFILL_API int busfill_set_option(int option, int value);

/* Which kernel a plain GEMM (busfill_gemm_q4_0 / _q4k / ...) of M batch rows,
 * N output columns and depth K runs with the current options: 0 = decode
 * kernel (launches of 64 rows), 1 = prefill kernel (one pass over the
 * weights; by default for M > 64, and for M > 32 when N <= K and
 * K >= 12288). Diagnostic;
 * no reference counterpart. */
BUSFILL_API int busfill_gemm_kernel_for(int M, int N, int K);

/* Kernel launches one plain GEMM call of that shape makes on a device with
 * sm_count SMs (sm_count <= 0: the current device): one decode launch per 64
 * batch rows, or the prefill kernel and, when its stream-K ranges split a
 * work item between CTAs, the fix-up kernel (with the per-stream workspace in
 * place; a first call inside a graph capture takes whole items instead, one
 * launch). A negative busfill_status for a bad shape. Diagnostic; no
 * reference counterpart. */
BUSFILL_API int busfill_gemm_launches(int M, int N, int K, int sm_count);

/* Known-answer probe of the tcgen05 operand layouts the GEMM relies on, in the
 * spirit of kernels/frag_probe.cu:1-48: d[128, nb] = a[128, 64] * b[nb, 64]^T
 * with a in tensor memory and b in 128-byte-swizzled shared memory.
 * nb in {16, 32, 64}; one CTA; fp32 out. */
BUSFILL_API int busfill_probe_umma(const uint16_t* a, const uint16_t* b, float* d, int nb, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* BUSFILL_H_ */
