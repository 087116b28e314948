/*
 * deepx_fused.h — C ABI of the B200 fused GEMM + bias + activation engine.
 *
 * One operation:  Y[M,N] = act(X[M,K] @ W[K,N] + bias[N]) (+ R[M,N])
 *
 * This is the drop-in replacement for the kernels the reference compiles for
 * its `linear*` fusion patterns:
 *   - deepx_op_gpukernelcompiler/kernel_triton.py:24-89  (Triton `_kernel`,
 *     `make_linear_kernel(activation) -> kernel_fn(A, B, bias) -> C`)
 *   - deepx_op_gpukernelcompiler/kernel_tilelang.py:23-55 (TileLang `main`)
 *   - the raw-pointer runtime entry the design docs describe but never build:
 *     `kernel_fn(x_ptr, W_ptr, b_ptr, out_ptr, cuda_stream)`
 *     (doc/kvlang-to-tilelang-interface.md:79-98,
 *      doc/kernel-compiler-analysis.md:113-134).
 *
 * Conventions (all entry points):
 *   - Matrices are row-major with an explicit leading dimension in ELEMENTS:
 *     X[m*ldx + k], W[k*ldw + n] (W is K x N, i.e. `x @ W`), Y[m*ldy + n],
 *     R[m*ldr + n].  bias is a dense vector of N elements.
 *   - X, W, bias, R and Y share one element type (`dtype`); accumulation is
 *     always fp32.  The output has the input dtype, as in the reference
 *     (kernel_triton.py:74 allocates C with A.dtype).
 *   - Epilogue order: Y = act(acc + bias) + R.  bias and R may be NULL.
 *   - The caller owns every buffer (inputs, output and workspace), as in the
 *     docs' runtime contract (doc/kvlang-to-tilelang-interface.md:86-89).  The
 *     library never allocates, frees or synchronises on the caller's behalf;
 *     every launch goes to `stream` (a cudaStream_t; NULL = legacy default).
 *   - Stream order holds as for any kernel.  The tensor-core and (for weight
 *     streams up to 160 MiB) decode kernels are launched with programmatic
 *     dependent launch: their set-up may overlap the tail of the preceding
 *     kernel on the stream, but they read and write no global memory before
 *     it has completed.  DX_PDL=0 in the environment turns this off.
 *   - Return value: DX_OK (0) or a negative DX_ERR_* code.  The message of the
 *     last failure on the calling thread is available from
 *     dx_last_error_string().
 *   - Device-side waits are bounded: a kernel that times out sets a per-device
 *     status word (read with dx_device_status) and returns instead of hanging.
 */
#ifndef DEEPX_FUSED_H_
#define DEEPX_FUSED_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- return codes ------------------------------------------------------ */
#define DX_OK                     0
#define DX_ERR_INVALID_ARGUMENT  -1   /* bad shape, stride, pointer or enum   */
#define DX_ERR_UNSUPPORTED       -2   /* valid request the library cannot run */
#define DX_ERR_CUDA              -3   /* a CUDA runtime/driver call failed    */
#define DX_ERR_WORKSPACE         -4   /* workspace missing or too small       */
#define DX_ERR_DEVICE_TIMEOUT    -5   /* a kernel's bounded wait ran out      */

/* ---- element types ----------------------------------------------------- */
#define DX_DTYPE_F32   0   /* exact fp32 FFMA path (no TF32)                 */
#define DX_DTYPE_F16   1   /* tcgen05 kind::f16, fp32 accumulate             */
#define DX_DTYPE_BF16  2   /* tcgen05 kind::f16 (bf16), fp32 accumulate      */

/* ---- activations (fusion.py ACTIVATION_PT + the kernels' erf GELU) ------ */
#define DX_ACT_NONE       0  /* pattern `linear`                             */
#define DX_ACT_RELU       1  /* `linear_relu`   (fusion.py:88)               */
#define DX_ACT_GELU_TANH  2  /* `linear_gelu`   (fusion.py:89, tanh approx)  */
#define DX_ACT_GELU_ERF   3  /* exact GELU of kernel_triton.py:61,
                                kernel_tilelang.py:17                        */
#define DX_ACT_SILU       4  /* `linear_silu` / `linear_swish` (fusion.py:90-91) */

/* ---- kernel variants --------------------------------------------------- */
#define DX_KERNEL_AUTO    0  /* pick by shape, dtype and alignment           */
#define DX_KERNEL_UMMA    1  /* persistent tcgen05 + TMEM + TMA GEMM (CTA
                                pairs with cta_group::2 when M >= 256)      */
#define DX_KERNEL_DECODE  2  /* swap-AB split-K tcgen05 kernel, M <= 64      */
#define DX_KERNEL_SIMT    3  /* CUDA-core FFMA kernel (fp32, odd strides)    */
#define DX_KERNEL_UMMA_1CTA 4 /* the tcgen05 GEMM with single-CTA tiles only */

/* Device status bits reported by dx_device_status. */
#define DX_DEVICE_STATUS_TIMEOUT  1

/*
 * Fused linear: Y = act(X @ W + bias) + R on `stream`.
 * Replaces kernel_triton.py:70-89 `kernel_fn(A, B, bias)` and
 * kernel_tilelang.py:26-53 `main(A, B, bias, C)`; the pointer form is the
 * docs' `kernel_fn(x_ptr, W_ptr, b_ptr, out_ptr, cuda_stream)`
 * (doc/kvlang-to-tilelang-interface.md:92) with the shape passed explicitly.
 * `workspace` may be NULL when dx_fused_linear_workspace_size() returns 0 for
 * the call; otherwise it must hold that many bytes, have been zero-filled
 * before its first use, and not be used by two calls at once.  Its first
 * 64 KiB hold split-K tickets that every successful call leaves at zero, so a
 * workspace can be reused by later calls of any shape; after a call that
 * reported DX_DEVICE_STATUS_TIMEOUT, zero it again.
 */
int dx_fused_linear(const void* X, const void* W, const void* bias,
                    const void* R, void* Y,
                    int64_t M, int64_t N, int64_t K,
                    int64_t ldx, int64_t ldw, int64_t ldr, int64_t ldy,
                    int dtype, int act,
                    void* workspace, size_t workspace_bytes,
                    void* stream);

/* Same as dx_fused_linear with the kernel variant forced (DX_KERNEL_*).
 * Used by tests and benchmarks to pin one implementation. */
int dx_fused_linear_ex(const void* X, const void* W, const void* bias,
                       const void* R, void* Y,
                       int64_t M, int64_t N, int64_t K,
                       int64_t ldx, int64_t ldw, int64_t ldr, int64_t ldy,
                       int dtype, int act, int kernel,
                       void* workspace, size_t workspace_bytes,
                       void* stream);

/*
 * Reduction of a row-parallel linear over `world` ranks (the second layer of
 * the MLP chain with its hidden dimension sharded; no reference counterpart —
 * the reference is single-GPU and fusion.py:42-43 marks two-layer FFNs
 * multi_kernel).  P[s] is rank s's partial Y (M x N, pitch ldp) and Y[s] its
 * output buffer (pitch ldy), all peer-mapped so this rank can reach them over
 * NVLink.  This rank handles rows rank*rows_per_rank .. +rows_per_rank: it
 * sums the world partials in rank order, adds bias[N] and the residual row
 * R[row] once, rounds to the dtype and writes the row into every Y[s]
 * (reduce-scatter and all-gather in one pass).  The caller orders it with the
 * peers: every partial complete before, every rank finished after (device
 * barriers).  bias and R may be NULL; N % 8 == 0; 16-byte-aligned buffers.
 */
int dx_reduce_broadcast(void* const* P, int world, int rank, int64_t rows_per_rank, int64_t N,
                        int64_t ldp, const void* bias, const void* R, int64_t ldr,
                        void* const* Y, int64_t ldy, int dtype, void* stream);

/*
 * Chunked, overlapped reduction of a row-parallel linear over `world` ranks
 * (no reference counterpart: the reference is single-GPU, and fusion.py:42-43
 * marks the two-layer FFN multi_kernel).  The second GEMM of the chain runs
 * in row chunks, each writing its partial Y into the rank's peer-mapped
 * buffer P.  One job per chunk, on each rank, does
 *   phase A (chunk a: rows a_row0 .. a_row0 + a_rows): announces the local
 *     partial of the chunk to every rank, waits until every rank's is
 *     complete, then sums this rank's slab of the chunk (rows a_row0 + rank *
 *     a_rows / world, a_rows / world of them) over all partials P[s] in rank
 *     order in fp32, adds bias[N] and R once, rounds, and writes the rows into
 *     Y and into its own slab buffer S[rank];
 *   phase B (chunk b, reduced by an earlier job of the same step): waits until
 *     every rank has announced its slab and copies the other ranks' slabs from
 *     S[s] into Y.
 * a_rows = 0 or b_rows = 0 skips a phase.  Only this rank writes Y, so Y is
 * any caller-owned device buffer [M][ldy].  P[s] ([M][ldp]), S[s]
 * ([2 * M / world][N]) and F[s] (dx_row_flag_words() int32 words, zeroed once
 * before first use) are rank s's buffers, mapped so every rank reaches them
 * over NVLink.  `epoch` numbers the step: the same positive value on every
 * rank, one larger per step; flags carry it, and its parity selects the half
 * of S the step uses, so a slab is never overwritten while a peer may still
 * read it.  The caller keeps steps apart on each rank (the stream that writes
 * P waits for the step's last job before the next step writes P again), and
 * gives the chunks of one step distinct indices (< 64).  Chunk starts and
 * sizes are multiples of `world`; N % 8 == 0; fp16/bf16 (`dtype`).  Waits are
 * bounded (2 s): on expiry the kernel sets DX_DEVICE_STATUS_TIMEOUT and
 * returns.
 */
typedef struct dx_row_reduce_job {
  void* P[8];   /* every rank's partial buffer */
  void* S[8];   /* every rank's slab buffer */
  int* F[8];    /* every rank's flag words */
  int world, rank;
  int64_t M, N, ldp;
  int64_t a_row0, a_rows;  /* phase A chunk (a_rows = 0: none) */
  int a_chunk;
  int64_t b_row0, b_rows;  /* phase B chunk (b_rows = 0: none) */
  int b_chunk;
  const void* bias;        /* [N] or NULL */
  const void* R;           /* residual [M][ldr] or NULL */
  int64_t ldr;
  void* Y;                 /* this rank's output [M][ldy] */
  int64_t ldy;
  int epoch, dtype;
  /* NVLink multicast (NVLS) form, used when mc_part is not NULL: the
   * multicast addresses of the partial buffers and of peer-written output
   * buffers Ysym (bound at the same offsets on every rank), and this rank's
   * own Ysym, pitch ldo.  Phase A then reads its slab's sum over the ranks
   * with one multimem.ld_reduce (the switch adds, fp32 accumulation, rounded
   * to the dtype), adds bias and R, writes Y and multicast-stores the rows
   * into every rank's Ysym; phase B copies the other ranks' slabs from the
   * local Ysym into Y.  S is unused.  Per GPU this moves about half the
   * NVLink bytes of the peer-load form. */
  void* mc_part;
  void* mc_out;
  void* out_sym;
  int64_t ldo;
} dx_row_reduce_job;

/* Runs a job as its own launch on `stream` (grid <= 0: one 512-thread CTA
 * per SM).  Used for the last chunk of a step, which has no GEMM left to
 * overlap. */
int dx_row_reduce(const dx_row_reduce_job* job, int grid, void* stream);

/* dx_fused_linear_ex that also carries `job` (may be NULL): when the launch is
 * a tensor-core GEMM (DX_KERNEL_UMMA / DX_KERNEL_UMMA_1CTA), two spare warps
 * per CTA run the job while the other warps compute the GEMM — the reduction
 * of one chunk overlaps the next chunk's GEMM on the same SMs.  Otherwise the
 * job runs as its own launch on `stream` right after the GEMM.  The job's
 * phase-A chunk of P must be complete in stream order before this call (it
 * is announced to the peers when the launch starts), and job->dtype must be
 * the GEMM's dtype. */
int dx_fused_linear_rowjob(const void* X, const void* W, const void* bias,
                           const void* R, void* Y,
                           int64_t M, int64_t N, int64_t K,
                           int64_t ldx, int64_t ldw, int64_t ldr, int64_t ldy,
                           int dtype, int act, int kernel,
                           void* workspace, size_t workspace_bytes,
                           const dx_row_reduce_job* job, void* stream);

/* dx_fused_gated_linear carrying a job, as dx_fused_linear_rowjob. */
int dx_fused_gated_linear_rowjob(const void* X, const void* Wg, const void* Wu,
                                 const void* bias_g, const void* bias_u, void* Y,
                                 int64_t M, int64_t N, int64_t K,
                                 int64_t ldx, int64_t ldwg, int64_t ldwu, int64_t ldy,
                                 int dtype, int act, int kernel,
                                 void* workspace, size_t workspace_bytes,
                                 const dx_row_reduce_job* job, void* stream);

/* int32 flag words a job needs in each rank's F buffer. */
int dx_row_flag_words(void);

/* Skinny-M (decode) fused linear that allocates nothing.  No counterpart in
 * the reference: it exists for callers that cannot allocate device memory at
 * call time — a runtime whose own heap manager owns every device buffer and
 * hands kernels only raw pointers and a stream, so it has no workspace to pass
 * and may not call cudaMalloc.  Same arguments and result as dx_fused_linear
 * with DX_KERNEL_DECODE (fp16/bf16, M <= 64, TMA-aligned X and W), but the
 * split-K scratch is a fixed 8 MiB device array inside the library; problems
 * whose scratch (the same bytes dx_fused_linear_workspace_size reports for
 * DX_KERNEL_DECODE) exceeds it return DX_ERR_WORKSPACE.  A plan that streams
 * whole tiles uses no scratch.  The first split-K call in a context (once per
 * device, normally) resolves the array's address and should precede any stream
 * capture; calls that overlap on the GPU race on the shared array. */
int dx_fused_linear_decode_noalloc(const void* X, const void* W, const void* bias,
                                   const void* R, void* Y,
                                   int64_t M, int64_t N, int64_t K,
                                   int64_t ldx, int64_t ldw, int64_t ldr, int64_t ldy,
                                   int dtype, int act, void* stream);

/* Workspace bytes that dx_fused_linear(_ex) needs for this problem and
 * variant (DX_KERNEL_AUTO resolves as dx_select_kernel does). */
size_t dx_fused_linear_workspace_size(int64_t M, int64_t N, int64_t K,
                                      int dtype, int kernel);

/* The variant DX_KERNEL_AUTO picks for a problem with contiguous rows
 * (ld == row length) and 16-byte-aligned pointers. */
int dx_select_kernel(int64_t M, int64_t N, int64_t K, int dtype);

/*
 * Gated dual-GEMM: Y = act(X @ Wg + bias_g) * (X @ Wu + bias_u), the first
 * two GEMMs of the gated FFN chain (`ffn_gated`, fusion.py:44-46; fixtures
 * test/fusion_cases/07_ffn_gated.kv and 08_ffn_swiglu.kv, with act = SiLU).
 * No reference kernel: the reference classifies that chain multi_kernel and
 * never runs it.  One launch reads X once for both weights: the tcgen05
 * kernels put Wg's and Wu's columns of a tile into one accumulator and
 * combine them in the epilogue.  Wg and Wu are [K, N] with pitches ldwg and
 * ldwu; bias_g, bias_u [N] may be NULL.  No residual.  Variants as for
 * dx_fused_linear_ex (DX_KERNEL_AUTO normally); the workspace rules are
 * those of dx_fused_linear, with dx_fused_gated_linear_workspace_size.
 */
int dx_fused_gated_linear(const void* X, const void* Wg, const void* Wu,
                          const void* bias_g, const void* bias_u, void* Y,
                          int64_t M, int64_t N, int64_t K,
                          int64_t ldx, int64_t ldwg, int64_t ldwu, int64_t ldy,
                          int dtype, int act, int kernel,
                          void* workspace, size_t workspace_bytes,
                          void* stream);

/* Rows of a strided 2-D region copied on `stream` (cudaMemcpy2DAsync with the
 * direction inferred from the pointers): `rows` rows of `width_bytes` bytes,
 * row pitches in bytes.  No reference counterpart: the staging step of the
 * host-buffer entry (Python fused_linear_host), which moves column blocks of
 * W and Y between pinned host memory and the device so that the copies of one
 * block overlap the fused launch of another.  Pinned host memory keeps the
 * copy asynchronous. */
int dx_copy_2d_async(void* dst, size_t dst_pitch, const void* src, size_t src_pitch,
                     size_t width_bytes, size_t rows, void* stream);

/* Workspace bytes that dx_fused_gated_linear needs (0: none). */
size_t dx_fused_gated_linear_workspace_size(int64_t M, int64_t N, int64_t K,
                                            int dtype, int kernel);

/*
 * Plans — the compile-then-call runtime of the reference design docs: the
 * compile step fixes shape, dtype and op sequence
 * (doc/kvlang-to-tilelang-interface.md:60-77,100-129) and the runtime calls
 * `kernel_fn(x_ptr, W_ptr, b_ptr, out_ptr, cuda_stream)`
 * (doc/kvlang-to-tilelang-interface.md:92, doc/kernel-compiler-analysis.md:118-123).
 * A plan computes out = act(alpha * x @ W + b) (+ r) for contiguous x[M,K],
 * W[K,N], b[N] (may be NULL), r and out [M,N]; alpha = 1 for the linear
 * patterns, the attention scale for `attention_score` (fusion.py:24).
 * `kernel` is a DX_KERNEL_* variant (DX_KERNEL_AUTO normally).  A plan holds
 * no device memory; give it the workspace dx_plan_workspace_size() asks for
 * (zero-filled once, one call at a time) with dx_plan_set_workspace.  The
 * workspace pointer is plan state: threads that share a plan serialise
 * dx_plan_set_workspace + dx_plan_call (the launch is asynchronous, so the
 * critical section is short), or use one plan per stream.
 */
typedef struct dx_plan dx_plan;
int dx_plan_create(dx_plan** plan, int64_t M, int64_t N, int64_t K, int dtype, int act,
                   float alpha, int kernel);
size_t dx_plan_workspace_size(const dx_plan* plan);
int dx_plan_set_workspace(dx_plan* plan, void* workspace, size_t bytes);
int dx_plan_call(const dx_plan* plan, const void* x, const void* W, const void* b, void* out,
                 void* stream);
int dx_plan_call_residual(const dx_plan* plan, const void* x, const void* W, const void* b,
                          const void* r, void* out, void* stream);
int dx_plan_destroy(dx_plan* plan);

/* Message of the last failed call on this thread ("" if none). */
const char* dx_last_error_string(void);

/* Description of the kernel launch made by the last successful call on this
 * thread: variant, tile shape, pipeline depth, grid ("" if none). */
const char* dx_last_launch_plan(void);

/* Timeline tracing of the tensor-core kernels (profiling aid).  With a
 * device buffer set, every later launch records %globaltimer stamps (ns) per
 * CTA: 16 uint64 slots per CTA in blockIdx order.  GEMM kernels: slot 0 after
 * set-up, slot 1+i when work item i's epilogue finished (i < 14), slot 15 at
 * exit.  Decode kernel: slot 0 after set-up, 1 / 2 first / last TMA issue,
 * 3 last MMA issue; for the CTA's last work item 4 accumulator ready, 5 read,
 * 6 arrival counted, 7 partial published / others' partials found written,
 * 8 fix-up sums done, 9 item finished; 10+i work item i finished (i < 2),
 * 12 kernel entry, 13 the SM id (not a time), 14 epilogue done, 15 exit.
 * The buffer must hold 16 * 8 bytes per CTA of the grid (148 SMs: 18,944 B);
 * launches whose grid does not fit are not traced.  NULL turns tracing off.
 * Process-wide setting; the caller owns the buffer. */
int dx_set_trace_buffer(void* device_buffer, size_t bytes);

/* Failure-path self-test (no reference counterpart): launches one CTA on
 * `stream` that waits, through the same bounded wait every kernel uses, on a
 * barrier nothing completes.  About a second later the wait gives up, the
 * device status word gets DX_DEVICE_STATUS_TIMEOUT and the device int
 * *result is set to 2 (1 would mean the wait completed).  The context stays
 * usable; read the status with dx_device_status. */
int dx_selftest_bounded_wait(int* result, void* stream);

/* Synchronises `stream`, then reads and clears the calling device's status
 * word (DX_DEVICE_STATUS_* bits) into *status. */
int dx_device_status(void* stream, int* status);

/* Architecture the library's kernels were compiled for, read from the loaded
 * module on the current device (cudaFuncGetAttributes): *binary_version is
 * 10 * major + minor of the SASS (100 for sm_100a) and *ptx_version that of
 * any embedded PTX (0 when there is none). */
int dx_kernel_arch(int* binary_version, int* ptx_version);

/* ABI version: 100 * major + minor. */
int dx_version(void);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* DEEPX_FUSED_H_ */
