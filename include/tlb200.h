/*
 * tlb200.h -- C ABI of libtlb200.so, the B200 (sm_100a) execution backend
 * for TensorLang programs.
 *
 * The reference lowers every `let` of a .tl program to one generated CUDA
 * kernel plus an `extern "C" void launch_<op>_<name>(float*..., int...)`
 * launcher (tensorlang/kernel_generator.py), compiles them with nvcc into a
 * per-program kernel.so, and calls the launchers through ctypes from
 * TensorCompiler._execute_single_kernel (tensorlang/compiler.py:365-673),
 * with PyCUDA allocations (compiler.py:1492-1503) and a
 * cudaDeviceSynchronize() inside every launcher.
 *
 * This library replaces that layer.  Conventions for every entry point:
 *   - plain pointers and sizes, no C++ or framework types;
 *   - every call returns an int status: 0 on success, a cudaError_t value
 *     for CUDA failures, or one of the TL_ERR_* codes below;
 *   - work is enqueued on the stream argument (a cudaStream_t passed as
 *     void*; NULL selects the library's per-device stream) and never
 *     synchronises the device;
 *   - tensors are dense row-major float32 ("f32" in .tl types); index results
 *     (argmax/argmin) are written as float values, as the reference does;
 *   - kernels never allocate.  Entry points that need temporary device memory
 *     take a `scratch` pointer whose minimum size is returned by the matching
 *     *_scratch_bytes() query; the scratch must be zero-filled once when it
 *     is first allocated (kernels leave it zeroed for the next call).
 */
#ifndef TLB200_H
#define TLB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (in addition to cudaError_t values) ------------------ */
#define TL_OK                 0
#define TL_ERR_INVALID_ARG    1001  /* bad size, null pointer, unsupported op */
#define TL_ERR_ALIGNMENT      1002  /* pointer or stride violates a documented alignment */
#define TL_ERR_JIT            1003  /* NVRTC compile or module load failed; see tl_jit_log */
#define TL_ERR_NO_NCCL        1004  /* libnccl.so.2 could not be loaded */
#define TL_ERR_NCCL           1005  /* an NCCL call failed; see tl_error_string */
#define TL_ERR_TIMEOUT        1006  /* a bounded device or host wait gave up */
#define TL_ERR_NOT_INIT       1007  /* tl_init not called for the current device */
#define TL_ERR_UNSUPPORTED    1008  /* shape/stride combination this kernel does not take */

/* ---- runtime: device, memory, streams, events, graphs ------------------
 * Replaces pycuda.autoinit / driver.mem_alloc / memcpy_htod / memcpy_dtoh /
 * DeviceAllocation.free used at compiler.py:1472-1503, 244-289, 680, 1666-1673.
 */
int  tl_init(int device);                       /* set device, create its stream and pool */
int  tl_device_count(int* count);
int  tl_device_info(int device, int* sm_count, int* cc_major, int* cc_minor,
                    size_t* total_mem);
const char* tl_error_string(int status);
void* tl_default_stream(void);                  /* the current device's library stream */

int  tl_malloc(void** ptr, size_t bytes, void* stream);   /* stream-ordered pool */
int  tl_free(void* ptr, void* stream);
int  tl_host_alloc(void** ptr, size_t bytes);             /* pinned host memory */
int  tl_host_free(void* ptr);
int  tl_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream);
int  tl_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream);
int  tl_memcpy_d2d(void* dst, const void* src, size_t bytes, void* stream);
int  tl_memset(void* dst, int value, size_t bytes, void* stream);

int  tl_stream_create(void** stream);
/* A stream whose blocks the GPU schedules first when SMs free up (urgent != 0:
 * the device's greatest priority), for work that must interleave with long
 * kernels -- the data-parallel gradient all-reduce.  No reference counterpart. */
int  tl_stream_create_priority(void** stream, int urgent);
int  tl_stream_destroy(void* stream);
int  tl_stream_sync(void* stream);
int  tl_device_sync(void);
int  tl_event_create(void** event);
int  tl_event_destroy(void* event);
int  tl_event_record(void* event, void* stream);
int  tl_event_elapsed_ms(void* start, void* end, float* ms);
int  tl_stream_wait_event(void* stream, void* event);

/* CUDA graph capture of a stream: replaces the reference's per-iteration
 * kernel-by-kernel replay of a for-loop body (compiler.py:206-303). */
int  tl_graph_begin(void* stream);
int  tl_graph_end(void* stream, void** graph_exec);
int  tl_graph_launch(void* graph_exec, void* stream);
int  tl_graph_destroy(void* graph_exec);
/* Graphs are instantiated with the nodes' own priorities, so that kernels
 * captured from tl_stream_create_priority(urgent) streams (the gradient
 * all-reduce) keep their priority when the graph replays.  Kernel nodes of
 * the last graph captured on the calling thread, and how many of them carry
 * a non-default priority. */
int  tl_graph_last_stats(int* kernel_nodes, int* prioritised_nodes);

/* Number of kernels this library has launched on the calling thread since
 * the last reset (graph replays are not counted). */
int  tl_launch_counter(uint64_t* count, int reset);

/* ---- fused elementwise regions (run-time compiled) ---------------------
 * Replaces the per-op elementwise launchers: elementwise
 * (kernel_generator.py:246-275), binary_broadcast (:281-348),
 * binary_1d_broadcast (:354-377), binary_general_broadcast (:383-463),
 * fill (:469-488), relu/sigmoid/tanh (:209-240, 531-558), greater/less/equal
 * (:646-778) and the fused SGD update of the rebind pattern
 * (compiler.py:309-347).  The host generates one CUDA kernel per fused
 * region; NVRTC compiles it for sm_100a; the cubin is cached in memory and
 * under `cache_dir` (may be NULL) keyed by `key`.
 */
int  tl_jit_compile(const char* source, const char* kernel_name, const char* key,
                    const char* cache_dir, void** function);
const char* tl_jit_log(void);                   /* last NVRTC log on this thread */
int  tl_jit_launch(void* function, unsigned grid, unsigned block, unsigned smem,
                   void** args, void* stream);

/* ---- reductions -----------------------------------------------------------
 * op codes for tl_reduce_*.
 * Replaces sum (kernel_generator.py:784-882), mean (:888-989),
 * max (:1246-1345), min (:1352-1453), argmax (:1459-1542), argmin (:1549-1578).
 * Sums accumulate in float64 and round once; argmax/argmin return the first
 * index of the extreme value (strict compare scan, as the reference's
 * axis kernels do).
 */
#define TL_RED_SUM    0
#define TL_RED_MEAN   1
#define TL_RED_MAX    2
#define TL_RED_MIN    3
#define TL_RED_ARGMAX 4
#define TL_RED_ARGMIN 5

/* out[r] = op over in[r, :]          (axis=1 of a [rows, cols] tensor) */
int  tl_reduce_rows(int op, const float* in, float* out, int64_t rows, int64_t cols,
                    void* stream);
/* out[c] = op over in[:, c]          (axis=0) */
size_t tl_reduce_cols_scratch_bytes(int op, int64_t rows, int64_t cols);
int  tl_reduce_cols(int op, const float* in, float* out, int64_t rows, int64_t cols,
                    void* scratch, void* stream);
/* Same result as tl_reduce_cols, but allocates nothing and takes no scratch
 * argument.  No counterpart in the reference: it exists for callers that
 * cannot allocate device memory (a plugin inside a host framework that owns
 * every device allocation, or a fixed-budget path that must not allocate
 * while it runs).  Its scratch is a 1 MiB file-scope device array of the
 * library, held by every GPU that loads the library until the process exits.
 * cols may be at most 64512 for argmax/argmin and 129024 for the other ops
 * ((1 MiB - 16 KiB of completion counters) / 16 or / 8 bytes of partials per
 * column), whatever the alignment of `in` or the remainder of cols / 4;
 * larger sizes return TL_ERR_INVALID_ARG without launching anything.  Each
 * call looks up the array's device address (cudaGetSymbolAddress) on the
 * current device; the first call on a device also loads the module there and
 * should come before any stream capture.  All calls share the array: calls
 * whose kernels overlap on the GPU race, so issue them in one stream order. */
int  tl_reduce_cols_noalloc(int op, const float* in, float* out, int64_t rows, int64_t cols,
                            void* stream);
/* out[0] = op over all n elements    (axis=None) */
size_t tl_reduce_full_scratch_bytes(int op, int64_t n);
int  tl_reduce_full(int op, const float* in, float* out, int64_t n,
                    void* scratch, void* stream);

/* ---- softmax and normalisation ---------------------------------------------
 * softmax (kernel_generator.py:564-640): exp(x-max)/sum along the row.
 * layer_norm (:1667-1810) and instance_norm (:2017-2061): population
 * statistics, (x-mean)/sqrt(var+eps), no affine parameters.
 * batch_norm (:1978-2011): running statistics per column.
 */
int  tl_softmax_rows(const float* in, float* out, int64_t rows, int64_t cols, void* stream);
size_t tl_norm_cols_scratch_bytes(int64_t rows, int64_t cols);
int  tl_layer_norm_rows(const float* in, float* out, int64_t rows, int64_t cols,
                        float eps, void* stream);
int  tl_layer_norm_cols(const float* in, float* out, int64_t rows, int64_t cols,
                        float eps, void* scratch, void* stream);
int  tl_batch_norm(const float* in, const float* running_mean, const float* running_var,
                   float* out, int64_t rows, int64_t cols, float eps, void* stream);

/* ---- losses -------------------------------------------------------------
 * mse_loss (kernel_generator.py:1891-1943): mean((p-t)^2).
 * cross_entropy (:1816-1885): class-index targets (float values clamped to
 * [0, C-1]) when onehot == 0; one-hot targets [B, C] when onehot != 0.
 * The probability is clamped to [1e-7, 1-1e-7] before -log.
 */
size_t tl_loss_scratch_bytes(int64_t n);
int  tl_mse_loss(const float* pred, const float* target, float* out, int64_t n,
                 void* scratch, void* stream);
int  tl_cross_entropy(const float* probs, const float* target, float* out,
                      int64_t batch, int64_t classes, int onehot,
                      void* scratch, void* stream);

/* ---- reverse-mode kernels (tensorlang/autograd.py on the device) --------- */
/* softmax VJP along rows, autograd.py:563-580: dx = s*(g - sum(g*s)) */
int  tl_softmax_backward_rows(const float* s, const float* g, float* dx,
                              int64_t rows, int64_t cols, int accumulate, void* stream);
/* cross_entropy VJP (autograd.py:691-704) fused with the softmax VJP that
 * follows it: gp = (p - t) / divisor * upstream[0] (divisor = the global
 * batch; upstream may be NULL for 1.0), written to dp when non-null, and
 * dz = gp*p - p*sum(gp*p) written (or added) to dz.  Class-index targets
 * (onehot == 0) use one-hot(t). */
int  tl_ce_softmax_backward(const float* p, const float* target, int onehot,
                            const float* upstream, float divisor,
                            float* dp, float* dz, int64_t rows, int64_t cols,
                            int accumulate, void* stream);
/* layer_norm VJP along rows, autograd.py:649-674 */
int  tl_layer_norm_backward_rows(const float* x, const float* g, float* dx, int64_t rows,
                                 int64_t cols, float eps, int accumulate, void* stream);

/* ---- data movement --------------------------------------------------------
 * transpose (kernel_generator.py:1949-1972), slice (:1112-1240),
 * concat (:2092-2132), reshape (:2067-2086, a copy).
 */
int  tl_transpose2d(const float* in, float* out, int64_t rows, int64_t cols, void* stream);
int  tl_slice2d(const float* in, float* out, int64_t in_cols, int64_t row_start,
                int64_t col_start, int64_t out_rows, int64_t out_cols, void* stream);
int  tl_concat_rows(const float* a, const float* b, float* out, int64_t rows_a,
                    int64_t rows_b, int64_t cols, void* stream);

/* ---- GEMM -----------------------------------------------------------------
 * Replaces matmul (kernel_generator.py:501-525) and linear (:1584-1661), and
 * serves the matmul/linear VJPs (autograd.py:520-537, 619-646).
 *   C[M,N] (+)= op(A)[M,K] @ op(B)[K,N] (+ bias[N]) (then epilogue)
 * op(X) = X when trans == 0, X^T when trans != 0; leading dimensions in
 * elements of the row-major storage.  f32 in, f32 out.  On sm_100a the
 * product runs on tcgen05 tensor cores as split-TF32 (three TF32 products
 * hi*hi + hi*lo + lo*hi with fp32 accumulation in tensor memory), which
 * keeps fp32-level accuracy (the default operand scheme splits each operand
 * into two bf16 terms instead; see tl_gemm_set_scheme); skinny products (N <= 32, or K <= 32 with B
 * transposed) take bandwidth-bound CUDA-core kernels; other shapes the TMA
 * path cannot describe take a tiled fp32 CUDA-core path.
 * epilogue: 0 none, 1 relu (y = max(0, y)).
 * accumulate: 0 overwrite C, 1 C += result.
 */
#define TL_EPI_NONE 0
#define TL_EPI_RELU 1
int  tl_gemm(int trans_a, int trans_b, int64_t M, int64_t N, int64_t K,
             const float* A, int64_t lda, const float* B, int64_t ldb,
             float* C, int64_t ldc, const float* bias, int accumulate, int epilogue,
             void* stream);
/* tl_gemm with a relu-mask epilogue (no reference counterpart: it fuses the
 * relu VJP grad * (x > 0) -- autograd.py:540-544 -- into the GEMM that
 * produces grad):  C (+)= epilogue(op(A) op(B) + bias) * (mask[m, n] > 0 ? 1 : 0),
 * the product rounded to nearest as a separate multiply.  mask is [M][ldm]
 * (ldm >= N) and may be null (then this is tl_gemm).  Every path of tl_gemm
 * supports it. */
int  tl_gemm_masked(int trans_a, int trans_b, int64_t M, int64_t N, int64_t K,
                    const float* A, int64_t lda, const float* B, int64_t ldb,
                    float* C, int64_t ldc, const float* bias, int accumulate, int epilogue,
                    const float* mask, int64_t ldm, void* stream);
/* Precomputed bf16 pair matrices for the TF32+bf16 and BF16X3 schemes (no
 * reference counterpart).  Both multiply on a pair matrix per operand (bf16
 * values beside bf16 lows; the low part depends on the scheme selected when
 * the pair is prepared); tl_gemm computes those pairs itself on every
 * call.  A caller that uses one operand in several products, or the same
 * operand over many calls, prepares its pairs once:
 *   tl_gemm_pair_bytes(rows, cols, layout)   bytes of the pair of X[rows][cols]
 *     layout TL_PAIR_KMAJOR  (X is [MN][K]): rows x ceil32(cols) x 4
 *     layout TL_PAIR_MNMAJOR (X is [K][MN]): ceil32(rows) x ceil8(cols) x 4
 *   tl_gemm_pair_prepare(X, ld, rows, cols, kmajor, klo, mnmajor, mlo, stream)
 *     writes either or both layouts from one read of X (16-byte aligned
 *     outputs; null skips one); *lo_first = 1 for a B operand, 0 for A
 *   tl_gemm_pairs(..., A, lda, a_pair, B, ldb, b_pair, ...)
 *     tl_gemm_masked taking those pairs (null: computed inside as usual).
 *     The layout an operand needs: A as stored (trans_a 0) -> K-major, A^T
 *     (trans_a 1) -> MN-major; B^T as stored (trans_b 1) -> K-major, B
 *     (trans_b 0) -> MN-major.  Paths other than the pair-scheme tensor-core
 *     path ignore the pairs.
 *   tl_gemm_uses_pairs(ta, tb, M, N, K, lda, ldb)  1 if such a call takes
 *     that path (so prepared pairs are used), else 0; depends only on the
 *     shapes and the selected scheme. */
#define TL_PAIR_KMAJOR 0
#define TL_PAIR_MNMAJOR 1
int64_t tl_gemm_pair_bytes(int64_t rows, int64_t cols, int layout);
int  tl_gemm_pair_prepare(const float* X, int64_t ld, int64_t rows, int64_t cols,
                          void* kmajor, int kmajor_lo_first, void* mnmajor,
                          int mnmajor_lo_first, void* stream);
/* tl_gemm_pair_prepare that also writes colsum[c] = sum over rows of X[r][c]
 * (summed in double, rounded once) from the same read of X: the bias
 * gradient db of a linear layer (autograd.py:619-646, replacing the separate
 * tl_reduce_cols sum over the same dY that the reference's backward runs).
 * scratch: at least tl_gemm_pair_colsum_scratch_bytes(rows, cols) bytes,
 * 8-byte aligned (per-block partial sums); cols up to 8192.  The result may
 * differ from tl_reduce_cols(TL_RED_SUM) in the last bit of a float where
 * the two double sums round differently.  No reference counterpart as a
 * single call. */
size_t tl_gemm_pair_colsum_scratch_bytes(int64_t rows, int64_t cols);
int  tl_gemm_pair_prepare_colsum(const float* X, int64_t ld, int64_t rows, int64_t cols,
                                 void* kmajor, int kmajor_lo_first, void* mnmajor,
                                 int mnmajor_lo_first, float* colsum, void* scratch,
                                 size_t scratch_bytes, void* stream);
int  tl_gemm_pairs(int trans_a, int trans_b, int64_t M, int64_t N, int64_t K,
                   const float* A, int64_t lda, const void* a_pair,
                   const float* B, int64_t ldb, const void* b_pair,
                   float* C, int64_t ldc, const float* bias, int accumulate, int epilogue,
                   const float* mask, int64_t ldm, void* stream);
int  tl_gemm_uses_pairs(int trans_a, int trans_b, int64_t M, int64_t N, int64_t K,
                        int64_t lda, int64_t ldb);
/* Which path tl_gemm would take (0 tensor-core, 1 CUDA-core) for this call. */
int  tl_gemm_path(int trans_a, int trans_b, int64_t M, int64_t N, int64_t K,
                  const float* A, int64_t lda, const float* B, int64_t ldb,
                  const float* C, int64_t ldc);
/* The tensor-core launch for an M x N x K product (no reference
 * counterpart; host-only, no GPU needed): plan[0] 0 for 128 x 256 single-CTA
 * tiles, 1 for 256 x 256 CTA-pair tiles on the static schedule, 2 on the
 * dynamic one (tl_gemm_set_tile_schedule); plan[1] K splits; plan[2] tiles
 * each cluster launch starts with; plan[3] clusters (CTA pairs) or CTAs
 * launched.  Uses this device's SM count (148 when no GPU is visible). */
int  tl_gemm_tc_plan(int64_t M, int64_t N, int64_t K, int* plan);
/* Path selection: 0 automatic (tensor cores when the shape allows, the raw
 * operand as the TF32 "hi" part); 1 force the CUDA-core path; 2 automatic,
 * with hi and lo both rounded to TF32 explicitly in the pre-pass. */
int  tl_gemm_force_simt(int force);
/* Tensor-core operand scheme for fp32 products (no reference counterpart:
 * the reference calls cuBLAS SGEMM / its own fp32 kernels).
 *   TL_GEMM_3XTF32     hi*hi + hi*lo + lo*hi, three TF32 MMAs per k-step
 *   TL_GEMM_TF32_BF16  hi*hi on TF32, both correction terms in one bf16 MMA
 *                      over [bf16(A)|bf16(loA)] . [bf16(loB)|bf16(B)]
 *   TL_GEMM_BF16X3     all bf16: a = a0 + a1 with a0 = bf16(a), a1 =
 *                      bf16(a - a0); a0*b0 plus one pair MMA over
 *                      [a0|a1] . [b1|b0]; operands are read only as pairs
 *                      (default: 3 bf16 MMA-times per product against 4,
 *                      half the operand bytes; max rel err ~5e-6 against
 *                      ~1.6e-6)
 * All stay within rel 1e-5 of an fp64 product on N(0,1) data.  Returns
 * TL_ERR_INVALID_ARG for an unknown scheme; *previous (if non-null) receives
 * the scheme that was in force.  Applies to launches made after the call;
 * pair matrices (tl_gemm_pair_prepare) are scheme-specific, so switch the
 * scheme before preparing a program, not between its launches. */
#define TL_GEMM_3XTF32 0
#define TL_GEMM_TF32_BF16 1
#define TL_GEMM_BF16X3 2
int  tl_gemm_set_scheme(int scheme, int* previous);
/* Tile shape of the tensor-core path (no reference counterpart).  enable = 1
 * (default): products with more than 128 rows use 256 x 256 tiles computed by
 * a cluster of two CTAs with tcgen05.mma.cta_group::2, each CTA loading half
 * of B; enable = 0: 128 x 256 single-CTA tiles only.  *previous (if non-null)
 * receives the setting that was in force. */
int  tl_gemm_set_cta_pair(int enable, int* previous);
/* Tile schedule of the 256 x 256 CTA-pair kernel (no reference
 * counterpart).  dynamic = 0: static groups -- each cluster launch computes
 * up to four consecutive tiles in turn on launches of many waves, one tile
 * otherwise, and the hardware balances the cluster launches; dynamic = 1:
 * one tile per cluster launch, and each running cluster goes on with the
 * tiles of clusters that have not started (sm_100 cluster launch control:
 * the launch of a pending cluster is cancelled and its tile computed by the
 * running one), so an SM pair computes tiles back to back, its stage ring
 * and accumulators running on, until none are left; dynamic = 2 (default):
 * dynamic for launches the static schedule leaves at one tile per cluster
 * and for K <= 1024, static otherwise.  Results are bit-identical under
 * every schedule.  *previous (if non-null) receives the setting that was in
 * force. */
int  tl_gemm_set_tile_schedule(int dynamic, int* previous);
/* How the CTA-pair kernel's epilogue writes its tiles (no reference
 * counterpart).  tma = 1 (default): each epilogue warp stages 32 x 32 slabs of
 * its rows in shared memory (128-byte swizzle) and stores them with TMA,
 * whole 128-byte row segments at a time, wherever the output has a 16-byte
 * aligned base and rows (split-K partial sums too); accumulate and other
 * layouts keep the per-row stores.  tma = 0: every lane stores its own row
 * (16 bytes per lane per instruction, 32 rows per warp store).  Results are
 * bit-identical either way.  *previous (if non-null) receives the setting
 * that was in force. */
int  tl_gemm_set_store_path(int tma, int* previous);
/* ---- classifier head of a training step, fused ---------------------------
 * linear (kernel_generator.py:1584-1661) with N <= 16 outputs, row softmax
 * (:564-640) and cross_entropy (:1816-1885), and their backward:
 * the cross_entropy VJP chained through the softmax VJP (autograd.py:691-704,
 * :563-580) and the linear VJP's dX (:619-646) with the relu-VJP mask of the
 * layer below (autograd.py:540-544), in one pass over A [M, K]:
 *   z = A W + bias; p = softmax(z); dp = (p - t) / divisor * upstream[0];
 *   dz = dp p - p sum(dp p); dx = (dz W^T) * (mask > 0).
 * W is [K, N] with leading dimension ldw; target one-hot [M, N] (onehot 1)
 * or class indices [M] (onehot 0); z, p, dp, dz ([M, N], leading dimension
 * N) are written when non-null; dx [M, K] (leading dimension lddx) and mask
 * [M, K] (leading dimension ldm) are required.  The results are
 * bit-identical to tl_gemm + tl_softmax_rows + tl_ce_softmax_backward +
 * tl_gemm_masked on the same operands; the loss itself is tl_cross_entropy's
 * (it reads p).  tl_head_ce_ok tells whether a shape is supported (N <= 16,
 * K a multiple of 4, 16-byte aligned A, dx and mask, lda, lddx and ldm
 * multiples of 4, M * K >= 65536); other shapes return TL_ERR_UNSUPPORTED.
 * No reference counterpart as one call. */
int  tl_head_ce_ok(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda,
                   const float* dx, int64_t lddx);
int  tl_head_ce(const float* A, int64_t lda, const float* W, int64_t ldw, const float* bias,
                const float* target, int onehot, const float* upstream, float divisor,
                float* z, float* p, float* dp, float* dz, float* dx, int64_t lddx,
                const float* mask, int64_t ldm, int64_t M, int64_t N, int64_t K, void* stream);

/* Device-side error flag (TL_ERR_TIMEOUT after a bounded wait in a kernel
 * gave up; 0 if none).  reset != 0 clears it. */
int  tl_device_error(int* code, int reset);

/* ---- data-parallel gradient exchange (NCCL over NVLink) ------------------
 * The reference has no multi-GPU path (README.md:583 lists it as future work);
 * these back the data-parallel for-loop executor.  libnccl.so.2 is loaded on
 * first use.  Communicators are created non-blocking; tl_nccl_wait polls for
 * completion and asynchronous errors up to timeout_ms and returns
 * TL_ERR_TIMEOUT (after aborting the communicator) if it passes.
 */
int  tl_nccl_unique_id(unsigned char id[128]);
int  tl_nccl_comm_init(void** comm, int nranks, const unsigned char id[128], int rank,
                       int timeout_ms);
int  tl_nccl_allreduce_sum(void* comm, float* buf, size_t count, void* stream);
int  tl_nccl_wait(void* comm, void* stream, int timeout_ms);
int  tl_nccl_comm_destroy(void* comm);
int  tl_nccl_comm_abort(void* comm);

#ifdef __cplusplus
}
#endif
#endif /* TLB200_H */
