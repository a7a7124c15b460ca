/*
 * kbb200.h — C ABI of the B200 (sm_100a) fp32 operator library.
 *
 * One shared library (libkbb200.so) exports every entry point below as plain
 * `extern "C"` functions: device pointers, element counts and a CUDA stream,
 * no torch types.  Each entry replaces the compiled entry of one candidate of
 * the reference operator library (candidates/<problem>/v*.py, whose C++ entry
 * took torch::Tensor arguments and launched on the current stream).
 *
 * Conventions (all entries):
 *   - Pointers are device pointers to contiguous fp32 data unless stated.
 *   - Launches are asynchronous on `stream` (NULL = legacy default stream).
 *   - Inputs are never written.  Outputs are fully overwritten.
 *   - Entries never allocate device memory.  Entries that need scratch take
 *     (workspace, workspace_bytes); query the size with the matching
 *     *_workspace_size() call.  Workspace need not be initialised.
 *   - Return KB_OK (0) or a kbStatus code; kb_last_error() describes the most
 *     recent failure on the calling thread.
 *   - Empty inputs (n == 0, rows == 0, ...) are valid and launch nothing,
 *     except reductions to a scalar, which write their identity result.
 */
#ifndef KBB200_H
#define KBB200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define KB_API __attribute__((visibility("default")))
#else
#define KB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* kbStream; /* same handle type as cudaStream_t */

typedef enum kbStatus {
  KB_OK = 0,
  KB_ERR_INVALID_ARG = 1,   /* bad size, null pointer, misaligned scratch */
  KB_ERR_UNSUPPORTED = 2,   /* shape outside the kernel's contract */
  KB_ERR_WORKSPACE = 3,     /* workspace missing or smaller than required */
  KB_ERR_CUDA = 4,          /* CUDA runtime error (launch / attribute) */
  KB_ERR_DEVICE = 5         /* device is not sm_100 class */
} kbStatus;

/* ---- library / diagnostics ------------------------------------------- */
KB_API int kb_version(void);                 /* MAJOR*10000 + MINOR*100 + PATCH */
KB_API const char* kb_status_string(int status);
KB_API const char* kb_last_error(void);      /* thread-local, never NULL */
KB_API int kb_device_sm_count(int device);   /* streaming multiprocessors, or -1 */
/* Device fault word of the current device: nonzero once a kernel gave up a
 * bounded wait (a pipeline stalled for > 2 s) and returned early instead of
 * hanging; its outputs are then invalid.  Synchronous; clear != 0 resets. */
KB_API int kb_read_fault(int clear, int* value);

/* ---- elementwise (y = f(x), n elements) ------------------------------- */
/* replaces mingpt_gelu_entry, candidates/88_MinGPTNewGelu/v1.py:21-26
 * y = 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))                      */
KB_API int kb_gelu_tanh_f32(const float* x, float* y, int64_t n, kbStream stream);
/* replaces gelu_entry, candidates/26_GELU_/v1.py:18-23 (exact erf form)    */
KB_API int kb_gelu_erf_f32(const float* x, float* y, int64_t n, kbStream stream);
/* replaces swish_entry, candidates/25_Swish/v1.py:18-23: y = x sigmoid(x)  */
KB_API int kb_swish_f32(const float* x, float* y, int64_t n, kbStream stream);
/* replaces relu_entry, candidates/19_ReLU/v1.py:15-20: y = max(x, 0)       */
KB_API int kb_relu_f32(const float* x, float* y, int64_t n, kbStream stream);

/* replaces diagmul_entry, candidates/12_Matmul_with_diagonal_matrices_/
 * v1.py:19-27: y[i, j] = a[i] * b[i, j], i.e. diag(a) @ B for a[rows],
 * b[rows, cols] — a broadcast row scale, never the rows x rows matrix.      */
KB_API int kb_diag_matmul_f32(const float* a, const float* b, float* y,
                              int64_t rows, int64_t cols, kbStream stream);

/* ---- row normalisation over the last `cols` elements of each row ------ */
/* replaces layernorm_entry, candidates/40_LayerNorm/v1.py:62-80.
 * gamma/beta may be NULL (identity affine).  Biased variance, eps inside
 * the square root, as torch.nn.functional.layer_norm.                      */
KB_API int kb_layernorm_f32(const float* x, const float* gamma, const float* beta,
                     float* y, int64_t rows, int64_t cols, float eps,
                     kbStream stream);
/* replaces rmsnorm_entry, candidates/36_RMSNorm_/v3.py:42-51.
 * x is viewed as [outer, features, inner]; each (outer, inner) position is
 * normalised over `features`: y = x / sqrt(mean(x^2) + eps) * gamma[f].
 * inner == 1 is the last-dim form; inner > 1 the channel (dim 1) form.
 * gamma may be NULL.                                                      */
KB_API int kb_rmsnorm_f32(const float* x, const float* gamma, float* y,
                   int64_t outer, int64_t features, int64_t inner, float eps,
                   kbStream stream);
/* replaces softmax_entry, candidates/23_Softmax/v1.py:47-52 (last dim)     */
KB_API int kb_softmax_f32(const float* x, float* y, int64_t rows, int64_t cols,
                   kbStream stream);
/* replaces logsoftmax_entry, candidates/24_LogSoftmax/v1.py:46-51          */
KB_API int kb_logsoftmax_f32(const float* x, float* y, int64_t rows, int64_t cols,
                      kbStream stream);

/* ---- reductions over dim 1 of x[B, I, J] ------------------------------ */
/* replaces colreduce_entry, candidates/47_Sum_reduction_over_a_dimension/
 * v1.py:28-35: out[b, j] = sum_i x[b, i, j]                                */
KB_API int kb_sum_dim1_f32(const float* x, float* out, int64_t B, int64_t I,
                    int64_t J, kbStream stream);
/* replaces colreduce_mean_entry, candidates/48_Mean_reduction_over_a_
 * dimension/v1.py:25-32: out[b, j] = sum_i x[b, i, j] / I                  */
KB_API int kb_mean_dim1_f32(const float* x, float* out, int64_t B, int64_t I,
                     int64_t J, kbStream stream);
/* replaces argmax_entry, candidates/51_Argmax_over_a_dimension/v1.py:27-31.
 * out[b, j] = lowest i attaining the maximum; NaN counts as the maximum
 * (torch.argmax).  out is int64.                                          */
KB_API int kb_argmax_dim1_f32(const float* x, int64_t* out, int64_t B, int64_t I,
                       int64_t J, kbStream stream);

/* ---- global reductions ------------------------------------------------ */
/* replaces mse_entry, candidates/94_MSELoss/v1.py:35-45:
 * out[0] = mean((a - b)^2) over n elements (deterministic order).          */
KB_API size_t kb_mse_workspace_size(int64_t n);
KB_API int kb_mse_f32(const float* a, const float* b, float* out, int64_t n,
               void* workspace, size_t workspace_bytes, kbStream stream);
/* sharded form: partial[0] = sum((a - b)^2) over this shard and
 * partial[1] = n, both fp64 (16 bytes), so one collective adds the sums and
 * the counts of all shards; kb_mse_finalize_f32 divides by total_n, or by
 * total[1] when total_n is 0 (shards of any sizes, empty ones included).  */
KB_API int kb_mse_partial_f64(const float* a, const float* b, double* partial,
                       int64_t n, void* workspace, size_t workspace_bytes,
                       kbStream stream);
KB_API int kb_mse_finalize_f32(const double* total, float* out, int64_t total_n,
                        kbStream stream);

/* replaces frobenius_entry, candidates/37_FrobeniusNorm_/v1.py:48-58:
 * y = x / ||x||_F over all n elements.                                    */
KB_API size_t kb_frobenius_workspace_size(int64_t n);
KB_API int kb_frobenius_normalize_f32(const float* x, float* y, int64_t n,
                               void* workspace, size_t workspace_bytes,
                               kbStream stream);
/* sharded form: sumsq[0] = sum(x^2) over this shard (fp64), then
 * y = x / sqrt(total) once a collective has summed the shards.            */
KB_API int kb_sumsq_partial_f64(const float* x, double* sumsq, int64_t n,
                         void* workspace, size_t workspace_bytes,
                         kbStream stream);
KB_API int kb_scale_by_inv_norm_f32(const float* x, float* y, int64_t n,
                             const double* total_sumsq, kbStream stream);

/* ---- spatial ---------------------------------------------------------- */
/* replaces maxpool_entry, candidates/42_Max_Pooling_2D/v1.py:37-44, with
 * stride and dilation honoured (the reference kernel ignored both).
 * NCHW; padding is -inf; NaN propagates as in torch.max_pool2d.            */
KB_API int kb_maxpool2d_f32(const float* x, float* y, int64_t N, int64_t C,
                     int64_t H, int64_t W, int64_t OH, int64_t OW,
                     int kernel, int stride, int pad, int dilation,
                     kbStream stream);

/* replaces bn_entry, candidates/33_BatchNorm/v1.py:53-68: training-mode
 * BatchNorm2d over NCHW x with batch statistics (biased variance).
 * gamma/beta may be NULL.  running_mean/running_var may be NULL; when given
 * they are updated in place with `momentum` and the unbiased variance,
 * as torch.nn.BatchNorm2d does in training mode.                          */
KB_API size_t kb_batchnorm_workspace_size(int64_t N, int64_t C, int64_t HW);
KB_API int kb_batchnorm_train_f32(const float* x, const float* gamma,
                           const float* beta, float* y, int64_t N, int64_t C,
                           int64_t HW, float eps, float momentum,
                           float* running_mean, float* running_var,
                           void* workspace, size_t workspace_bytes,
                           kbStream stream);
/* Allocation-free training-mode BatchNorm: no counterpart in the reference.
 * Same arguments and results as kb_batchnorm_train_f32 minus the workspace,
 * for callers that may not allocate device memory themselves: libraries
 * running inside a host framework that owns every device allocation through
 * its own pool or budget, and latency-bound loops where cudaMalloc's implicit
 * device synchronisation is not acceptable.  The per-channel partial sums
 * live in a 128 KiB file-scope device array (8192 fp64 pairs) that every
 * device loading the library keeps until process exit, so C * splits must be
 * <= 8192, where splits = max(1, min(N, ceil(4 * SMs / C))), so any
 * C <= 8192 fits on a 148-SM B200.  Larger C returns KB_ERR_UNSUPPORTED.  Each
 * call looks up the array's device address on the current device
 * (cudaGetSymbolAddress), so the address stays valid across a
 * cudaDeviceReset; the first call on a device also loads the module there,
 * so make it before any stream capture.  Every call
 * shares the one array, so calls that overlap on the GPU (for example on two
 * streams) race; the caller must serialise them.  Calls no cudaMalloc.     */
KB_API int kb_batchnorm_train_f32_noalloc(const float* x, const float* gamma,
                                          const float* beta, float* y, int64_t N,
                                          int64_t C, int64_t HW, float eps,
                                          float momentum, float* running_mean,
                                          float* running_var, kbStream stream);
/* sharded form: stats[0:C] = per-channel sum, stats[C:2C] = per-channel sum
 * of squares, stats[2C] = elements per channel (N * HW) over this shard,
 * 2C + 1 doubles; a collective adds them across shards, then
 * kb_batchnorm_apply_f32 normalises with `total_count` elements per channel,
 * or with stats[2C] when total_count is 0 (shards of any sizes).  A shard
 * with no elements still updates running_mean / running_var.              */
KB_API int kb_batchnorm_stats_f64(const float* x, double* stats, int64_t N,
                           int64_t C, int64_t HW, void* workspace,
                           size_t workspace_bytes, kbStream stream);
KB_API int kb_batchnorm_apply_f32(const float* x, const float* gamma,
                           const float* beta, float* y, const double* stats,
                           int64_t N, int64_t C, int64_t HW,
                           int64_t total_count, float eps, float momentum,
                           float* running_mean, float* running_var,
                           kbStream stream);

/* ---- dense contractions ----------------------------------------------- */
/* replaces sgemm_entry, candidates/1_Square_matrix_multiplication_/
 * v1.py:83-102: C[M,N] = op(A) B with op(A) = A[M,K] (trans_a = 0) or
 * A[K,M]^T (trans_a = 1); B[K,N]; row-major with leading dimensions.
 * 3xTF32 on tcgen05 tensor cores: fp32-level accuracy.                     */
KB_API int kb_sgemm_3xtf32(const float* A, const float* B, float* C, int64_t M,
                    int64_t N, int64_t K, int64_t lda, int64_t ldb,
                    int64_t ldc, int trans_a, kbStream stream);
/* The same GEMM with a caller workspace: when the output has fewer tiles
 * than the GPU has SMs (e.g. a 256-row strip of an 8192-wide, 8192-deep
 * GEMM: 64 tiles on 148 SMs), K is split into s parts whose partial tiles
 * go to the workspace and are summed in a fixed order (deterministic).
 * kb_sgemm_workspace_size returns s * M * N * 4 bytes, or 0 when no split
 * pays; a smaller workspace runs the GEMM unsplit.  trans_a is never split.
 * Replaces sgemm_entry, candidates/1_Square_matrix_multiplication_/v1.py:83-102. */
KB_API size_t kb_sgemm_workspace_size(int64_t M, int64_t N, int64_t K, int trans_a);
KB_API int kb_sgemm_3xtf32_ws(const float* A, const float* B, float* C, int64_t M,
                              int64_t N, int64_t K, int64_t lda, int64_t ldb,
                              int64_t ldc, int trans_a, void* workspace,
                              size_t workspace_bytes, kbStream stream);
/* replaces sgemm_entry batched mode, candidates/3_Batched_matrix_
 * multiplication/v1.py:83-102 (with C's row stride = N, fixing the ldc
 * bug there): C[b] = A[b] B[b] for contiguous A[batch,M,K], B[batch,K,N].  */
KB_API int kb_bgemm_3xtf32(const float* A, const float* B, float* C, int64_t batch,
                    int64_t M, int64_t N, int64_t K, kbStream stream);
/* replaces splitk_gemm_entry, candidates/6_Matmul_with_large_K_dimension_/
 * v1.py:67-78: C[M,N] = A[M,K] B[K,N] with K split across the SMs and a
 * deterministic reduction of the partial tiles (no atomics).               */
KB_API size_t kb_gemm_splitk_workspace_size(int64_t M, int64_t N, int64_t K);
KB_API int kb_gemm_splitk_3xtf32(const float* A, const float* B, float* C,
                          int64_t M, int64_t N, int64_t K, void* workspace,
                          size_t workspace_bytes, kbStream stream);
/* replaces gemv_entry, candidates/4_Matrix_vector_multiplication_/
 * v1.py:36-43: y[M] = A[M,K] x[K] (deterministic, no atomics).            */
KB_API int kb_gemv_f32(const float* A, const float* x, float* y, int64_t M,
                int64_t K, kbStream stream);

/* ---- problems the reference lists but never attempted ------------------
 * harness/problems.py:45-56 names 45_Average_Pooling_2D, 89_cumsum and
 * 95_CrossEntropyLoss, and scripts/milestone_table.py:16-24 marks them not
 * attempted, so these entries replace no reference entry; they follow the
 * torch semantics named on each.                                          */
/* torch.nn.functional.avg_pool2d (floor mode) over NCHW: the window sum
 * (padding counts as 0) divided by the window's size clipped to the padded
 * input (count_include_pad != 0), to the real input (count_include_pad == 0),
 * or by divisor_override when it is nonzero.                              */
KB_API int kb_avgpool2d_f32(const float* x, float* y, int64_t N, int64_t C,
                     int64_t H, int64_t W, int64_t OH, int64_t OW, int kernel,
                     int stride, int pad, int count_include_pad,
                     int divisor_override, kbStream stream);
/* torch.cumsum(x, dim) for x viewed as [outer, len, inner] with dim the
 * middle axis: y[o, i, j] = sum_{k <= i} x[o, k, j] (inclusive).          */
KB_API int kb_cumsum_f32(const float* x, float* y, int64_t outer, int64_t len,
                  int64_t inner, kbStream stream);
/* torch.nn.functional.cross_entropy(logits[rows, classes], targets[rows]
 * int64, reduction='mean', ignore_index): out[0] = mean over rows whose
 * target is not ignore_index of logsumexp(logits[i]) - logits[i, t_i];
 * deterministic.  A target outside [0, classes) gives NaN.                */
KB_API size_t kb_cross_entropy_workspace_size(int64_t rows);
KB_API int kb_cross_entropy_f32(const float* logits, const int64_t* targets,
                         float* out, int64_t rows, int64_t classes,
                         int64_t ignore_index, void* workspace,
                         size_t workspace_bytes, kbStream stream);
/* sharded form: total[0..1] = (sum of row losses, number of rows not
 * ignored) over this shard (fp64); after a collective has summed the
 * shards' totals, out[0] = total[0] / total[1].                           */
KB_API int kb_cross_entropy_partial_f64(const float* logits, const int64_t* targets,
                                 double* total, int64_t rows, int64_t classes,
                                 int64_t ignore_index, void* workspace,
                                 size_t workspace_bytes, kbStream stream);
KB_API int kb_cross_entropy_finalize_f32(const double* total, float* out, kbStream stream);

/* ---- cross-GPU reduction over peer memory ------------------------------
 * The sharded forms of MSE, Frobenius, BatchNorm, split-K GEMM and
 * cross-entropy exchange one small partial per rank.  The reference runs on
 * one GPU and has no collective; these entries replace the NCCL all_reduce
 * between each partial entry and its finish entry with one cooperative
 * kernel over peer memory (CUDA IPC over NVLink, no multicast):
 *   buffer   kb_p2p_buffer_alloc(kb_p2p_buffer_bytes(payload, world), &p) on
 *            every rank (zeroed); kb_p2p_ipc_handle / kb_p2p_ipc_open share
 *            it; `bufs` is a DEVICE array of the world base pointers (own at
 *            [rank]).  Each rank pushes its contribution into every rank's
 *            buffer, so payload bytes per call <= the `payload` given here.
 *   call     every rank makes the same calls in the same order with the
 *            same epoch, starting at 1 and increasing by 1 per call;
 *            dst = sum over ranks of src (rank order: bit-identical on all
 *            ranks).  src may equal dst.
 *   failure  a wait longer than timeout_ns records (phase << 8 | peer) in
 *            the fault word (kb_p2p_read_fault) and writes NaN into dst;
 *            the buffer set must then be discarded.                       */
KB_API size_t kb_p2p_header_bytes(void);
KB_API size_t kb_p2p_buffer_bytes(size_t payload_bytes, int world);
KB_API int kb_p2p_buffer_alloc(size_t bytes, void** ptr);
KB_API int kb_p2p_buffer_free(void* ptr);
KB_API int kb_p2p_ipc_handle(void* ptr, void* handle /* 64 bytes */);
KB_API int kb_p2p_ipc_open(const void* handle, void** peer_ptr);
KB_API int kb_p2p_ipc_close(void* peer_ptr);
KB_API int kb_p2p_read_fault(int clear, int* value);
KB_API int kb_p2p_allreduce_f64(void* const* bufs, int rank, int world,
                         size_t buf_bytes, const double* src, double* dst,
                         int64_t n, unsigned epoch, uint64_t timeout_ns,
                         kbStream stream);
KB_API int kb_p2p_allreduce_f32(void* const* bufs, int rank, int world,
                         size_t buf_bytes, const float* src, float* dst,
                         int64_t n, unsigned epoch, uint64_t timeout_ns,
                         kbStream stream);
/* split-K fused form: this rank's `splits` partial tiles [splits][n] (from
 * kb_gemm_splitk_partials_3xtf32) are summed in split order, then across
 * ranks, in one kernel: dst[n] = the full C on every rank.                */
KB_API int kb_p2p_splitk_allreduce_f32(void* const* bufs, int rank, int world,
                                size_t buf_bytes, const float* partials,
                                int splits, float* dst, int64_t n,
                                unsigned epoch, uint64_t timeout_ns,
                                kbStream stream);
/* Fused sharded reductions, one launch each: this rank's partial pass, a
 * fixed-order fold by the CTA that finishes last, and that CTA's exchange
 * of the folded values over the peer buffers (same buffers, epochs and
 * fault word as kb_p2p_allreduce_*; a call takes one epoch).  They replace
 * the three to four launches of partial entry + all-reduce + finish entry
 * of the sharded MSE, Frobenius and BatchNorm (replaced reference entries:
 * mse_entry, candidates/94_MSELoss/v1.py:35-45; fro_entry,
 * candidates/37_FrobeniusNorm_/v1.py:48-58; bn_entry,
 * candidates/33_BatchNorm/v1.py:53-68).  The workspace begins with a
 * 256-byte arrival counter that must be zero before the first call; every
 * call leaves it zero, so one zeroed workspace serves every call of a
 * stream.  On an expired wait the results are NaN and the fault word is
 * set.
 *   kb_mse_sharded_f32      out = sum over ranks of sum (a-b)^2 / sum over
 *                           ranks of n (shards of any size, empty too)
 *   kb_sumsq_sharded_f64    total = sum over ranks of sum x^2; then
 *                           kb_scale_by_inv_norm_f32 on the shard
 *   kb_batchnorm_stats_sharded_f64   stats[2C + 1] = global per-channel
 *                           sums, sums of squares and elements per channel;
 *                           then kb_batchnorm_apply_f32 on the shard      */
KB_API size_t kb_sharded_workspace_size(void);
KB_API int kb_mse_sharded_f32(const float* a, const float* b, float* out, int64_t n,
                              void* workspace, size_t workspace_bytes, void* const* bufs,
                              int rank, int world, size_t buf_bytes, unsigned epoch,
                              uint64_t timeout_ns, kbStream stream);
KB_API int kb_sumsq_sharded_f64(const float* x, double* total, int64_t n, void* workspace,
                                size_t workspace_bytes, void* const* bufs, int rank,
                                int world, size_t buf_bytes, unsigned epoch,
                                uint64_t timeout_ns, kbStream stream);
KB_API size_t kb_batchnorm_sharded_workspace_size(int64_t N, int64_t C, int64_t HW);
KB_API int kb_batchnorm_stats_sharded_f64(const float* x, double* stats, int64_t N,
                                          int64_t C, int64_t HW, void* workspace,
                                          size_t workspace_bytes, void* const* bufs,
                                          int rank, int world, size_t buf_bytes,
                                          unsigned epoch, uint64_t timeout_ns,
                                          kbStream stream);
/* the K-split partial tiles of C = A[M,K] B[K,N] without their reduction:
 * workspace[z][M][N] for z < *splits.                                     */
KB_API size_t kb_gemm_splitk_partials_workspace_size(int64_t M, int64_t N, int64_t K);
KB_API int kb_gemm_splitk_partials_3xtf32(const float* A, const float* B, int64_t M,
                                   int64_t N, int64_t K, void* workspace,
                                   size_t workspace_bytes, int* splits,
                                   kbStream stream);

#ifdef __cplusplus
}
#endif

#endif /* KBB200_H */
