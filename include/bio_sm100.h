/*
 * bio_sm100.h -- C ABI of the B200 (sm_100a) batch-invariant operator library.
 *
 * Every entry point takes plain device pointers, int64 sizes/strides (in
 * ELEMENTS, not bytes), a dtype enum and a cudaStream_t passed as void*.
 * The library never allocates, never frees, keeps no reference to caller
 * memory after the call returns and never synchronises the stream: all work
 * is enqueued asynchronously on `stream`.  Outputs and workspaces are owned by
 * the caller (the Python layer allocates them through PyTorch).
 *
 * Batch invariance contract: for every op, the arithmetic that produces one
 * output row (GEMM), one output vector (row reductions) or one query row
 * (attention) is a function of that row's inputs and of the problem's
 * per-row geometry (N, K, row length, head_dim, dtype) only.  It never depends
 * on M, on the batch count, on the position of the row in the batch or on the
 * number of SMs.
 *
 * Each declaration names the reference interface it replaces
 * (batch_invariant_ops/batch_invariant_ops.py:<line> in the reference
 * project yiannisha/robotics-batch-invariant-ops).
 */
#ifndef BIO_SM100_H_
#define BIO_SM100_H_

#include <stdint.h>

#if defined(__GNUC__)
#define BIO_API __attribute__((visibility("default")))
#else
#define BIO_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (returned by every entry point) ---------------------- */
#define BIO_OK 0
#define BIO_ERR_SHAPE 1       /* inconsistent or unsupported sizes           */
#define BIO_ERR_STRIDE 2      /* stride layout not accepted by this path     */
#define BIO_ERR_ALIGN 3       /* pointer/stride alignment not accepted (TMA) */
#define BIO_ERR_DTYPE 4       /* unsupported dtype combination               */
#define BIO_ERR_LAUNCH 5      /* CUDA launch / attribute error               */
#define BIO_ERR_DRIVER 6      /* driver entry point or tensor map failure    */
#define BIO_ERR_ARG 7         /* invalid argument value (null ptr, flags)    */
#define BIO_ERR_DEVICE 8      /* a device-side check fired (see status word) */

/* ---- device status word bits (set by kernels, read by the host) -------- */
#define BIO_DEV_TIMEOUT 1     /* a bounded mbarrier wait gave up             */
#define BIO_DEV_INDEX 2       /* an index operand was out of range           */

/* ---- dtypes ------------------------------------------------------------ */
#define BIO_F32 0
#define BIO_F16 1
#define BIO_BF16 2

/* ---- library ----------------------------------------------------------- */
BIO_API int bio_abi_version(void);
BIO_API const char* bio_status_string(int status);
/* Number of SMs of `device` (cached).  Replaces get_compute_units()
 * (batch_invariant_ops.py:232-253). */
BIO_API int bio_sm_count(int device, int* out);
/* Device status word: OR of BIO_DEV_* bits raised by kernels since the last
 * clear.  Reading synchronises the device. */
BIO_API int bio_device_status(int device, int* out);
BIO_API int bio_clear_device_status(int device);

/* ---- GEMM / batched GEMM ------------------------------------------------
 * C[b][m][n] = alpha * sum_k A[b][m][k] * B[b][k][n]  (+ bias[n])
 *
 * Batch index b = b1 * batch2 + b2.  Operand X (A or B) of batch b lives at
 *   X.ptr + b1 * X.s1 + (b2 / X.div2) * X.s2
 * so stride-0 broadcast (expanded weights) and grouped-query head sharing
 * (div2 = query heads per KV head) need no copy.  C of batch b lives at
 * c + b1 * c_s1 + b2 * c_s2.
 *
 * A element (m, k) at a_sm*m + a_sk*k; B element (k, n) at b_sk*k + b_sn*n;
 * C element (m, n) at c_sm*m + c_sn*n.
 *
 * fp32 runs on CUDA cores with IEEE fp32 FMA in sequential k order (no TF32).
 * bf16/fp16 run on tcgen05 tensor cores with fp32 accumulation; A must be
 * K-contiguous (a_sk == 1) or M-contiguous (a_sm == 1) and B K-contiguous
 * (b_sk == 1) or N-contiguous (b_sn == 1), with 16-byte aligned pointers and
 * strides (BIO_ERR_ALIGN otherwise; the caller packs with bio_pack_rows).
 * The tile shape and K order are chosen from (n, k, dtype) only: the result
 * of row m never depends on m, on M or on the batch count.  Bias is added in
 * fp32 after the full K reduction, then the sum is rounded to the C dtype.
 *
 * Replaces matmul_kernel_persistent / matmul_persistent
 * (batch_invariant_ops.py:61-139, 271-343) and bmm_kernel_persistent /
 * bmm_persistent (batch_invariant_ops.py:143-229, 346-431). */
#define BIO_GEMM_BIAS_PER_ROW 1 /* flags: bias indexed by m instead of n */

typedef struct bio_gemm_args {
  int32_t dtype;   /* BIO_F32 / BIO_F16 / BIO_BF16: A, B, C and bias dtype */
  int32_t flags;   /* 0 or BIO_GEMM_BIAS_PER_ROW                           */
  int64_t batch1, batch2;
  int64_t m, n, k;
  const void* a;
  int64_t a_sm, a_sk, a_s1, a_s2, a_div2;
  const void* b;
  int64_t b_sk, b_sn, b_s1, b_s2, b_div2;
  void* c;
  int64_t c_sm, c_sn, c_s1, c_s2;
  const void* bias; /* bias + b2 * bias_s2 + (n, or m with BIAS_PER_ROW), or NULL */
  int64_t bias_s2;
  float alpha;      /* 1.0f for plain GEMM   */
  int32_t device;   /* CUDA device ordinal of every pointer */
} bio_gemm_args;

BIO_API int bio_gemm(const bio_gemm_args* args, void* stream);

/* Tile configuration id chosen for (n, k, dtype); exposed so tests can prove
 * that the schedule does not depend on m or the batch count.  Encodes
 * block_m * 1000000 + block_n * 1000 + block_k. */
BIO_API int bio_gemm_tile_config(int64_t n, int64_t k, int32_t dtype);

/* Copy a strided [nb1][nb2][rows][cols] operand into a dense
 * [nb1][nb2][rows][cols_pad] buffer (cols_pad >= cols, zero filled tail).
 * Used to bring odd strides into the 16-byte aligned K-contiguous layout the
 * tensor-core GEMM reads with TMA.  Exact copy: packing never changes a
 * GEMM result.  Replaces the implicit strided tl.load of
 * batch_invariant_ops.py:113-123. */
BIO_API int bio_pack_rows(int32_t dtype, const void* src, int64_t nb1, int64_t nb2,
                  int64_t rows, int64_t cols, int64_t s_b1, int64_t s_b2,
                  int64_t s_row, int64_t s_col, void* dst, int64_t cols_pad,
                  int32_t device, void* stream);

/* ---- row kernels ---------------------------------------------------------
 * The input is a CONTIGUOUS [outer][n][inner] tensor reduced over n.  Row
 * mode (inner == 1) assigns one fixed thread team per row (team size a
 * function of n only) with a fixed fold + xor-shuffle tree; column mode
 * (inner > 1) folds each column sequentially.  Arithmetic in fp32, one
 * rounding to the output dtype. */

/* Softmax / log-softmax over n.  Softmax keeps the reference's edge rules:
 * a row whose maximum is -inf, or whose denominator is 0, produces zeros.
 * Log-softmax requires dtype_out == dtype_in.  Output has the input's shape.
 * Replaces _softmax_kernel / softmax (batch_invariant_ops.py:1075-1145) and
 * _log_softmax_kernel / log_softmax (batch_invariant_ops.py:975-1071). */
BIO_API int bio_softmax(int32_t dtype_in, int32_t dtype_out, const void* x, void* y,
                        int64_t outer, int64_t n, int64_t inner, int32_t log_softmax,
                        int32_t device, void* stream);

#define BIO_REDUCE_MEAN 0
#define BIO_REDUCE_L2NORM 1
/* Mean (sum / n) or Euclidean norm (sqrt of sum of squares) over n; output
 * is [outer][inner].  Replaces mean_kernel / mean_dim
 * (batch_invariant_ops.py:1348-1482) and _vector_norm_kernel /
 * linalg_vector_norm_batch_invariant (batch_invariant_ops.py:1486-1597). */
BIO_API int bio_reduce(int32_t kind, int32_t dtype_in, int32_t dtype_out, const void* x,
                       void* y, int64_t outer, int64_t n, int64_t inner, int32_t device,
                       void* stream);

#ifdef __cplusplus
}
#endif

#endif /* BIO_SM100_H_ */
