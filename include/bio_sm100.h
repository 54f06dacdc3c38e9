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
#define BIO_ERR_SCRATCH 9     /* scratch / workspace too small for the problem */

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
 * fp32 runs on CUDA cores: exact fp64 products summed with fp64 FMA in
 * sequential k order, one rounding to fp32 (no TF32); bio_gemm_f32_exact
 * below is the faster fp32 path.  bf16/fp16 run on tcgen05 tensor cores with
 * fp32 accumulation; A must be K-contiguous (a_sk == 1) or M-contiguous
 * (a_sm == 1) and B K-contiguous (b_sk == 1) or N-contiguous (b_sn == 1),
 * with 16-byte aligned pointers and strides (BIO_ERR_ALIGN otherwise; the
 * caller packs with bio_pack_rows).  Every output element is accumulated in
 * the same fixed sequence (64-wide K blocks in increasing order, four K=16
 * MMAs per block into one fp32 accumulator, one rounding); the output tile,
 * which bio_gemm_tile_for reports, is picked from m, n, the batch count and
 * the SM count and only decides which SM computes which elements, so the
 * result of row m never depends on m, on M or on the batch count.  Bias is
 * added in fp32 after the full K reduction, then the sum is rounded to the C
 * dtype.
 *
 * Replaces matmul_kernel_persistent / matmul_persistent
 * (batch_invariant_ops.py:61-139, 271-343) and bmm_kernel_persistent /
 * bmm_persistent (batch_invariant_ops.py:143-229, 346-431). */
#define BIO_GEMM_BIAS_PER_ROW 1 /* flags: bias indexed by m instead of n */
#define BIO_GEMM_GATE_GELU_TANH 2 /* flags (bio_gemm_swiglu only): GELU-tanh gate */

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

/* bio_gemm followed by a residual add in the epilogue (f16/bf16, one plain
 * 2-D GEMM: batch1 == batch2 == 1, no flags, c_sn == 1): C = round(round(
 * alpha A B + bias) + R), the rounding steps of a linear layer followed by
 * `residual + output`, bit for bit; R is [m, n] with residual_row_stride
 * (>= n) elements between rows and must not overlap C.  Saves the separate
 * add's read and write of the GEMM output and its launch.  No counterpart in the reference (a
 * transformer's residual adds run as stock elementwise ops there). */
BIO_API int bio_gemm_residual(const bio_gemm_args* args, const void* residual,
                              int64_t residual_row_stride, void* stream);

/* Configuration id for (n, k, dtype): the large-M output tile and the K block
 * whose fixed order defines every output element's accumulation.  Encodes
 * block_m * 1000000 + block_n * 1000 + block_k.  The output tile of a given
 * call also depends on m (bio_gemm_tile_for); all tiles run the same
 * per-element sequence, which bio_gemm_tiled lets tests check. */
BIO_API int bio_gemm_tile_config(int64_t n, int64_t k, int32_t dtype);

/* The output tile bio_gemm runs (f16/bf16 tensor-core path) for an m x n
 * GEMM over `batch` independent products on a device with `sms` SMs, with B
 * N-contiguous when b_mn != 0: *tile_m 128 (one CTA) or 256 (CTA pair),
 * *tile_n 32..256.  Pure function, needs no GPU.  BIO_ERR_ARG for a null
 * pointer or a non-positive size.  No counterpart in the reference (its
 * matmul_persistent, batch_invariant_ops.py:294-319, has one tile per
 * dtype). */
BIO_API int bio_gemm_tile_for(int64_t m, int64_t n, int64_t batch, int32_t sms, int32_t b_mn,
                              int32_t* tile_m, int32_t* tile_n);

/* Workspace bytes that bio_gemm_f32_exact needs for these arguments; 0 when
 * that path does not apply (dtype not BIO_F32, K == 0 or K > 65536, empty or
 * invalid shapes). */
BIO_API int64_t bio_gemm_f32_exact_workspace(const bio_gemm_args* args);

/* fp32 GEMM (same arguments and result layout as bio_gemm) on the int8 tensor
 * cores with exact integer slices: every row of A and column of B is scaled
 * by a power of two and cut into four signed digits in [-64, 64], digit products are
 * summed exactly in int32 TMEM accumulators, and the epilogue recombines them
 * in fp64 with alpha and bias, rounding once to fp32.  Each output is within
 * K * 2^-26 * max|A[m,:]| * max|B[:,n]| of the exact sum, and depends on its
 * own A row and on B only (batch invariant).  `workspace`: device memory of
 * at least bio_gemm_f32_exact_workspace(args) bytes, 256-byte aligned
 * (BIO_ERR_SCRATCH if smaller).  Rows/columns holding Inf or NaN give NaN.
 * Replaces the fp32 configuration of matmul_persistent / bmm_persistent
 * (batch_invariant_ops.py:271-431), which accumulates in fp32. */
BIO_API int bio_gemm_f32_exact(const bio_gemm_args* args, void* workspace,
                               int64_t workspace_bytes, void* stream);

/* bio_gemm with an explicit output tile for the tensor-core path (f16/bf16):
 * tile_m 128 (one CTA) or 256 (CTA pair), tile_n 32/64/96/128/256 (pair: 128
 * or 256; an N-contiguous B needs tile_n 64, 128 or 256).  The per-element arithmetic of
 * every tile is the same sequence (64-wide K blocks in increasing order, four
 * K=16 MMAs per block into an fp32 accumulator, one rounding), so all tiles
 * must produce identical bits; tests use this entry to check exactly that.
 * BIO_ERR_ARG for an unsupported tile.  No counterpart in the reference
 * (its matmul_persistent, batch_invariant_ops.py:271-343, has one fixed
 * configuration per dtype). */
BIO_API int bio_gemm_tiled(const bio_gemm_args* args, int32_t tile_m, int32_t tile_n,
                           void* stream);

/* Segmented GEMM (f16/bf16 tensor-core path): segment s = 0..batch1-1 owns
 * rows [seg[s], seg[s+1]) of A and C and multiplies them by B batch s
 * (b + s * b_s1).  A and C are single matrices of m rows (a_s1 == c_s1 == 0,
 * A K-contiguous), batch2 == 1, 1 <= batch1 <= 1024, k >= 1, no flags.  seg
 * is a device int32 array [batch1 + 1] read on the device (no host sync);
 * segments whose offsets are decreasing or outside [0, m] are skipped and
 * raise BIO_DEV_INDEX; C rows outside every segment are not written.  Row r
 * of a segment gets exactly the bits bio_gemm gives that row against the
 * same B.  No counterpart in the reference (its experts run as one dense
 * bmm over all tokens, moe.py:67-79). */
BIO_API int bio_gemm_segmented(const bio_gemm_args* args, const int32_t* seg, void* stream);

/* Fused SwiGLU expert GEMM (f16/bf16): C = silu(A·gateᵀ) * (A·upᵀ) with the
 * roundings of two bio_gemm calls followed by bio_silu_mul (gate and up
 * rounded to the dtype, silu rounded, product rounded), bit for bit.  `args`
 * describes the gate GEMM (b = gate weights, n = output columns, no bias;
 * flags 0, or BIO_GEMM_GATE_GELU_TANH for GeGLU: the gate activation is
 * 0.5 g (1 + tanh(sqrt(2/pi) (g + 0.044715 g^3))) in fp32, the rounding steps
 * of F.gelu(gate, approximate="tanh") * up); `up` has the same dims and
 * strides as b.  One CTA pair computes a
 * 256-row tile of gate and up for 128 output columns in one 256-wide
 * accumulator (the leader loads gate rows, its peer the same up rows), so A
 * is read once and the gate/up outputs never reach HBM.  `seg` (optional)
 * selects the segmented mode of bio_gemm_segmented.  No counterpart in the
 * reference (moe.py:75-79 runs gate, up and silu*up as separate ops). */
BIO_API int bio_gemm_swiglu(const bio_gemm_args* args, const void* up, const int32_t* seg,
                            void* stream);

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
 * Log-softmax requires dtype_out == dtype_in or BIO_F32 (half_to_float).
 * Output has the input's shape.
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

#define BIO_NORM_LAYER 0
#define BIO_NORM_RMS 1
/* Fused normalisation over the last n elements of each of `rows` rows (row r
 * of x at x + r * x_row_stride, of y at y + r * y_row_stride, elements
 * contiguous).  BIO_NORM_LAYER: y = (x - mean) * rsqrt(var + eps) * w + b with
 * the biased variance; BIO_NORM_RMS: y = x * rsqrt(mean(x^2) + eps) * w (bias
 * must be NULL).  weight / bias [n] in w_dtype, or NULL (1 / 0).  fp32
 * arithmetic with a fixed team per row (32 / 256 / 1024 threads by n) and a
 * fixed fold + xor-shuffle tree, one rounding to dtype; mean_out / rstd_out
 * (fp32 [rows], optional) receive the row statistics (mean is 0 for RMS).
 * A row's bits depend on that row and n only.  No counterpart in the
 * reference, which leaves layer norms to stock torch and builds RMSNorm from
 * mean_dim (batch_invariant_ops.py:1395-1482); these replace
 * aten::native_layer_norm and aten::_fused_rms_norm under the mode. */
BIO_API int bio_norm(int32_t kind, int32_t dtype, int32_t w_dtype, const void* x,
                     const void* weight, const void* bias, void* y, float* mean_out,
                     float* rstd_out, int64_t rows, int64_t n, int64_t x_row_stride,
                     int64_t y_row_stride, float eps, int32_t device, void* stream);

/* ---- convolution lowering -------------------------------------------------
 * Geometry of an N-d convolution, N <= 3, in NC[D][H]W layout; unused
 * leading spatial dims have in = kernel = stride = dilation = out = 1 and
 * padding 0.  For transposed convolution `in` is the input spatial size and
 * `kernel` equals the stride (non-overlapping). */
typedef struct bio_conv_geom {
  int64_t batch, channels, groups;
  int64_t in[3], kernel[3], stride[3], padding[3], dilation[3], out[3];
} bio_conv_geom;

/* Gather receptive fields of CONTIGUOUS x [B][C][in...] into patches
 * [B][G][L][kpad] (L = prod(out), K = C/G * prod(kernel) <= kpad, zero tail
 * and zero padding), K index = (c, kd, kh, kw) row-major like the weight.
 * The caller then runs one bio_gemm per (sample, group).  Replaces the
 * F.unfold / as_strided im2col of conv1d/2d/3d_batch_invariant
 * (batch_invariant_ops.py:566-595, 640-667, 731-760). */
BIO_API int bio_im2col(int32_t dtype, const void* x, const bio_conv_geom* geom, void* patches,
                       int64_t kpad, int32_t device, void* stream);

/* Depthwise 1-D convolution (groups == C == O, one tap row per channel):
 * y[b,c,l] = sum_k x[b,c,l*stride-pad+k*dil] * w[c,k] (+ bias[c]), fp32
 * accumulation in tap order.  x [B][C][lin], w [C][ksize], y [B][C][lout],
 * all contiguous.  Replaces depthwise_conv1d_kernel
 * (batch_invariant_ops.py:435-494, launch :531-564). */
BIO_API int bio_depthwise_conv1d(int32_t dtype, const void* x, const void* w, const void* bias,
                                 void* y, int64_t batch, int64_t channels, int64_t lin,
                                 int64_t lout, int32_t ksize, int32_t stride, int32_t padding,
                                 int32_t dilation, int32_t device, void* stream);

/* Layout transform of a non-overlapping transposed convolution: src is the
 * per-(sample, group) GEMM result [B][G][Og*kvol][prod(in)], dst is
 * [B][G*Og][in0*k0][in1*k1][in2*k2]; dst = src (+ bias[channel]).  Replaces
 * the bias add and pixel-shuffle permute of conv_transpose2d/3d_batch_invariant
 * (batch_invariant_ops.py:846-861, 926-941). */
/* Non-overlapping transposed convolution (stride == kernel, no padding,
 * dilation 1; f16/bf16) in one GEMM whose epilogue writes the final layout:
 * per (sample, group) C[m = input position, n = (o, kernel offset)] =
 * sum_c x[b, g*Cg + c, m] * w[g*Cg + c, n] with fixed K order, rounded, plus
 * bias[g*Og + o] (added after rounding, as the reference's output + bias),
 * stored at y[b, g*Og + o, s*k + t] (runs of k2 outputs as one vector).  x
 * [B][C][in...], w [C][Og][k...], y [B][G*Og][in*k...], all contiguous;
 * prod(in) and Og*prod(k) multiples of 8 (BIO_ERR_ALIGN otherwise; the
 * caller then uses bio_gemm + bio_conv_transpose_scatter).  Same bits as
 * that two-step path.  Replaces conv_transpose2d/3d_batch_invariant's bmm,
 * bias add and permute (batch_invariant_ops.py:783-941). */
BIO_API int bio_conv_transpose(int32_t dtype, const void* x, const void* w, const void* bias,
                               void* y, const bio_conv_geom* geom, int64_t out_channels_per_group,
                               int32_t device, void* stream);

BIO_API int bio_conv_transpose_scatter(int32_t dtype, const void* src, const void* bias,
                                       void* dst, const bio_conv_geom* geom,
                                       int64_t out_channels_per_group, int32_t device,
                                       void* stream);

/* ---- attention ------------------------------------------------------------
 * Fused attention with an online softmax in fp32; a row's bits do not depend
 * on the other rows, sequences or heads of the launch.  bf16/fp16 run on
 * tcgen05 (128 query rows per CTA, keys in fixed blocks of 128, S and O in
 * TMEM, one softmax thread per query row); base pointers and token/head
 * strides must then be 16-byte aligned (BIO_ERR_ALIGN otherwise).  fp32 runs
 * on CUDA cores (one warp per query row, keys in fixed blocks of 32).  Tensors
 * are [batch][head][token][dim] through element strides (dim contiguous); KV
 * head of query head h is h / (heads / kv_heads).  Fully masked rows and empty
 * KV ranges produce zeros.  d, dv <= 256. */
#define BIO_MASK_NONE 0
#define BIO_MASK_BOOL 1 /* uint8/bool keep-mask: 0 drops the key           */
#define BIO_MASK_ADD 2  /* additive float mask in mask_dtype                */

#define BIO_CAUSAL_NONE 0
#define BIO_CAUSAL_TOP_LEFT 1     /* key j visible iff j <= i                  */
#define BIO_CAUSAL_BOTTOM_RIGHT 2 /* key j visible iff j <= i + (lk - lq)     */
#define BIO_CAUSAL_EQUAL 3        /* top-left; varlen requires lq == lk       */

typedef struct bio_attn_args {
  int32_t dtype;
  int32_t device;
  const void* q;
  const void* k;
  const void* v;
  void* o;
  int64_t q_sb, q_sh, q_st;
  int64_t k_sb, k_sh, k_st;
  int64_t v_sb, v_sh, v_st;
  int64_t o_sb, o_sh, o_st;
  int64_t batch, heads, kv_heads;
  int64_t lq, lk;      /* varlen: total packed query / key tokens          */
  int32_t d, dv;
  float scale;
  int32_t causal;      /* BIO_CAUSAL_*                                      */
  int32_t mask_kind;   /* BIO_MASK_* (dense only)                           */
  int32_t mask_dtype;  /* BIO_F32/F16/BF16 for BIO_MASK_ADD                 */
  const void* mask;    /* element (b, h, i, j) at b*m_sb + h*m_sh + i*m_sq + j*m_sk */
  int64_t m_sb, m_sh, m_sq, m_sk;
  const void* cu_q;    /* varlen: [nseq + 1] offsets (int32 or int64)      */
  const void* cu_k;
  int32_t cu_is64;
  int64_t nseq;
  void* workspace;     /* varlen, bf16/fp16: int32 [2 * nseq + 1] scratch  */
} bio_attn_args;

/* Dense SDPA over [batch][heads][lq|lk][d|dv].  Replaces
 * scaled_dot_product_attention_batch_invariant (batch_invariant_ops.py:1148-1213). */
BIO_API int bio_attention(const bio_attn_args* args, void* stream);

/* Sequence-packed attention: q [lq tokens][heads][d], k/v [lk tokens][kv_heads]
 * (batch strides ignored); sequence s covers query tokens [cu_q[s], cu_q[s+1])
 * and keys [cu_k[s], cu_k[s+1]); query tokens outside every sequence are
 * written as zeros (bf16/fp16: the caller pre-zeroes o and passes an int32
 * [2 * nseq + 1] workspace).  Offsets are read on the device (no host sync);
 * invalid offsets raise BIO_DEV_INDEX and leave the affected rows zero.  Replaces
 * varlen_scaled_dot_product_attention_batch_invariant
 * (batch_invariant_ops.py:1216-1344). */
BIO_API int bio_attention_varlen(const bio_attn_args* args, void* stream);

/* ---- mixture of experts ---------------------------------------------------
 * The expert GEMMs themselves run through bio_gemm (one fixed-schedule GEMM
 * per expert, tokens broadcast with a stride-0 batch). */

/* act[i] = silu(gate[i]) * up[i] over n contiguous elements, silu rounded to
 * the dtype before the product (the reference's F.silu(gate) * up,
 * batch_invariant_ops/moe.py:79). */
BIO_API int bio_silu_mul(int32_t dtype, const void* gate, const void* up, void* out, int64_t n,
                         int32_t device, void* stream);

/* out[t, :] = sum_{j=0..top_k-1} (left to right) expert_out[sel[t,j], t, :] *
 * w[t, j], each product and partial sum rounded to dtype.  expert_out
 * [experts][tokens][hidden], w [tokens][top_k] in w_dtype, sel int64
 * [tokens][top_k], out [tokens][hidden], all contiguous.  Out-of-range expert
 * ids raise BIO_DEV_INDEX and zero the row.  Replaces the gather / weight /
 * route-sum chain of deterministic_token_choice_moe (moe.py:67-92). */
BIO_API int bio_moe_route_sum(int32_t dtype, const void* expert_out, int32_t w_dtype,
                              const void* routing_weights, const int64_t* selected_experts,
                              void* out, int64_t experts, int64_t tokens, int64_t top_k,
                              int64_t hidden, int32_t device, void* stream);

/* Sparse MoE path: the same outputs as the dense path above, bit for bit,
 * with each expert evaluated only on the tokens routed to it.
 *
 * bio_moe_plan sorts the slots (t, j) of selected_experts [tokens][top_k]
 * by expert, stably (slot order within an expert), into an int32 workspace
 * of at least bio_moe_plan_workspace(...) bytes laid out as
 *   seg[experts + 1]       rows of expert e are [seg[e], seg[e+1])
 *   slot_row[tokens*top_k] sorted row of slot t*top_k + j, -1 if invalid
 *   row_token[tokens*top_k] token of sorted row r (r < seg[experts])
 * followed by scratch.  Invalid expert ids raise BIO_DEV_INDEX and their
 * slots get no row.  experts <= 1024.  Counting sort without atomic
 * positions: the plan depends only on selected_experts.
 *
 * bio_moe_gather_rows writes x_sorted[r, :] = x[row_token[r], :] for the
 * routed rows.  The expert GEMMs then run through bio_gemm_segmented with
 * `seg` (segment e = expert e), followed by bio_silu_mul, and
 * bio_moe_route_sum_sorted adds each token's routes left to right with the
 * rounding of bio_moe_route_sum, reading route j from row slot_row[t*top_k+j].
 * Every expert output row is computed by the same per-row arithmetic as in
 * the dense path (the GEMM result of a row never depends on the other rows),
 * so the two paths agree exactly.  No counterpart in the reference, which
 * evaluates every expert on every token (moe.py:67-92). */
BIO_API int64_t bio_moe_plan_workspace(int64_t experts, int64_t tokens, int64_t top_k);
BIO_API int bio_moe_plan(const int64_t* selected_experts, int64_t experts, int64_t tokens,
                         int64_t top_k, void* workspace, int64_t workspace_bytes,
                         int32_t device, void* stream);
BIO_API int bio_moe_gather_rows(int32_t dtype, const void* x, int64_t hidden, const void* plan,
                                int64_t experts, int64_t tokens, int64_t top_k,
                                void* x_sorted, int32_t device, void* stream);
BIO_API int bio_moe_route_sum_sorted(int32_t dtype, const void* y_sorted, int32_t w_dtype,
                                     const void* routing_weights, const void* plan, void* out,
                                     int64_t experts, int64_t tokens, int64_t top_k,
                                     int64_t hidden, int32_t device, void* stream);

/* ---- failure detection self-test -----------------------------------------
 * Runs the bounded-wait exit path of the pipelined kernels on purpose: one
 * CTA with a TMA producer and a consumer on a two-stage ring (the same
 * mbar_wait / mbar_wait_drain the GEMM and attention kernels use), in which
 * the consumer never releases a stage and then waits on a barrier nothing
 * arrives at.  Both waits give up after `timeout_ns` (1 us .. 2 s); the
 * kernel raises BIO_DEV_TIMEOUT in the status word, drains its two copies
 * (src: 8192 bytes, 16-byte aligned, device memory), frees its tensor
 * memory and returns, so the context stays usable.  `out` (device int32[4])
 * receives: producer gave up, consumer gave up, stage 0 landed intact, drain
 * completed (1 each when the path works).  No counterpart in the reference,
 * whose MoE index check is a trapping device assert (moe.py:67-74). */
BIO_API int bio_selftest_bounded_wait(const void* src, int32_t* out, int64_t timeout_ns,
                                      int32_t device, void* stream);

/* ---- convolution that allocates nothing ---------------------------------
 * No counterpart in the reference (its convolutions allocate their im2col
 * buffers through PyTorch on every call).  This entry point is for callers
 * that cannot allocate device memory while they run: real-time robot control
 * loops that reserve all memory up front (a cudaMalloc can block and
 * synchronise the device mid-cycle), C/C++ hosts without a caching
 * allocator, and code running inside another runtime's stream capture where
 * allocation calls are not permitted.
 *
 * Same bits as the regular path (bio_im2col, then bio_gemm for f16/bf16 or
 * bio_gemm_f32_exact for fp32, K <= 65536; regular N-d convolution, any
 * groups, stride, padding, dilation; bias per output channel): the patch
 * matrix, a zero-padded copy of the weight when its rows are not 16-byte
 * aligned, and (fp32) the exact GEMM's digit workspace are kept in ONE
 * file-scope device array of BIO_NOALLOC_SCRATCH_BYTES (32 MiB) that every
 * GPU which loads the library holds until the process exits.
 * The caller passes contiguous x [B][C][in...], weight [O][C/G][kernel...],
 * bias [O] or NULL and y [B][O][out...].  geom->out must be the extent the
 * geometry implies, (in + 2*pad - dil*(kernel-1) - 1) / stride + 1 per dim
 * (BIO_ERR_SHAPE otherwise).  Problems needing more scratch
 * (B*G*prod(out)*roundup8(C/G*prod(kernel))*dtype bytes, plus the padded
 * weight or the fp32 workspace) return BIO_ERR_SCRATCH before anything is
 * launched; every size is checked against overflow before it is compared.
 * The first call on a device looks up the array's device address (module
 * load) and caches it; make that first call before any stream capture.  The
 * cached address belongs to the device's primary context: after
 * cudaDeviceReset the process must not call this entry point again.  Every
 * call shares the array, so calls that may overlap on the GPU (different
 * streams, or different host threads on one device) race on it: serialise
 * them.  Nothing in the array needs to start at zero (every byte used is
 * written first).  Never calls cudaMalloc, cudaFree or an allocating
 * library routine. */
#define BIO_NOALLOC_SCRATCH_BYTES (32ull << 20)
BIO_API int bio_conv_nd_noalloc(int32_t dtype, const void* x, const void* weight,
                                const void* bias, void* y, const bio_conv_geom* geom,
                                int64_t out_channels, int32_t device, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* BIO_SM100_H_ */
