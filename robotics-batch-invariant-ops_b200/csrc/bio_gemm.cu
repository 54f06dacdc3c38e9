// Batch-invariant GEMM / batched GEMM for sm_100a.
//
// bf16 / fp16: persistent, warp-specialised tcgen05 kernel.
//   warp 0      TMA producer: A tile 128x64 and B tile BNx64 per stage,
//               128-byte swizzle, mbarrier ring of STAGES stages.
//   warp 1      MMA issuer: 4 x tcgen05.mma (M=128, N=BN, K=16) per stage,
//               fp32 accumulators in TMEM, double buffered (2 x BN columns).
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns, alpha, bias (fp32),
//               round to the output dtype, store.
// The K loop always runs k-block 0..K/64-1, four MMA-K 16 steps per block in
// order, into one fp32 TMEM accumulator per output element, in every kernel
// variant; the output tile (CTA pair 256 x 128/256, single CTA 128 x
// 32..256, chosen from M, N, the batch count and the SM count by pick_tile)
// only decides which SM computes which elements.  So the bits of output row
// m depend on row m of A and on B only (never on M, the batch count or the
// tile a row lands in); tests run every tile on the same inputs and require
// identical bits.  No split-K, no stream-K.
//
// fp32 (bio_gemm): CUDA-core GEMM (128x128x8 tiles, 8x8 outputs per thread);
// exact fp64 products accumulated with DFMA in sequential k order from k = 0,
// one final rounding to fp32.  (The Python layer sends fp32 with K <= 65536 to
// the exact-slice int8 tensor-core GEMM of bio_gemm_exact.cu instead.)
//
// Reference: matmul_kernel_persistent / bmm_kernel_persistent in
// batch_invariant_ops/batch_invariant_ops.py:61-229 and their launchers
// :271-431 (tile table :294-319, input_precision="ieee" :340).
#include "bio_gemm_tc.cuh"

namespace bio {

// ---------------------------------------------------------------------------
// fp32 CUDA-core GEMM with fp64 accumulation.
//
// Products of two fp32 values are exact in fp64 and the running sum is kept in
// fp64 (DFMA, sequential k from 0), so the only fp32 rounding is the final
// store: results sit within ~1 ulp of the exact dot product, far inside the
// 1e-5 normwise fp32 bar, including the ill-conditioned linspace inputs of
// the fp32 batch-invariance check where any fp32 accumulation order loses
// ~5e-4.  Operands are converted to fp64 once when staged into shared memory.
// ---------------------------------------------------------------------------
struct F32GemmParams {
  int64_t m, n, k;
  int64_t batch2, nbatch;
  const float* a;
  int64_t a_sm, a_sk, a_s1, a_s2, a_div2;
  const float* b;
  int64_t b_sk, b_sn, b_s1, b_s2, b_div2;
  float* c;
  int64_t c_sm, c_sn, c_s1, c_s2;
  const float* bias;
  int64_t bias_s2;
  int bias_per_row;
  float alpha;
  int a_kfast, b_nfast;
};

constexpr int kF32BM = 128, kF32BN = 128, kF32BK = 8;

__global__ void __launch_bounds__(256) gemm_f32_kernel(const F32GemmParams p) {
  __shared__ __align__(16) double As[2][kF32BK][kF32BM];
  __shared__ __align__(16) double Bs[2][kF32BK][kF32BN];
  const int tid = threadIdx.x;
  const int tm = tid >> 4, tn = tid & 15;
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * kF32BM;
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * kF32BN;

  for (int64_t bi = blockIdx.z; bi < p.nbatch; bi += gridDim.z) {
    const int64_t b1 = bi / p.batch2, b2 = bi - b1 * p.batch2;
    const float* A = p.a + b1 * p.a_s1 + (b2 / p.a_div2) * p.a_s2;
    const float* B = p.b + b1 * p.b_s1 + (b2 / p.b_div2) * p.b_s2;
    float* C = p.c + b1 * p.c_s1 + b2 * p.c_s2;

    double acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] = 0.0;

    float ra[4], rb[4];
    auto load_tile = [&](int64_t k0) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int idx = tid + i * 256;
        int mm, kk;
        if (p.a_kfast) {
          kk = idx & 7;
          mm = idx >> 3;
        } else {
          mm = idx & 127;
          kk = idx >> 7;
        }
        const int64_t gm = m0 + mm, gk = k0 + kk;
        ra[i] = (gm < p.m && gk < p.k) ? A[gm * p.a_sm + gk * p.a_sk] : 0.f;
        int nn, kb;
        if (p.b_nfast) {
          nn = idx & 127;
          kb = idx >> 7;
        } else {
          kb = idx & 7;
          nn = idx >> 3;
        }
        const int64_t gn = n0 + nn, gkb = k0 + kb;
        rb[i] = (gn < p.n && gkb < p.k) ? B[gkb * p.b_sk + gn * p.b_sn] : 0.f;
      }
    };
    auto store_tile = [&](int buf) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int idx = tid + i * 256;
        if (p.a_kfast)
          As[buf][idx & 7][idx >> 3] = static_cast<double>(ra[i]);
        else
          As[buf][idx >> 7][idx & 127] = static_cast<double>(ra[i]);
        if (p.b_nfast)
          Bs[buf][idx >> 7][idx & 127] = static_cast<double>(rb[i]);
        else
          Bs[buf][idx & 7][idx >> 3] = static_cast<double>(rb[i]);
      }
    };

    const int64_t k_tiles = (p.k + kF32BK - 1) / kF32BK;
    load_tile(0);
    store_tile(0);
    __syncthreads();
    for (int64_t kt = 0; kt < k_tiles; ++kt) {
      const int buf = static_cast<int>(kt & 1);
      if (kt + 1 < k_tiles) load_tile((kt + 1) * kF32BK);
#pragma unroll
      for (int kk = 0; kk < kF32BK; ++kk) {
        double a[8], b[8];
        const double2* pa0 = reinterpret_cast<const double2*>(&As[buf][kk][tm * 4]);
        const double2* pa1 = reinterpret_cast<const double2*>(&As[buf][kk][64 + tm * 4]);
        const double2* pb0 = reinterpret_cast<const double2*>(&Bs[buf][kk][tn * 4]);
        const double2* pb1 = reinterpret_cast<const double2*>(&Bs[buf][kk][64 + tn * 4]);
        double2 t;
        t = pa0[0]; a[0] = t.x; a[1] = t.y;
        t = pa0[1]; a[2] = t.x; a[3] = t.y;
        t = pa1[0]; a[4] = t.x; a[5] = t.y;
        t = pa1[1]; a[6] = t.x; a[7] = t.y;
        t = pb0[0]; b[0] = t.x; b[1] = t.y;
        t = pb0[1]; b[2] = t.x; b[3] = t.y;
        t = pb1[0]; b[4] = t.x; b[5] = t.y;
        t = pb1[1]; b[6] = t.x; b[7] = t.y;
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[i][j] = fma(a[i], b[j], acc[i][j]);
      }
      if (kt + 1 < k_tiles) store_tile(buf ^ 1);
      __syncthreads();
    }

#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t gm = m0 + (i < 4 ? tm * 4 + i : 64 + tm * 4 + (i - 4));
      if (gm >= p.m) continue;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int64_t gn = n0 + (j < 4 ? tn * 4 + j : 64 + tn * 4 + (j - 4));
        if (gn >= p.n) continue;
        double v = acc[i][j] * static_cast<double>(p.alpha);
        if (p.bias != nullptr)
          v += static_cast<double>(p.bias[b2 * p.bias_s2 + (p.bias_per_row ? gm : gn)]);
        C[gm * p.c_sm + gn * p.c_sn] = static_cast<float>(v);
      }
    }
    __syncthreads();
  }
}

// C = alpha * 0 + bias (K == 0): an empty reduction.
template <typename T>
__global__ void gemm_fill_kernel(T* c, int64_t m, int64_t n, int64_t nbatch, int64_t batch2,
                                 int64_t c_sm, int64_t c_sn, int64_t c_s1, int64_t c_s2,
                                 const T* bias, int64_t bias_s2, int bias_per_row) {
  const int64_t total = nbatch * m * n;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t col = i % n;
    const int64_t row = (i / n) % m;
    const int64_t bi = i / (n * m);
    const int64_t b1 = bi / batch2, b2 = bi - b1 * batch2;
    const float v =
        bias != nullptr ? to_f32(bias[b2 * bias_s2 + (bias_per_row ? row : col)]) : 0.f;
    c[b1 * c_s1 + b2 * c_s2 + row * c_sm + col * c_sn] = from_f32<T>(v);
  }
}

template <typename T>
__global__ void pack_rows_kernel(const T* __restrict__ src, int64_t nb2, int64_t rows,
                                 int64_t cols, int64_t s_b1, int64_t s_b2, int64_t s_row,
                                 int64_t s_col, T* __restrict__ dst, int64_t cols_pad,
                                 int64_t total) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t col = i % cols_pad;
    const int64_t rest = i / cols_pad;
    const int64_t row = rest % rows;
    const int64_t b = rest / rows;
    const int64_t b1 = b / nb2, b2 = b - b1 * nb2;
    dst[i] = col < cols ? src[b1 * s_b1 + b2 * s_b2 + row * s_row + col * s_col]
                        : from_f32<T>(0.f);
  }
}
}  // namespace bio

using namespace bio_gemm_tc;

namespace {

int launch_f32(const bio_gemm_args* a, cudaStream_t stream) {
  bio::F32GemmParams p;
  p.m = a->m;
  p.n = a->n;
  p.k = a->k;
  p.batch2 = a->batch2;
  p.nbatch = a->batch1 * a->batch2;
  p.a = static_cast<const float*>(a->a);
  p.a_sm = a->a_sm;
  p.a_sk = a->a_sk;
  p.a_s1 = a->a_s1;
  p.a_s2 = a->a_s2;
  p.a_div2 = a->a_div2;
  p.b = static_cast<const float*>(a->b);
  p.b_sk = a->b_sk;
  p.b_sn = a->b_sn;
  p.b_s1 = a->b_s1;
  p.b_s2 = a->b_s2;
  p.b_div2 = a->b_div2;
  p.c = static_cast<float*>(a->c);
  p.c_sm = a->c_sm;
  p.c_sn = a->c_sn;
  p.c_s1 = a->c_s1;
  p.c_s2 = a->c_s2;
  p.bias = static_cast<const float*>(a->bias);
  p.bias_s2 = a->bias_s2;
  p.bias_per_row = (a->flags & BIO_GEMM_BIAS_PER_ROW) ? 1 : 0;
  p.alpha = a->alpha;
  p.a_kfast = (a->a_sk == 1) ? 1 : 0;
  p.b_nfast = (a->b_sn == 1) ? 1 : 0;
  const int64_t gx = (a->n + bio::kF32BN - 1) / bio::kF32BN;
  const int64_t gy = (a->m + bio::kF32BM - 1) / bio::kF32BM;
  if (gx > 2147483647 || gy > 65535) return BIO_ERR_SHAPE;
  const int64_t nb = p.nbatch;
  const unsigned gz = static_cast<unsigned>(nb < 65535 ? nb : 65535);
  dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(gy), gz);
  bio::gemm_f32_kernel<<<grid, 256, 0, stream>>>(p);
  return bio_host::launch_status(cudaGetLastError());
}

template <typename T>
int launch_fill(const bio_gemm_args* a, cudaStream_t stream) {
  const int64_t total = a->batch1 * a->batch2 * a->m * a->n;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 65536) blocks = 65536;
  bio::gemm_fill_kernel<T><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
      static_cast<T*>(a->c), a->m, a->n, a->batch1 * a->batch2, a->batch2, a->c_sm, a->c_sn,
      a->c_s1, a->c_s2, static_cast<const T*>(a->bias), a->bias_s2,
      (a->flags & BIO_GEMM_BIAS_PER_ROW) ? 1 : 0);
  return bio_host::launch_status(cudaGetLastError());
}

}  // namespace


extern "C" {

int bio_gemm_tile_config(int64_t n, int64_t k, int32_t dtype) {
  if (dtype == BIO_F32) return bio::kF32BM * 1000000 + bio::kF32BN * 1000 + bio::kF32BK;
  (void)k;
  const TileChoice tc = reported_tile(n);
  return (tc.pair ? 256 : kBM) * 1000000 + tc.bn * 1000 + kBK;
}

int bio_gemm_tile_for(int64_t m, int64_t n, int64_t batch, int32_t sms, int32_t b_mn,
                      int32_t* tile_m, int32_t* tile_n) {
  if (tile_m == nullptr || tile_n == nullptr || m < 1 || n < 1 || batch < 1 || sms < 1)
    return BIO_ERR_ARG;
  const TileChoice tc = run_tile(m, n, batch, sms, b_mn != 0);
  *tile_m = tc.pair ? 256 : kBM;
  *tile_n = tc.bn;
  return BIO_OK;
}

}  // extern "C"

namespace {

// Shared body of bio_gemm / bio_gemm_tiled; `forced` (when non-null) replaces
// the library's tile choice for the tensor-core path.
int gemm_impl(const bio_gemm_args* a, const TileChoice* forced, void* stream_v,
              const EpiResidual* res = nullptr) {
  if (a == nullptr) return BIO_ERR_ARG;
  if ((a->flags & ~BIO_GEMM_BIAS_PER_ROW) != 0) return BIO_ERR_ARG;
  if (a->m < 0 || a->n < 0 || a->k < 0 || a->batch1 < 0 || a->batch2 < 1) return BIO_ERR_SHAPE;
  if (a->a_div2 < 1 || a->b_div2 < 1) return BIO_ERR_ARG;
  if (a->dtype != BIO_F32 && a->dtype != BIO_F16 && a->dtype != BIO_BF16) return BIO_ERR_DTYPE;
  const int64_t batch = a->batch1 * a->batch2;
  if (batch == 0 || a->m == 0 || a->n == 0) return BIO_OK;
  if (a->c == nullptr) return BIO_ERR_ARG;
  int st = bio_host::ensure_device(a->device);
  if (st != BIO_OK) return st;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);

  if (a->k == 0) {
    switch (a->dtype) {
      case BIO_F32: return launch_fill<float>(a, stream);
      case BIO_F16: return launch_fill<__half>(a, stream);
      default: return launch_fill<__nv_bfloat16>(a, stream);
    }
  }
  if (a->a == nullptr || a->b == nullptr) return BIO_ERR_ARG;
  if (a->dtype == BIO_F32) return launch_f32(a, stream);

  // Tensor-core path: TMA needs 16-byte aligned bases and strides, K-contiguous A
  // and K- or N-contiguous B; int32 tile coordinates.
  if (a->m > 2147483647 || a->n > 2147483647 || a->k > 2147483647) return BIO_ERR_SHAPE;
  if (a->batch1 > 2147483647 || a->batch2 > 2147483647) return BIO_ERR_SHAPE;
  if (!aligned16(a->a) || !aligned16(a->b)) return BIO_ERR_ALIGN;
  bool a_mn;
  if (a->a_sk == 1) {
    a_mn = false;
  } else if (a->a_sm == 1) {
    a_mn = true;
  } else {
    return BIO_ERR_STRIDE;
  }
  bool b_mn;
  if (a->b_sk == 1) {
    b_mn = false;
  } else if (a->b_sn == 1) {
    b_mn = true;
  } else {
    return BIO_ERR_STRIDE;
  }
  TileChoice tc = forced != nullptr
                     ? *forced
                     : run_tile(a->m, a->n, a->batch1 * a->batch2, bio_host::sm_count(a->device),
                                b_mn);
  if (!tile_supported(tc)) return BIO_ERR_ARG;
  // An N-contiguous B is staged in 64-column swizzle atoms: tiles narrower
  // than one atom are not built for it.
  if (b_mn && !tc.pair && (tc.bn < 64 || tc.bn == 96)) return BIO_ERR_ARG;
  if (a->dtype == BIO_BF16)
    return dispatch_tc<__nv_bfloat16>(a, tc, stream, a_mn, b_mn, nullptr, nullptr, nullptr, res);
  return dispatch_tc<__half>(a, tc, stream, a_mn, b_mn, nullptr, nullptr, nullptr, res);
}

template <typename T>
int dispatch_swiglu(const bio_gemm_args* a, const int* seg, const void* up, cudaStream_t stream,
                    bool a_mn, bool b_mn) {
  return dispatch_tc<T>(a, TileChoice{true, 256}, stream, a_mn, b_mn, seg, nullptr, up);
}

// Shared body of bio_gemm_segmented (seg != null) and bio_gemm_swiglu (up !=
// null; seg optional).
int grouped_impl(const bio_gemm_args* a, const int32_t* seg, const void* up, void* stream_v) {
  if (a == nullptr) return BIO_ERR_ARG;
  // the only flag of the grouped modes: GELU-tanh instead of silu (gated only)
  const int32_t allowed = up != nullptr ? BIO_GEMM_GATE_GELU_TANH : 0;
  if ((a->flags & ~allowed) != 0 || a->a_div2 < 1 || a->b_div2 < 1) return BIO_ERR_ARG;
  if (up != nullptr && a->bias != nullptr) return BIO_ERR_ARG;
  if (a->dtype != BIO_F16 && a->dtype != BIO_BF16) return BIO_ERR_DTYPE;
  if (a->m < 0 || a->n < 0 || a->k < 1 || a->batch1 < 1 || a->batch2 < 1) return BIO_ERR_SHAPE;
  if (a->m > 2147483647 || a->n > 2147483647 || a->k > 2147483647) return BIO_ERR_SHAPE;
  if (a->batch1 > 2147483647 || a->batch2 > 2147483647) return BIO_ERR_SHAPE;
  if (seg != nullptr) {
    if (a->batch2 != 1 || a->batch1 > bio::kMaxSegs) return BIO_ERR_SHAPE;
    // one A and one C matrix whose rows the segments share; A rows start at
    // arbitrary offsets, so A must be K-contiguous (a row index is never the
    // innermost tensor-map coordinate)
    if (a->a_s1 != 0 || a->c_s1 != 0 || a->a_sk != 1) return BIO_ERR_STRIDE;
  }
  if (a->m == 0 || a->n == 0) return BIO_OK;
  if (a->a == nullptr || a->b == nullptr || a->c == nullptr) return BIO_ERR_ARG;
  int st = bio_host::ensure_device(a->device);
  if (st != BIO_OK) return st;
  if (!aligned16(a->a) || !aligned16(a->b) || (up != nullptr && !aligned16(up)))
    return BIO_ERR_ALIGN;
  bool a_mn;
  if (a->a_sk == 1) {
    a_mn = false;
  } else if (a->a_sm == 1) {
    a_mn = true;
  } else {
    return BIO_ERR_STRIDE;
  }
  bool b_mn;
  if (a->b_sk == 1) {
    b_mn = false;
  } else if (a->b_sn == 1) {
    b_mn = true;
  } else {
    return BIO_ERR_STRIDE;
  }
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  if (up != nullptr) {
    if (a->dtype == BIO_BF16)
      return dispatch_swiglu<__nv_bfloat16>(a, seg, up, stream, a_mn, b_mn);
    return dispatch_swiglu<__half>(a, seg, up, stream, a_mn, b_mn);
  }
  // tile from the mean rows per segment (the counts live on the device); any
  // tile gives the same bits
  TileChoice tc = pick_tile((a->m + a->batch1 - 1) / a->batch1, a->n, a->batch1,
                            bio_host::sm_count(a->device));
  tc = for_layout(tc, b_mn);
  if (a->dtype == BIO_BF16) return dispatch_tc<__nv_bfloat16>(a, tc, stream, a_mn, b_mn, seg);
  return dispatch_tc<__half>(a, tc, stream, a_mn, b_mn, seg);
}

}  // namespace

extern "C" {

int bio_gemm(const bio_gemm_args* a, void* stream_v) { return gemm_impl(a, nullptr, stream_v); }

int bio_gemm_residual(const bio_gemm_args* a, const void* residual, int64_t residual_row_stride,
                      void* stream_v) {
  if (a == nullptr || residual == nullptr) return BIO_ERR_ARG;
  if (a->dtype != BIO_F16 && a->dtype != BIO_BF16) return BIO_ERR_DTYPE;
  if (a->batch1 != 1 || a->batch2 != 1 || a->flags != 0) return BIO_ERR_ARG;
  if (a->k < 1) return BIO_ERR_SHAPE;
  if (a->c_sn != 1 || residual_row_stride < a->n) return BIO_ERR_STRIDE;
  const EpiResidual res{residual, residual_row_stride};
  return gemm_impl(a, nullptr, stream_v, &res);
}

int bio_gemm_tiled(const bio_gemm_args* a, int32_t tile_m, int32_t tile_n, void* stream_v) {
  if (tile_m != 128 && tile_m != 256) return BIO_ERR_ARG;
  const TileChoice tc{tile_m == 256, static_cast<int>(tile_n)};
  if (!tile_supported(tc)) return BIO_ERR_ARG;
  return gemm_impl(a, &tc, stream_v);
}

int bio_gemm_segmented(const bio_gemm_args* a, const int32_t* seg, void* stream_v) {
  if (seg == nullptr) return BIO_ERR_ARG;
  return grouped_impl(a, seg, nullptr, stream_v);
}

int bio_conv_transpose(int32_t dtype, const void* x, const void* w, const void* bias, void* y,
                       const bio_conv_geom* g, int64_t og, int32_t device, void* stream_v) {
  if (g == nullptr || og < 1) return BIO_ERR_SHAPE;
  if (dtype != BIO_F16 && dtype != BIO_BF16) return BIO_ERR_DTYPE;
  const int64_t nb = g->batch, cin = g->channels, groups = g->groups;
  if (nb < 0 || cin < 1 || groups < 1 || cin % groups != 0) return BIO_ERR_SHAPE;
  int64_t p_in = 1, kvol = 1, so = 1;
  for (int d = 0; d < 3; ++d) {
    if (g->in[d] < 1 || g->kernel[d] < 1) return BIO_ERR_SHAPE;
    if (g->stride[d] != g->kernel[d] || g->padding[d] != 0 || g->dilation[d] != 1)
      return BIO_ERR_ARG;  // non-overlapping (stride == kernel) only
    p_in *= g->in[d];
    kvol *= g->kernel[d];
    so *= g->in[d] * g->kernel[d];
  }
  const int64_t cg = cin / groups;
  const int64_t n = og * kvol;
  if (nb == 0) return BIO_OK;
  if (p_in > 2147483647 || n > 2147483647 || cg > 2147483647) return BIO_ERR_SHAPE;
  if (x == nullptr || w == nullptr || y == nullptr) return BIO_ERR_ARG;
  int st = bio_host::ensure_device(device);
  if (st != BIO_OK) return st;
  // tensor maps: 16-byte aligned bases and strides (P and og*kvol multiples of 8)
  if (!aligned16(x) || !aligned16(w) || p_in % 8 != 0 || n % 8 != 0) return BIO_ERR_ALIGN;
  bio_gemm_args a{};
  a.dtype = dtype;
  a.flags = 0;
  a.batch1 = nb;
  a.batch2 = groups;
  a.m = p_in;  // A[m = input position, k = c] = x[b, g*cg + c, m]
  a.n = n;     // B[k = c, n = (o, kernel offset)] = w[g*cg + c, n]
  a.k = cg;
  a.a = x;
  a.a_sm = 1;
  a.a_sk = p_in;
  a.a_s1 = cin * p_in;
  a.a_s2 = cg * p_in;
  a.a_div2 = 1;
  a.b = w;
  a.b_sk = n;
  a.b_sn = 1;
  a.b_s1 = 0;
  a.b_s2 = cg * n;
  a.b_div2 = 1;
  a.c = y;
  a.c_sm = 0;
  a.c_sn = 0;
  a.c_s1 = groups * og * so;
  a.c_s2 = og * so;
  a.bias = bias;
  a.bias_s2 = og;
  a.alpha = 1.0f;
  a.device = device;
  ScatterSpec sc;
  sc.s1 = static_cast<int>(g->in[1]);
  sc.s2 = static_cast<int>(g->in[2]);
  sc.k0 = static_cast<int>(g->kernel[0]);
  sc.k1 = static_cast<int>(g->kernel[1]);
  sc.k2 = static_cast<int>(g->kernel[2]);
  sc.o2 = static_cast<int>(g->in[2] * g->kernel[2]);
  sc.so = so;
  sc.o1o2 = g->in[1] * g->kernel[1] * g->in[2] * g->kernel[2];
  sc.vec = aligned16(y);
  TileChoice tc = pick_tile(p_in, n, nb * groups, bio_host::sm_count(device));
  tc = for_layout(tc, true);  // N-contiguous B: whole 64-column atoms
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  if (dtype == BIO_BF16)
    return dispatch_tc<__nv_bfloat16>(&a, tc, stream, true, true, nullptr, &sc);
  return dispatch_tc<__half>(&a, tc, stream, true, true, nullptr, &sc);
}

int bio_gemm_swiglu(const bio_gemm_args* a, const void* up, const int32_t* seg,
                    void* stream_v) {
  if (up == nullptr) return BIO_ERR_ARG;
  return grouped_impl(a, seg, up, stream_v);
}

int bio_pack_rows(int32_t dtype, const void* src, int64_t nb1, int64_t nb2, int64_t rows,
                  int64_t cols, int64_t s_b1, int64_t s_b2, int64_t s_row, int64_t s_col,
                  void* dst, int64_t cols_pad, int32_t device, void* stream_v) {
  if (nb1 < 0 || nb2 < 0 || rows < 0 || cols < 0 || cols_pad < cols) return BIO_ERR_SHAPE;
  const int64_t total = nb1 * nb2 * rows * cols_pad;
  if (total == 0) return BIO_OK;
  if (src == nullptr || dst == nullptr) return BIO_ERR_ARG;
  int st = bio_host::ensure_device(device);
  if (st != BIO_OK) return st;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  int64_t blocks = (total + 255) / 256;
  if (blocks > 65536) blocks = 65536;
  const unsigned g = static_cast<unsigned>(blocks);
  switch (dtype) {
    case BIO_F32:
      bio::pack_rows_kernel<float><<<g, 256, 0, stream>>>(
          static_cast<const float*>(src), nb2, rows, cols, s_b1, s_b2, s_row, s_col,
          static_cast<float*>(dst), cols_pad, total);
      break;
    case BIO_F16:
      bio::pack_rows_kernel<__half><<<g, 256, 0, stream>>>(
          static_cast<const __half*>(src), nb2, rows, cols, s_b1, s_b2, s_row, s_col,
          static_cast<__half*>(dst), cols_pad, total);
      break;
    case BIO_BF16:
      bio::pack_rows_kernel<__nv_bfloat16><<<g, 256, 0, stream>>>(
          static_cast<const __nv_bfloat16*>(src), nb2, rows, cols, s_b1, s_b2, s_row, s_col,
          static_cast<__nv_bfloat16*>(dst), cols_pad, total);
      break;
    default: return BIO_ERR_DTYPE;
  }
  return bio_host::launch_status(cudaGetLastError());
}

}  // extern "C"
