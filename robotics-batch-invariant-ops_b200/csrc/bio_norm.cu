// Batch-invariant fused LayerNorm and RMSNorm over the last dimension.
//
// One fixed team of threads owns one row of n elements: 32 threads (one
// warp) for n <= 2048, 256 threads for n <= 16384, 1024 threads beyond.  The
// team and its work split are functions of n only.  Element i belongs to
// 8-element group i/8, group g to thread g % team; a thread folds its groups
// in increasing g (elements of a group in order), a fixed xor-shuffle tree
// combines the warp, and multi-warp teams add the per-warp partials in warp
// order.  16-byte loads/stores are used when a group is complete and
// aligned; that changes the instruction, never the order of the sums.
//
// LayerNorm: mean = sum(x) / n, var = sum((x - mean)^2) / n (two passes over
// the row held in registers), rstd = rsqrt(var + eps),
// y = (x - mean) * rstd * w + b.  RMSNorm: rstd = rsqrt(sum(x^2) / n + eps),
// y = x * rstd * w.  All in fp32, one rounding to the output dtype; the fp32
// mean / rstd per row can be written out (aten::native_layer_norm and
// aten::_fused_rms_norm return them).
//
// Not in the reference, which normalises with stock torch or builds RMSNorm
// from its mean_dim (batch_invariant_ops.py:1395-1482); these are the fused
// kernels its row-reduction design implies.  A row's bits depend on that row
// and on n only, so every output is batch invariant.
#include "bio_common.cuh"

namespace bio {

constexpr int kNormWarpMax = 2048;   // one warp per row up to here
constexpr int kNormCtaMax = 16384;   // one 256-thread CTA per row up to here

template <typename T>
__device__ __forceinline__ void norm_load8(const T* __restrict__ row, int base, int n,
                                           float (&v)[8]) {
  const T* p = row + base;
  if (base + 8 <= n && (reinterpret_cast<uintptr_t>(p) & 15u) == 0 && sizeof(T) == 2) {
    const uint4 w = *reinterpret_cast<const uint4*>(p);
    const T* e = reinterpret_cast<const T*>(&w);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = to_f32(e[j]);
  } else if (base + 8 <= n && (reinterpret_cast<uintptr_t>(p) & 15u) == 0 && sizeof(T) == 4) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = (base + j < n) ? to_f32(p[j]) : 0.f;
  }
}

template <typename T>
__device__ __forceinline__ void norm_store8(T* __restrict__ row, int base, int n,
                                            const float (&o)[8]) {
  T* p = row + base;
  if (base + 8 <= n && (reinterpret_cast<uintptr_t>(p) & 15u) == 0) {
    if constexpr (sizeof(T) == 2) {
      uint4 w;
      T* e = reinterpret_cast<T*>(&w);
#pragma unroll
      for (int j = 0; j < 8; ++j) e[j] = from_f32<T>(o[j]);
      *reinterpret_cast<uint4*>(p) = w;
    } else {
      *reinterpret_cast<float4*>(p) = make_float4(o[0], o[1], o[2], o[3]);
      *reinterpret_cast<float4*>(p + 4) = make_float4(o[4], o[5], o[6], o[7]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (base + j < n) p[j] = from_f32<T>(o[j]);
  }
}

__device__ __forceinline__ float warp_sum_fixed(float v) {
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
  return v;
}

// Team-wide sum in fixed order: per-warp xor tree, then (multi-warp teams)
// the warp partials added in warp order by every thread.
template <int TEAM>
__device__ __forceinline__ float team_sum(float v, float* red) {
  v = warp_sum_fixed(v);
  if constexpr (TEAM == 32) {
    return v;
  } else {
    constexpr int kWarps = TEAM / 32;
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) red[warp] = v;
    __syncthreads();
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s += red[w];
    __syncthreads();  // red is reused by the next reduction
    return s;
  }
}

struct NormParams {
  const void* x;
  const void* w;
  const void* b;
  void* y;
  float* mean_out;
  float* rstd_out;
  int64_t rows;
  int n;
  float eps;
  int64_t x_stride, y_stride;  // elements between rows
};

// Affine parameters of one 8-element group (16-byte loads when aligned, the
// same values as element loads): `fill` where the parameter is absent.
template <typename W>
__device__ __forceinline__ void param8(const W* p, int base, int n, float fill, float (&o)[8]) {
  if (p != nullptr) {
    norm_load8<W>(p, base, n, o);
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = fill;
  }
}

// Row held in registers: GPT (groups per thread) groups of 8 per thread.
template <typename T, typename W, int TEAM, int GPT, bool RMS>
// One-warp teams: 8 rows per 256-thread CTA, and enough CTAs per SM to keep
// rows in flight.  Three CTAs cap a thread at 80 registers, which holds the
// 16-bit RMSNorm rows and LayerNorm rows of up to 5 groups without spills;
// the rest keep two CTAs (128 registers).
__global__ void __launch_bounds__(
    TEAM == 32 ? 256 : TEAM,
    TEAM == 32 ? ((sizeof(T) == 2 && sizeof(W) == 2 && (RMS || GPT <= 5)) ? 3 : 2) : 1)
    norm_reg_kernel(const NormParams p) {
  __shared__ float red[32];
  const int lane_in_team = TEAM == 32 ? (threadIdx.x & 31) : threadIdx.x;
  const int64_t row = TEAM == 32 ? static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5)
                                 : static_cast<int64_t>(blockIdx.x);
  if (row >= p.rows) return;  // warp-uniform (TEAM == 32); CTA-uniform otherwise
  const int n = p.n;
  const T* xr = static_cast<const T*>(p.x) + row * p.x_stride;
  T* yr = static_cast<T*>(p.y) + row * p.y_stride;
  const W* w = static_cast<const W*>(p.w);
  const W* b = static_cast<const W*>(p.b);

  float v[GPT][8];
#pragma unroll
  for (int j = 0; j < GPT; ++j) {
    const int base = (lane_in_team + j * TEAM) * 8;
    if (base < n)
      norm_load8<T>(xr, base, n, v[j]);
    else
#pragma unroll
      for (int e = 0; e < 8; ++e) v[j][e] = 0.f;
  }
  const float inv_n = 1.0f / static_cast<float>(n);
  float mean = 0.f, rstd;
  if constexpr (RMS) {
    float sq = 0.f;
#pragma unroll
    for (int j = 0; j < GPT; ++j)
#pragma unroll
      for (int e = 0; e < 8; ++e) sq = fmaf(v[j][e], v[j][e], sq);
    sq = team_sum<TEAM>(sq, red);
    rstd = rsqrtf(sq * inv_n + p.eps);
  } else {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < GPT; ++j)
#pragma unroll
      for (int e = 0; e < 8; ++e) s += v[j][e];
    s = team_sum<TEAM>(s, red);
    mean = s * inv_n;
    float sq = 0.f;
#pragma unroll
    for (int j = 0; j < GPT; ++j) {
      const int base = (lane_in_team + j * TEAM) * 8;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float d = base + e < n ? v[j][e] - mean : 0.f;
        sq = fmaf(d, d, sq);
      }
    }
    sq = team_sum<TEAM>(sq, red);
    rstd = rsqrtf(sq * inv_n + p.eps);
  }
  if (lane_in_team == 0) {
    if (p.mean_out != nullptr) p.mean_out[row] = mean;
    if (p.rstd_out != nullptr) p.rstd_out[row] = rstd;
  }
#pragma unroll
  for (int j = 0; j < GPT; ++j) {
    const int base = (lane_in_team + j * TEAM) * 8;
    if (base >= n) continue;
    float o[8], wv[8], bv[8];
    param8<W>(w, base, n, 1.f, wv);
    if constexpr (!RMS) param8<W>(b, base, n, 0.f, bv);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      if constexpr (RMS) {
        o[e] = v[j][e] * rstd * wv[e];
      } else {
        const float t = (v[j][e] - mean) * rstd * wv[e];
        o[e] = b != nullptr ? t + bv[e] : t;
      }
    }
    norm_store8<T>(yr, base, n, o);
  }
}

// Rows longer than kNormCtaMax: a 1024-thread team reads the row from
// global memory once per pass (same group-to-thread assignment).
template <typename T, typename W, bool RMS>
__global__ void __launch_bounds__(1024) norm_loop_kernel(const NormParams p) {
  __shared__ float red[32];
  constexpr int TEAM = 1024;
  const int64_t row = blockIdx.x;
  if (row >= p.rows) return;
  const int n = p.n;
  const int groups = (n + 7) / 8;
  const T* xr = static_cast<const T*>(p.x) + row * p.x_stride;
  T* yr = static_cast<T*>(p.y) + row * p.y_stride;
  const W* w = static_cast<const W*>(p.w);
  const W* b = static_cast<const W*>(p.b);
  const float inv_n = 1.0f / static_cast<float>(n);
  float mean = 0.f;
  if constexpr (!RMS) {
    float s = 0.f;
    for (int g = threadIdx.x; g < groups; g += TEAM) {
      float v[8];
      norm_load8<T>(xr, g * 8, n, v);
#pragma unroll
      for (int e = 0; e < 8; ++e) s += v[e];
    }
    mean = team_sum<TEAM>(s, red) * inv_n;
  }
  float sq = 0.f;
  for (int g = threadIdx.x; g < groups; g += TEAM) {
    float v[8];
    norm_load8<T>(xr, g * 8, n, v);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float d = g * 8 + e < n ? v[e] - mean : 0.f;
      sq = fmaf(d, d, sq);
    }
  }
  const float rstd = rsqrtf(team_sum<TEAM>(sq, red) * inv_n + p.eps);
  if (threadIdx.x == 0) {
    if (p.mean_out != nullptr) p.mean_out[row] = mean;
    if (p.rstd_out != nullptr) p.rstd_out[row] = rstd;
  }
  for (int g = threadIdx.x; g < groups; g += TEAM) {
    float v[8], o[8], wv[8], bv[8];
    norm_load8<T>(xr, g * 8, n, v);
    param8<W>(w, g * 8, n, 1.f, wv);
    if constexpr (!RMS) param8<W>(b, g * 8, n, 0.f, bv);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float t = (v[e] - mean) * rstd * wv[e];
      o[e] = (!RMS && b != nullptr) ? t + bv[e] : t;
    }
    norm_store8<T>(yr, g * 8, n, o);
  }
}

}  // namespace bio

namespace {

template <typename T, typename W, bool RMS>
int launch_norm(const bio::NormParams& p, cudaStream_t s) {
  const int n = p.n;
  const int64_t rows = p.rows;
  const unsigned warp_blocks = static_cast<unsigned>((rows + 7) / 8);
  const unsigned cta_blocks = static_cast<unsigned>(rows);
  if (n <= 256) {
    bio::norm_reg_kernel<T, W, 32, 1, RMS><<<warp_blocks, 256, 0, s>>>(p);
  } else if (n <= 512) {
    bio::norm_reg_kernel<T, W, 32, 2, RMS><<<warp_blocks, 256, 0, s>>>(p);
  } else if (n <= 1024) {
    bio::norm_reg_kernel<T, W, 32, 4, RMS><<<warp_blocks, 256, 0, s>>>(p);
  } else if (n <= 1280) {
    // e.g. the 1152-wide vision rows: five groups of 8 per lane
    bio::norm_reg_kernel<T, W, 32, 5, RMS><<<warp_blocks, 256, 0, s>>>(p);
  } else if (n <= bio::kNormWarpMax) {
    bio::norm_reg_kernel<T, W, 32, 8, RMS><<<warp_blocks, 256, 0, s>>>(p);
  } else if (n <= 4096) {
    bio::norm_reg_kernel<T, W, 256, 2, RMS><<<cta_blocks, 256, 0, s>>>(p);
  } else if (n <= 8192) {
    bio::norm_reg_kernel<T, W, 256, 4, RMS><<<cta_blocks, 256, 0, s>>>(p);
  } else if (n <= bio::kNormCtaMax) {
    bio::norm_reg_kernel<T, W, 256, 8, RMS><<<cta_blocks, 256, 0, s>>>(p);
  } else {
    bio::norm_loop_kernel<T, W, RMS><<<cta_blocks, 1024, 0, s>>>(p);
  }
  return bio_host::launch_status(cudaGetLastError());
}

template <typename T, bool RMS>
int dispatch_w(int32_t w_dtype, const bio::NormParams& p, cudaStream_t s) {
  switch (w_dtype) {
    case BIO_F32: return launch_norm<T, float, RMS>(p, s);
    case BIO_F16: return launch_norm<T, __half, RMS>(p, s);
    case BIO_BF16: return launch_norm<T, __nv_bfloat16, RMS>(p, s);
    default: return BIO_ERR_DTYPE;
  }
}

template <bool RMS>
int dispatch_norm(int32_t dtype, int32_t w_dtype, const bio::NormParams& p, cudaStream_t s) {
  switch (dtype) {
    case BIO_F32: return dispatch_w<float, RMS>(w_dtype, p, s);
    case BIO_F16: return dispatch_w<__half, RMS>(w_dtype, p, s);
    case BIO_BF16: return dispatch_w<__nv_bfloat16, RMS>(w_dtype, p, s);
    default: return BIO_ERR_DTYPE;
  }
}

}  // namespace

extern "C" {

int bio_norm(int32_t kind, int32_t dtype, int32_t w_dtype, const void* x, const void* weight,
             const void* bias, void* y, float* mean_out, float* rstd_out, int64_t rows, int64_t n,
             int64_t x_row_stride, int64_t y_row_stride, float eps, int32_t device,
             void* stream) {
  if (kind != BIO_NORM_LAYER && kind != BIO_NORM_RMS) return BIO_ERR_ARG;
  if (rows < 0 || n < 0 || n > 2147483647 / 2) return BIO_ERR_SHAPE;
  if (kind == BIO_NORM_RMS && bias != nullptr) return BIO_ERR_ARG;
  if (rows == 0 || n == 0) return BIO_OK;
  if (rows > 2147483647) return BIO_ERR_SHAPE;
  if (x == nullptr || y == nullptr) return BIO_ERR_ARG;
  if (x_row_stride < n || y_row_stride < n) return BIO_ERR_STRIDE;
  if (!(eps >= 0.f)) return BIO_ERR_ARG;
  int st = bio_host::ensure_device(device);
  if (st != BIO_OK) return st;
  bio::NormParams p;
  p.x = x;
  p.w = weight;
  p.b = bias;
  p.y = y;
  p.mean_out = mean_out;
  p.rstd_out = rstd_out;
  p.rows = rows;
  p.n = static_cast<int>(n);
  p.eps = eps;
  p.x_stride = x_row_stride;
  p.y_stride = y_row_stride;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return kind == BIO_NORM_RMS ? dispatch_norm<true>(dtype, w_dtype, p, s)
                              : dispatch_norm<false>(dtype, w_dtype, p, s);
}

}  // extern "C"
