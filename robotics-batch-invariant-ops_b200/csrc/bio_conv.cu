// Convolution lowering kernels.
//
// * bio_im2col: gathers the receptive fields of an N-d (N <= 3) convolution
//   into a dense [B][G][L][Kpad] patch matrix (K = C/G * kernel volume, zero
//   padded to Kpad); the GEMM then computes out[b, g] = W_g [Og, K] x
//   patches[b, g]^T, one independent fixed-schedule GEMM per (sample, group),
//   so a sample's output never depends on the other samples.
// * bio_depthwise_conv1d: direct depthwise kernel, fp32 accumulation over the
//   taps in order k = 0..K-1, bias added after the taps.
// * bio_conv_transpose_scatter: pixel-shuffle layout transform (+ bias) of the
//   per-(sample, group) GEMM output of a non-overlapping transposed
//   convolution (stride == kernel).
//
// Reference: conv1d_batch_invariant (batch_invariant_ops.py:497-595, depthwise
// kernel :435-494), conv2d_batch_invariant (:598-682), conv3d_batch_invariant
// (:685-780), conv_transpose2d/3d_batch_invariant (:783-941).
#include <mutex>

#include "bio_common.cuh"

namespace bio {

struct Geom {
  int64_t batch, channels, groups;
  int64_t in[3], kernel[3], stride[3], padding[3], dilation[3], out[3];
};

// One warp per patch row (b, group, l): the row's output position and input
// base are decomposed once, lanes walk the row's kpad entries (32-bit index
// arithmetic within the row) and store them contiguously.
template <typename T>
__global__ void __launch_bounds__(256)
    im2col_kernel(const T* __restrict__ x, T* __restrict__ patches, Geom g, int64_t k_real,
                  int64_t kpad, int64_t rows) {
  const uint32_t k1 = static_cast<uint32_t>(g.kernel[1]);
  const uint32_t k2 = static_cast<uint32_t>(g.kernel[2]);
  const uint32_t kvol = static_cast<uint32_t>(g.kernel[0]) * k1 * k2;
  const int64_t L = g.out[0] * g.out[1] * g.out[2];
  const int64_t cg = g.channels / g.groups;
  const int64_t in_vol = g.in[0] * g.in[1] * g.in[2];
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
       row < rows; row += warps) {
    const int64_t l = row % L;
    const int64_t bg = row / L;
    const int64_t grp = bg % g.groups;
    const int64_t b = bg / g.groups;
    const int64_t o2 = l % g.out[2];
    const int64_t t = l / g.out[2];
    const int64_t o1 = t % g.out[1];
    const int64_t o0 = t / g.out[1];
    const int64_t b0 = o0 * g.stride[0] - g.padding[0];
    const int64_t b1 = o1 * g.stride[1] - g.padding[1];
    const int64_t b2 = o2 * g.stride[2] - g.padding[2];
    const T* xs = x + (b * g.channels + grp * cg) * in_vol;
    T* dst = patches + row * kpad;
    for (int64_t kk = lane; kk < kpad; kk += 32) {
      T v = from_f32<T>(0.f);
      if (kk < k_real) {
        const uint32_t k32 = static_cast<uint32_t>(kk);
        const uint32_t c = k32 / kvol;
        uint32_t z = k32 - c * kvol;
        const uint32_t z12 = z % (k1 * k2);
        const uint32_t z0 = z / (k1 * k2);
        const uint32_t z1 = z12 / k2;
        const uint32_t z2 = z12 - z1 * k2;
        const int64_t i0 = b0 + static_cast<int64_t>(z0) * g.dilation[0];
        const int64_t i1 = b1 + static_cast<int64_t>(z1) * g.dilation[1];
        const int64_t i2 = b2 + static_cast<int64_t>(z2) * g.dilation[2];
        if (i0 >= 0 && i0 < g.in[0] && i1 >= 0 && i1 < g.in[1] && i2 >= 0 && i2 < g.in[2])
          v = xs[static_cast<int64_t>(c) * in_vol + (i0 * g.in[1] + i1) * g.in[2] + i2];
      }
      dst[kk] = v;
    }
  }
}

// Table-driven im2col for patch rows of at most kIm2colTable entries: each
// CTA first tabulates, per patch column kk, the input offset of its tap
// (channel, z0*dil0, z1*dil1, z2*dil2) and the three dilated tap positions;
// a warp then fills one patch row with one table read, the bounds test (only
// for rows that touch the padding) and one load per entry.
constexpr int kIm2colTable = 2048;

template <typename T>
__global__ void __launch_bounds__(256)
    im2col_table_kernel(const T* __restrict__ x, T* __restrict__ patches, Geom g, int k_real,
                        int kpad, int64_t rows) {
  __shared__ int toff[kIm2colTable];
  __shared__ short tz[3][kIm2colTable];
  const int k1 = static_cast<int>(g.kernel[1]), k2 = static_cast<int>(g.kernel[2]);
  const int kvol = static_cast<int>(g.kernel[0]) * k1 * k2;
  const int64_t in1 = g.in[1], in2 = g.in[2];
  const int64_t in_vol = g.in[0] * in1 * in2;
  for (int kk = threadIdx.x; kk < k_real; kk += blockDim.x) {
    const int c = kk / kvol;
    const int z = kk - c * kvol;
    const int z0 = z / (k1 * k2), z1 = (z / k2) % k1, z2 = z % k2;
    const int d0 = z0 * static_cast<int>(g.dilation[0]);
    const int d1 = z1 * static_cast<int>(g.dilation[1]);
    const int d2 = z2 * static_cast<int>(g.dilation[2]);
    toff[kk] = static_cast<int>(c * in_vol + (d0 * in1 + d1) * in2 + d2);
    tz[0][kk] = static_cast<short>(d0);
    tz[1][kk] = static_cast<short>(d1);
    tz[2][kk] = static_cast<short>(d2);
  }
  __syncthreads();
  const int64_t L = g.out[0] * g.out[1] * g.out[2];
  const int64_t cg = g.channels / g.groups;
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  const int span0 = static_cast<int>((g.kernel[0] - 1) * g.dilation[0]);
  const int span1 = static_cast<int>((g.kernel[1] - 1) * g.dilation[1]);
  const int span2 = static_cast<int>((g.kernel[2] - 1) * g.dilation[2]);
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
       row < rows; row += warps) {
    const int64_t l = row % L;
    const int64_t bg = row / L;
    const int64_t grp = bg % g.groups;
    const int64_t b = bg / g.groups;
    const int64_t o2 = l % g.out[2];
    const int64_t t = l / g.out[2];
    const int64_t o1 = t % g.out[1];
    const int64_t o0 = t / g.out[1];
    const int64_t b0 = o0 * g.stride[0] - g.padding[0];
    const int64_t b1 = o1 * g.stride[1] - g.padding[1];
    const int64_t b2 = o2 * g.stride[2] - g.padding[2];
    const bool interior = b0 >= 0 && b1 >= 0 && b2 >= 0 && b0 + span0 < g.in[0] &&
                          b1 + span1 < in1 && b2 + span2 < in2;
    const T* xs = x + (b * g.channels + grp * cg) * in_vol + (b0 * in1 + b1) * in2 + b2;
    T* dst = patches + row * kpad;
    if (interior) {
      for (int kk = lane; kk < kpad; kk += 32)
        dst[kk] = kk < k_real ? xs[toff[kk]] : from_f32<T>(0.f);
    } else {
      for (int kk = lane; kk < kpad; kk += 32) {
        T v = from_f32<T>(0.f);
        if (kk < k_real) {
          const int64_t i0 = b0 + tz[0][kk], i1 = b1 + tz[1][kk], i2 = b2 + tz[2][kk];
          if (i0 >= 0 && i0 < g.in[0] && i1 >= 0 && i1 < in1 && i2 >= 0 && i2 < in2)
            v = xs[toff[kk]];
        }
        dst[kk] = v;
      }
    }
  }
}

// One warp per (sample, channel) row; lanes walk the output positions, each
// folding its taps in order k = 0..K-1 in fp32, bias added after the taps.
template <typename T>
__global__ void __launch_bounds__(256)
    depthwise_conv1d_kernel(const T* __restrict__ x, const T* __restrict__ w,
                            const T* __restrict__ bias, T* __restrict__ y, int64_t channels,
                            int64_t lin, int64_t lout, int ksize, int stride, int pad, int dil,
                            int64_t rows) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  for (int64_t bc = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
       bc < rows; bc += warps) {
    const int64_t c = bc % channels;
    const T* xr = x + bc * lin;
    const T* wr = w + c * ksize;
    const float bv = bias != nullptr ? to_f32(bias[c]) : 0.f;
    T* yr = y + bc * lout;
    for (int64_t l = lane; l < lout; l += 32) {
      float acc = 0.f;
      const int64_t i0 = l * stride - pad;
      for (int k = 0; k < ksize; ++k) {
        const int64_t i = i0 + static_cast<int64_t>(k) * dil;
        if (i >= 0 && i < lin) acc += to_f32(xr[i]) * to_f32(wr[k]);
      }
      if (bias != nullptr) acc += bv;
      yr[l] = from_f32<T>(acc);
    }
  }
}

// Depthwise 1-D convolution with the input row staged in shared memory: a
// warp copies its (sample, channel) row with all loads in flight, then each
// lane computes outputs from shared memory (same tap order k = 0..K-1 and
// bias after the taps as depthwise_conv1d_kernel, so results are identical).
template <typename T, int KS>
__global__ void __launch_bounds__(256)
    depthwise_conv1d_smem_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                 const T* __restrict__ bias, T* __restrict__ y, int64_t channels,
                                 int lin, int lout, int ksize, int stride, int pad, int dil,
                                 int64_t rows) {
  extern __shared__ __align__(16) unsigned char dw_smem[];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  T* srow = reinterpret_cast<T*>(dw_smem) + static_cast<int64_t>(wid) * lin;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  for (int64_t bc = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + wid; bc < rows;
       bc += warps) {
    const int64_t c = bc % channels;
    const T* xr = x + bc * lin;
    __syncwarp();
    if (sizeof(T) == 2 && (lin & 1) == 0) {
      // 4-byte copies (rows of even length start 4-byte aligned)
      const uint32_t* xw = reinterpret_cast<const uint32_t*>(xr);
      uint32_t* sw = reinterpret_cast<uint32_t*>(srow);
#pragma unroll 8
      for (int i = lane; i < lin / 2; i += 32) sw[i] = xw[i];
    } else {
#pragma unroll 8
      for (int i = lane; i < lin; i += 32) srow[i] = xr[i];
    }
    __syncwarp();
    const T* wr = w + c * ksize;
    const float bv = bias != nullptr ? to_f32(bias[c]) : 0.f;
    T* yr = y + bc * lout;
    if (KS > 0 && ksize == KS) {
      constexpr int kTaps = KS > 0 ? KS : 1;
      float wk[kTaps];
#pragma unroll
      for (int k = 0; k < kTaps; ++k) wk[k] = to_f32(wr[k]);
      // outputs whose taps all lie inside the row need no bounds test
      const int l_lo = pad > 0 ? (pad + stride - 1) / stride : 0;
      const int l_hi_raw = (lin - 1 - (kTaps - 1) * dil + pad) / stride;  // last interior l
      const int l_hi = (lin - 1 - (kTaps - 1) * dil + pad) < 0 ? -1 : l_hi_raw;
      for (int l = lane; l < lout; l += 32) {
        float acc = 0.f;
        const int i0 = l * stride - pad;
        if (l >= l_lo && l <= l_hi) {
#pragma unroll
          for (int k = 0; k < kTaps; ++k) acc += to_f32(srow[i0 + k * dil]) * wk[k];
        } else {
#pragma unroll
          for (int k = 0; k < kTaps; ++k) {
            const int i = i0 + k * dil;
            if (i >= 0 && i < lin) acc += to_f32(srow[i]) * wk[k];
          }
        }
        if (bias != nullptr) acc += bv;
        yr[l] = from_f32<T>(acc);
      }
    } else {
      for (int l = lane; l < lout; l += 32) {
        float acc = 0.f;
        const int i0 = l * stride - pad;
        for (int k = 0; k < ksize; ++k) {
          const int i = i0 + k * dil;
          if (i >= 0 && i < lin) acc += to_f32(srow[i]) * to_f32(wr[k]);
        }
        if (bias != nullptr) acc += bv;
        yr[l] = from_f32<T>(acc);
      }
    }
  }
}

// dst[b, g*Og + o, s*k + z ...] = src[b, g, o*kvol + z, s] (+ bias[g*Og + o]).
// One warp per output row (b, oc, p0, p1) of length D2 = s2*k2: lane X reads
// src[..., z2 = X % k2][i2 = X / k2] and the row is written contiguously; the
// (i2, z2) pair advances by 32 positions per step without a division.
template <typename T>
__global__ void __launch_bounds__(256)
    convt_scatter_kernel(const T* __restrict__ src, const T* __restrict__ bias,
                         T* __restrict__ dst, Geom g, int64_t og, int64_t rows) {
  const int64_t k0 = g.kernel[0], k1 = g.kernel[1], k2 = g.kernel[2];
  const int64_t s1 = g.in[1], s2 = g.in[2];
  const int64_t d0 = g.in[0] * k0, d1 = s1 * k1, d2 = s2 * k2;
  const int64_t in_vol = g.in[0] * s1 * s2;
  const int64_t kvol = k0 * k1 * k2;
  const int64_t cout = og * g.groups;
  const int lane = threadIdx.x & 31;
  const int64_t step_i = 32 / k2, step_z = 32 % k2;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
       r < rows; r += warps) {
    const int64_t p1 = r % d1;
    int64_t rest = r / d1;
    const int64_t p0 = rest % d0;
    rest /= d0;
    const int64_t oc = rest % cout;
    const int64_t b = rest / cout;
    const int64_t i0 = p0 / k0, z0 = p0 - i0 * k0;
    const int64_t i1 = p1 / k1, z1 = p1 - i1 * k1;
    const int64_t grp = oc / og, o = oc - grp * og;
    const T* srow = src + ((b * g.groups + grp) * og * kvol + o * kvol + (z0 * k1 + z1) * k2) * in_vol +
                    (i0 * s1 + i1) * s2;
    const float bv = bias != nullptr ? to_f32(bias[oc]) : 0.f;
    T* drow = dst + r * d2;
    int64_t i2 = lane / k2, z2 = lane - (lane / k2) * k2;
    for (int64_t X = lane; X < d2; X += 32) {
      float v = to_f32(srow[z2 * in_vol + i2]);
      if (bias != nullptr) v += bv;
      drow[X] = from_f32<T>(v);
      i2 += step_i;
      z2 += step_z;
      if (z2 >= k2) {
        z2 -= k2;
        ++i2;
      }
    }
  }
}

// One CTA per output channel plane (b, oc): the plane's kvol source rows
// (contiguous in the GEMM output) are staged in shared memory with a padded
// row stride (no bank conflicts between the k2 rows a warp reads), then every
// warp writes output rows contiguously, (i2, z2) advancing by 32 per step.
// 32-bit index arithmetic; used when the plane fits in shared memory.
template <typename T>
__global__ void __launch_bounds__(256)
    convt_plane_kernel(const T* __restrict__ src, const T* __restrict__ bias,
                       T* __restrict__ dst, Geom g, int og, int srow) {
  extern __shared__ __align__(16) unsigned char convt_smem[];
  T* sm = reinterpret_cast<T*>(convt_smem);
  const int k0 = static_cast<int>(g.kernel[0]), k1 = static_cast<int>(g.kernel[1]),
            k2 = static_cast<int>(g.kernel[2]);
  const int s1 = static_cast<int>(g.in[1]), s2 = static_cast<int>(g.in[2]);
  const int in_vol = static_cast<int>(g.in[0]) * s1 * s2;
  const int kvol = k0 * k1 * k2;
  const int d1 = s1 * k1, d2 = s2 * k2;
  const int rows = static_cast<int>(g.in[0]) * k0 * d1;  // output rows of the plane
  const int cout = og * static_cast<int>(g.groups);
  const int64_t plane = blockIdx.x;
  const int64_t b = plane / cout;
  const int oc = static_cast<int>(plane - b * cout);
  const int grp = oc / og, o = oc - grp * og;
  const T* sp = src + ((b * g.groups + grp) * og + o) * static_cast<int64_t>(kvol) * in_vol;
  if (sizeof(T) == 2 && (in_vol & 7) == 0 && (srow & 7) == 0 &&
      (reinterpret_cast<uintptr_t>(sp) & 15u) == 0) {
    // 16-byte copies (8 elements); srow keeps every staged row 16-byte aligned
    const int vrow = in_vol / 8;
    for (int e = threadIdx.x; e < kvol * vrow; e += blockDim.x) {
      const int z = e / vrow, i = e - z * vrow;
      *reinterpret_cast<uint4*>(sm + z * srow + i * 8) =
          reinterpret_cast<const uint4*>(sp + static_cast<int64_t>(z) * in_vol)[i];
    }
  } else {
    for (int z = 0; z < kvol; ++z)
      for (int i = threadIdx.x; i < in_vol; i += blockDim.x) sm[z * srow + i] = sp[z * in_vol + i];
  }
  __syncthreads();
  const float bv = bias != nullptr ? to_f32(bias[oc]) : 0.f;
  T* dp = dst + plane * static_cast<int64_t>(rows) * d2;
  const int lane = threadIdx.x & 31;
  const int step_i = 32 / k2, step_z = 32 % k2;
  for (int r = threadIdx.x >> 5; r < rows; r += blockDim.x >> 5) {
    const int p1 = r % d1, p0 = r / d1;
    const int i0 = p0 / k0, z0 = p0 - i0 * k0;
    const int i1 = p1 / k1, z1 = p1 - i1 * k1;
    const T* srow_p = sm + ((z0 * k1 + z1) * k2) * srow + (i0 * s1 + i1) * s2;
    T* drow = dp + static_cast<int64_t>(r) * d2;
    if (sizeof(T) == 2 && (d2 & 3) == 0 && (reinterpret_cast<uintptr_t>(drow) & 7u) == 0) {
      // four consecutive outputs per lane, one 8-byte store
      for (int X0 = lane * 4; X0 < d2; X0 += 128) {
        int i2 = X0 / k2, z2 = X0 - (X0 / k2) * k2;
        float v[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          v[e] = to_f32(srow_p[z2 * srow + i2]);
          if (bias != nullptr) v[e] += bv;
          if (++z2 == k2) {
            z2 = 0;
            ++i2;
          }
        }
        T o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) o[e] = from_f32<T>(v[e]);
        *reinterpret_cast<uint2*>(drow + X0) = *reinterpret_cast<const uint2*>(o);
      }
      continue;
    }
    int i2 = lane / k2, z2 = lane - (lane / k2) * k2;
    for (int X = lane; X < d2; X += 32) {
      float v = to_f32(srow_p[z2 * srow + i2]);
      if (bias != nullptr) v += bv;
      drow[X] = from_f32<T>(v);
      i2 += step_i;
      z2 += step_z;
      if (z2 >= k2) {
        z2 -= k2;
        ++i2;
      }
    }
  }
}

}  // namespace bio

namespace {

bio::Geom to_geom(const bio_conv_geom* c) {
  bio::Geom g;
  g.batch = c->batch;
  g.channels = c->channels;
  g.groups = c->groups;
  for (int i = 0; i < 3; ++i) {
    g.in[i] = c->in[i];
    g.kernel[i] = c->kernel[i];
    g.stride[i] = c->stride[i];
    g.padding[i] = c->padding[i];
    g.dilation[i] = c->dilation[i];
    g.out[i] = c->out[i];
  }
  return g;
}

// Grid for the warp-per-row kernels (8 warps per 256-thread block).
unsigned blocks_for_rows(int64_t rows) {
  int64_t b = (rows + 7) / 8;
  if (b > 65536 * 4) b = 65536 * 4;
  return static_cast<unsigned>(b);
}

bool geom_ok(const bio_conv_geom* c) {
  if (c == nullptr) return false;
  if (c->batch < 0 || c->channels <= 0 || c->groups <= 0 || c->channels % c->groups) return false;
  for (int i = 0; i < 3; ++i) {
    if (c->in[i] < 1 || c->kernel[i] < 1 || c->stride[i] < 1 || c->dilation[i] < 1) return false;
    if (c->padding[i] < 0 || c->out[i] < 0) return false;
  }
  return true;
}

}  // namespace

// Depthwise launch with the tap count as a template parameter for 2, 3 and
// 4 taps (0 = any count).
template <typename T>
int launch_dw_smem(const void* x, const void* w, const void* bias, void* y, int64_t channels,
                   int lin, int lout, int ksize, int stride, int pad, int dil, int64_t rows,
                   int64_t smem, cudaStream_t s) {
  const T* xt = static_cast<const T*>(x);
  const T* wt = static_cast<const T*>(w);
  const T* bt = static_cast<const T*>(bias);
  T* yt = static_cast<T*>(y);
  const unsigned g = blocks_for_rows(rows);
  switch (ksize) {
    case 2:
      bio::depthwise_conv1d_smem_kernel<T, 2><<<g, 256, smem, s>>>(xt, wt, bt, yt, channels, lin,
                                                                   lout, ksize, stride, pad, dil,
                                                                   rows);
      break;
    case 3:
      bio::depthwise_conv1d_smem_kernel<T, 3><<<g, 256, smem, s>>>(xt, wt, bt, yt, channels, lin,
                                                                   lout, ksize, stride, pad, dil,
                                                                   rows);
      break;
    case 4:
      bio::depthwise_conv1d_smem_kernel<T, 4><<<g, 256, smem, s>>>(xt, wt, bt, yt, channels, lin,
                                                                   lout, ksize, stride, pad, dil,
                                                                   rows);
      break;
    default:
      bio::depthwise_conv1d_smem_kernel<T, 0><<<g, 256, smem, s>>>(xt, wt, bt, yt, channels, lin,
                                                                   lout, ksize, stride, pad, dil,
                                                                   rows);
      break;
  }
  return bio_host::launch_status(cudaGetLastError());
}

extern "C" {

int bio_im2col(int32_t dtype, const void* x, const bio_conv_geom* geom, void* patches,
               int64_t kpad, int32_t device, void* stream) {
  if (!geom_ok(geom)) return BIO_ERR_SHAPE;
  const int64_t cg = geom->channels / geom->groups;
  const int64_t k_real = cg * geom->kernel[0] * geom->kernel[1] * geom->kernel[2];
  if (kpad < k_real) return BIO_ERR_SHAPE;
  const int64_t L = geom->out[0] * geom->out[1] * geom->out[2];
  const int64_t total = geom->batch * geom->groups * L * kpad;
  if (total == 0) return BIO_OK;
  if (x == nullptr || patches == nullptr) return BIO_ERR_ARG;
  int st = bio_host::ensure_device(device);
  if (st != BIO_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bio::Geom g = to_geom(geom);
  const int64_t rows = geom->batch * geom->groups * L;
  bool table = kpad <= bio::kIm2colTable && cg * geom->in[0] * geom->in[1] * geom->in[2] <
                                                2147483647;
  for (int i = 0; i < 3; ++i)
    table = table && (geom->kernel[i] - 1) * geom->dilation[i] < 32767;
  if (table) {
    const int kr = static_cast<int>(k_real), kp = static_cast<int>(kpad);
    switch (dtype) {
      case BIO_F32:
        bio::im2col_table_kernel<float><<<blocks_for_rows(rows), 256, 0, s>>>(
            static_cast<const float*>(x), static_cast<float*>(patches), g, kr, kp, rows);
        break;
      case BIO_F16:
        bio::im2col_table_kernel<__half><<<blocks_for_rows(rows), 256, 0, s>>>(
            static_cast<const __half*>(x), static_cast<__half*>(patches), g, kr, kp, rows);
        break;
      case BIO_BF16:
        bio::im2col_table_kernel<__nv_bfloat16><<<blocks_for_rows(rows), 256, 0, s>>>(
            static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(patches), g, kr,
            kp, rows);
        break;
      default: return BIO_ERR_DTYPE;
    }
    return bio_host::launch_status(cudaGetLastError());
  }
  switch (dtype) {
    case BIO_F32:
      bio::im2col_kernel<float><<<blocks_for_rows(rows), 256, 0, s>>>(
          static_cast<const float*>(x), static_cast<float*>(patches), g, k_real, kpad, rows);
      break;
    case BIO_F16:
      bio::im2col_kernel<__half><<<blocks_for_rows(rows), 256, 0, s>>>(
          static_cast<const __half*>(x), static_cast<__half*>(patches), g, k_real, kpad, rows);
      break;
    case BIO_BF16:
      bio::im2col_kernel<__nv_bfloat16><<<blocks_for_rows(rows), 256, 0, s>>>(
          static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(patches), g, k_real,
          kpad, rows);
      break;
    default: return BIO_ERR_DTYPE;
  }
  return bio_host::launch_status(cudaGetLastError());
}

int bio_depthwise_conv1d(int32_t dtype, const void* x, const void* w, const void* bias, void* y,
                         int64_t batch, int64_t channels, int64_t lin, int64_t lout,
                         int32_t ksize, int32_t stride, int32_t padding, int32_t dilation,
                         int32_t device, void* stream) {
  if (batch < 0 || channels < 0 || lin < 0 || lout < 0 || ksize < 1 || stride < 1 ||
      dilation < 1 || padding < 0)
    return BIO_ERR_SHAPE;
  const int64_t total = batch * channels * lout;
  if (total == 0) return BIO_OK;
  if (x == nullptr || w == nullptr || y == nullptr) return BIO_ERR_ARG;
  int st = bio_host::ensure_device(device);
  if (st != BIO_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t rows = batch * channels;
  {
    const int64_t es = dtype == BIO_F32 ? 4 : 2;
    const int64_t smem = 8 * lin * es;
    if (smem <= 48 * 1024 && lout <= 2147483647 &&
        (lout - 1) * static_cast<int64_t>(stride) + static_cast<int64_t>(ksize - 1) * dilation <
            2147483647) {
      const int li = static_cast<int>(lin), lo = static_cast<int>(lout);
      switch (dtype) {
        case BIO_F32:
          st = launch_dw_smem<float>(x, w, bias, y, channels, li, lo, ksize, stride, padding,
                                     dilation, rows, smem, s);
          break;
        case BIO_F16:
          st = launch_dw_smem<__half>(x, w, bias, y, channels, li, lo, ksize, stride, padding,
                                      dilation, rows, smem, s);
          break;
        case BIO_BF16:
          st = launch_dw_smem<__nv_bfloat16>(x, w, bias, y, channels, li, lo, ksize, stride,
                                             padding, dilation, rows, smem, s);
          break;
        default: return BIO_ERR_DTYPE;
      }
      if (st != BIO_OK) return st;
      return bio_host::launch_status(cudaGetLastError());
    }
  }
  switch (dtype) {
    case BIO_F32:
      bio::depthwise_conv1d_kernel<float><<<blocks_for_rows(rows), 256, 0, s>>>(
          static_cast<const float*>(x), static_cast<const float*>(w),
          static_cast<const float*>(bias), static_cast<float*>(y), channels, lin, lout, ksize,
          stride, padding, dilation, rows);
      break;
    case BIO_F16:
      bio::depthwise_conv1d_kernel<__half><<<blocks_for_rows(rows), 256, 0, s>>>(
          static_cast<const __half*>(x), static_cast<const __half*>(w),
          static_cast<const __half*>(bias), static_cast<__half*>(y), channels, lin, lout, ksize,
          stride, padding, dilation, rows);
      break;
    case BIO_BF16:
      bio::depthwise_conv1d_kernel<__nv_bfloat16><<<blocks_for_rows(rows), 256, 0, s>>>(
          static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(w),
          static_cast<const __nv_bfloat16*>(bias), static_cast<__nv_bfloat16*>(y), channels, lin,
          lout, ksize, stride, padding, dilation, rows);
      break;
    default: return BIO_ERR_DTYPE;
  }
  return bio_host::launch_status(cudaGetLastError());
}

int bio_conv_transpose_scatter(int32_t dtype, const void* src, const void* bias, void* dst,
                               const bio_conv_geom* geom, int64_t out_channels_per_group,
                               int32_t device, void* stream) {
  if (!geom_ok(geom) || out_channels_per_group < 1) return BIO_ERR_SHAPE;
  const int64_t out_vol = geom->in[0] * geom->kernel[0] * geom->in[1] * geom->kernel[1] *
                          geom->in[2] * geom->kernel[2];
  const int64_t total = geom->batch * geom->groups * out_channels_per_group * out_vol;
  if (total == 0) return BIO_OK;
  if (src == nullptr || dst == nullptr) return BIO_ERR_ARG;
  int st = bio_host::ensure_device(device);
  if (st != BIO_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bio::Geom g = to_geom(geom);
  const int64_t rows = total / (geom->in[2] * geom->kernel[2]);
  {
    // plane path: the plane's source rows fit in 48 KB of shared memory
    const int64_t es = dtype == BIO_F32 ? 4 : 2;
    const int64_t in_vol = geom->in[0] * geom->in[1] * geom->in[2];
    const int64_t kvol = geom->kernel[0] * geom->kernel[1] * geom->kernel[2];
    // row stride: 16-byte aligned and an odd multiple of 4 words for 2-byte
    // types (k2 rows read by one warp fall in different banks), odd words
    // for fp32
    const int64_t srow = es == 2 ? ((in_vol + 7) / 8 * 8 + ((((in_vol + 7) / 8 * 8) / 8) % 2 == 0 ? 8 : 0))
                                 : in_vol + 1;
    const int64_t planes = geom->batch * geom->groups * out_channels_per_group;
    const int64_t smem = kvol * srow * es;
    if (smem <= 48 * 1024 && planes <= 2147483647 && out_vol <= 2147483647 &&
        out_channels_per_group * geom->groups <= 2147483647) {
      const unsigned grid = static_cast<unsigned>(planes);
      const int og = static_cast<int>(out_channels_per_group);
      const int sr = static_cast<int>(srow);
      switch (dtype) {
        case BIO_F32:
          bio::convt_plane_kernel<float><<<grid, 256, smem, s>>>(
              static_cast<const float*>(src), static_cast<const float*>(bias),
              static_cast<float*>(dst), g, og, sr);
          break;
        case BIO_F16:
          bio::convt_plane_kernel<__half><<<grid, 256, smem, s>>>(
              static_cast<const __half*>(src), static_cast<const __half*>(bias),
              static_cast<__half*>(dst), g, og, sr);
          break;
        case BIO_BF16:
          bio::convt_plane_kernel<__nv_bfloat16><<<grid, 256, smem, s>>>(
              static_cast<const __nv_bfloat16*>(src), static_cast<const __nv_bfloat16*>(bias),
              static_cast<__nv_bfloat16*>(dst), g, og, sr);
          break;
        default: return BIO_ERR_DTYPE;
      }
      return bio_host::launch_status(cudaGetLastError());
    }
  }
  switch (dtype) {
    case BIO_F32:
      bio::convt_scatter_kernel<float><<<blocks_for_rows(rows), 256, 0, s>>>(
          static_cast<const float*>(src), static_cast<const float*>(bias),
          static_cast<float*>(dst), g, out_channels_per_group, rows);
      break;
    case BIO_F16:
      bio::convt_scatter_kernel<__half><<<blocks_for_rows(rows), 256, 0, s>>>(
          static_cast<const __half*>(src), static_cast<const __half*>(bias),
          static_cast<__half*>(dst), g, out_channels_per_group, rows);
      break;
    case BIO_BF16:
      bio::convt_scatter_kernel<__nv_bfloat16><<<blocks_for_rows(rows), 256, 0, s>>>(
          static_cast<const __nv_bfloat16*>(src), static_cast<const __nv_bfloat16*>(bias),
          static_cast<__nv_bfloat16*>(dst), g, out_channels_per_group, rows);
      break;
    default: return BIO_ERR_DTYPE;
  }
  return bio_host::launch_status(cudaGetLastError());
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Convolution without any allocation (bio_conv_nd_noalloc).
//
// The patch matrix (and, when needed, a packed copy of the weight) lives in a
// fixed file-scope device array instead of caller-provided memory.  The array
// is a host-side stand-in in host code: its device address is obtained once
// per device with cudaGetSymbolAddress (with that device current) and passed
// to the kernels.
// ---------------------------------------------------------------------------
namespace {

__device__ __align__(256) unsigned char g_noalloc_scratch[BIO_NOALLOC_SCRATCH_BYTES];

std::mutex g_scratch_mu;
void* g_scratch_addr[bio_host::kMaxDevices] = {nullptr};

// Device address of the scratch array on `device` (which must be current).
int scratch_address(int device, unsigned char** out) {
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (g_scratch_addr[device] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) return BIO_ERR_LAUNCH;
    g_scratch_addr[device] = p;
  }
  *out = static_cast<unsigned char*>(g_scratch_addr[device]);
  return BIO_OK;
}

int64_t dtype_size(int32_t dtype) { return dtype == BIO_F32 ? 4 : 2; }

int64_t round_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

// *acc *= v unless the product leaves [0, 2^62): the scratch bound is the
// only limit on what the kernels write, so no size may wrap.
bool mul_in_range(int64_t* acc, int64_t v) {
  int64_t r = 0;
  if (v < 0 || __builtin_mul_overflow(*acc, v, &r) || r >= (int64_t{1} << 62)) return false;
  *acc = r;
  return true;
}

// The output extent of every spatial dim must be the one the geometry
// implies, (in + 2p - d(k-1) - 1) / s + 1 >= 1, with every field below 2^31
// (so the expression itself cannot overflow).
bool out_dims_consistent(const bio_conv_geom* g) {
  constexpr int64_t kLim = int64_t{1} << 31;
  for (int i = 0; i < 3; ++i) {
    if (g->in[i] >= kLim || g->kernel[i] >= kLim || g->stride[i] >= kLim ||
        g->padding[i] >= kLim || g->dilation[i] >= kLim || g->out[i] >= kLim)
      return false;
    const int64_t span = g->in[i] + 2 * g->padding[i] - g->dilation[i] * (g->kernel[i] - 1) - 1;
    if (span < 0 || span / g->stride[i] + 1 != g->out[i]) return false;
  }
  return true;
}

}  // namespace

extern "C" int bio_conv_nd_noalloc(int32_t dtype, const void* x, const void* weight,
                                   const void* bias, void* y, const bio_conv_geom* geom,
                                   int64_t out_channels, int32_t device, void* stream) {
  if (dtype != BIO_F32 && dtype != BIO_F16 && dtype != BIO_BF16) return BIO_ERR_DTYPE;
  if (!geom_ok(geom) || out_channels < 1 || out_channels % geom->groups != 0)
    return BIO_ERR_SHAPE;
  if (geom->batch == 0) return BIO_OK;
  if (!out_dims_consistent(geom)) return BIO_ERR_SHAPE;
  const int64_t groups = geom->groups;
  const int64_t cg = geom->channels / groups;
  const int64_t og = out_channels / groups;
  const int64_t es = dtype_size(dtype);
  // every size below is checked against wrap-around before it is trusted
  int64_t k = cg;
  int64_t L = 1;
  for (int i = 0; i < 3; ++i)
    if (!mul_in_range(&k, geom->kernel[i]) || !mul_in_range(&L, geom->out[i]))
      return BIO_ERR_SCRATCH;
  const int64_t kpad = round_up(k, 8);
  int64_t patch_raw = geom->batch;
  if (!mul_in_range(&patch_raw, groups) || !mul_in_range(&patch_raw, L) ||
      !mul_in_range(&patch_raw, kpad) || !mul_in_range(&patch_raw, es))
    return BIO_ERR_SCRATCH;
  const int64_t patch_bytes = round_up(patch_raw, 256);
  if (x == nullptr || weight == nullptr || y == nullptr) return BIO_ERR_ARG;
  // the tensor-core GEMM reads the weight with TMA: rows must be 16-byte
  // aligned, otherwise a zero-padded copy goes into the scratch as well
  const bool pack_w = dtype != BIO_F32 &&
                      ((k * es) % 16 != 0 || (reinterpret_cast<uintptr_t>(weight) & 15u) != 0);
  int64_t w_raw = pack_w ? groups : 0;
  if (pack_w && (!mul_in_range(&w_raw, og) || !mul_in_range(&w_raw, kpad) ||
                 !mul_in_range(&w_raw, es)))
    return BIO_ERR_SCRATCH;
  const int64_t w_bytes = round_up(w_raw, 256);
  constexpr int64_t kScratch = static_cast<int64_t>(BIO_NOALLOC_SCRATCH_BYTES);
  if (patch_bytes > kScratch || w_bytes > kScratch - patch_bytes) return BIO_ERR_SCRATCH;
  const int64_t w_row = pack_w ? kpad : k;

  // One GEMM per (sample, group): y[b, g*og + o, l] = W_g[o, :] . patches[b, g, l, :]
  // (+ bias per output channel), the layout of the regular entry point.
  bio_gemm_args g = {};
  g.dtype = dtype;
  g.flags = BIO_GEMM_BIAS_PER_ROW;
  g.batch1 = geom->batch;
  g.batch2 = groups;
  g.m = og;
  g.n = L;
  g.k = k;
  g.a_sm = w_row;
  g.a_sk = 1;
  g.a_s1 = 0;
  g.a_s2 = og * w_row;
  g.a_div2 = 1;
  g.b_sk = 1;
  g.b_sn = kpad;
  g.b_s1 = groups * L * kpad;
  g.b_s2 = L * kpad;
  g.b_div2 = 1;
  g.c = y;
  g.c_sm = L;
  g.c_sn = 1;
  g.c_s1 = out_channels * L;
  g.c_s2 = og * L;
  g.bias = bias;
  g.bias_s2 = og;
  g.alpha = 1.0f;
  g.device = device;
  // fp32 takes the exact-slice tensor-core GEMM whenever it applies, as the
  // regular entry point does (same bits); its digit workspace follows the
  // patches in the array.
  const int64_t ws_bytes = dtype == BIO_F32 ? bio_gemm_f32_exact_workspace(&g) : 0;
  if (ws_bytes > kScratch - patch_bytes - w_bytes) return BIO_ERR_SCRATCH;

  int st = bio_host::ensure_device(device);
  if (st != BIO_OK) return st;
  unsigned char* scratch = nullptr;
  st = scratch_address(device, &scratch);
  if (st != BIO_OK) return st;

  st = bio_im2col(dtype, x, geom, scratch, kpad, device, stream);
  if (st != BIO_OK) return st;
  g.a = weight;
  g.b = scratch;
  if (pack_w) {
    st = bio_pack_rows(dtype, weight, 1, groups, og, k, 0, og * k, k, 1, scratch + patch_bytes,
                       kpad, device, stream);
    if (st != BIO_OK) return st;
    g.a = scratch + patch_bytes;
  }
  if (ws_bytes > 0) return bio_gemm_f32_exact(&g, scratch + patch_bytes + w_bytes, ws_bytes, stream);
  return bio_gemm(&g, stream);
}
