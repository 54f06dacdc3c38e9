// Batch-invariant row kernels: softmax, log-softmax, mean, L2 norm.
//
// The input is a contiguous [outer][n][inner] view reduced over n.
//
// Row mode (inner == 1): a fixed team of threads owns one row.  The team size
// is a function of n only (32, 256 or 1024 threads).  Element i belongs to the
// 8-element group i/8, group g to thread g % team, each thread folds its groups
// in increasing g (elements of a group in order), then a fixed xor-shuffle tree
// combines the warp and, for multi-warp teams, warp 0 combines the per-warp
// partials in warp order.  16-byte vector loads are used when a group is
// aligned; that changes the load instruction, never the order of the sums.
//
// Column mode (inner > 1): one thread owns one output column and folds the n
// elements in increasing order (loads coalesced across columns).
//
// Either way the reduction tree of an output depends on n alone, never on the
// number of rows/columns, so every output is batch invariant.  All arithmetic
// is fp32; the result is rounded once to the output dtype.
//
// Reference: _softmax_kernel / softmax (batch_invariant_ops.py:1075-1145),
// _log_softmax_kernel / log_softmax (:975-1071), mean_kernel / mean_dim
// (:1348-1482), _vector_norm_kernel / linalg_vector_norm_batch_invariant
// (:1486-1597).
#include "bio_common.cuh"

namespace bio {

enum RowOp : int { kSoftmax = 0, kLogSoftmax = 1, kMean = 2, kL2Norm = 3 };

template <typename T>
__device__ __forceinline__ void load_group(const T* __restrict__ row, int64_t g, int64_t n,
                                           float (&v)[8], float fill) {
  const int64_t base = g * 8;
  const T* p = row + base;
  if (base + 8 <= n && (reinterpret_cast<uintptr_t>(p) % 16) == 0 && sizeof(T) == 2) {
    const uint4 w = *reinterpret_cast<const uint4*>(p);
    const T* e = reinterpret_cast<const T*>(&w);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = to_f32(e[j]);
  } else if (base + 8 <= n && (reinterpret_cast<uintptr_t>(p) % 16) == 0 && sizeof(T) == 4) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = (base + j < n) ? to_f32(p[j]) : fill;
  }
}

// Store 8 consecutive outputs of group g: one 16-byte store (two for fp32)
// when the group is complete and aligned, element stores otherwise.
template <typename TO>
__device__ __forceinline__ void store_group(TO* __restrict__ row, int64_t g, int64_t n,
                                            const float (&o)[8]) {
  const int64_t base = g * 8;
  TO* p = row + base;
  if (base + 8 <= n && (reinterpret_cast<uintptr_t>(p) % 16) == 0) {
    if constexpr (sizeof(TO) == 2) {
      uint4 w;
      TO* e = reinterpret_cast<TO*>(&w);
#pragma unroll
      for (int j = 0; j < 8; ++j) e[j] = from_f32<TO>(o[j]);
      *reinterpret_cast<uint4*>(p) = w;
    } else {
      *reinterpret_cast<float4*>(p) = make_float4(o[0], o[1], o[2], o[3]);
      *reinterpret_cast<float4*>(p + 4) = make_float4(o[4], o[5], o[6], o[7]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (base + j < n) p[j] = from_f32<TO>(o[j]);
  }
}

// Loads of kUnroll groups are issued before any of them is folded, so that
// several 16-byte loads per thread are in flight; the fold order (increasing
// g, elements in order) is unchanged.
constexpr int kUnroll = 4;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return __shfl_sync(0xffffffffu, v, 0);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return __shfl_sync(0xffffffffu, v, 0);
}

// Team-wide reduction with a fixed tree.  `scratch` holds TEAM/32 floats per
// team; all threads of the team receive the result of the tree.
template <int TEAM, bool IS_MAX>
__device__ __forceinline__ float team_reduce(float v, float* scratch) {
  v = IS_MAX ? warp_max(v) : warp_sum(v);
  if constexpr (TEAM == 32) {
    return v;
  } else {
    constexpr int W = TEAM / 32;
    const int t = threadIdx.x % TEAM;
    const int w = t >> 5, lane = t & 31;
    __syncthreads();
    if (lane == 0) scratch[w] = v;
    __syncthreads();
    float r;
    if (w == 0) {
      float x = lane < W ? scratch[lane] : (IS_MAX ? -INFINITY : 0.f);
      r = IS_MAX ? warp_max(x) : warp_sum(x);
      if (lane == 0) scratch[W] = r;
    }
    __syncthreads();
    r = scratch[W];
    return r;
  }
}

template <typename TI, typename TO, int OP, int TEAM>
__global__ void __launch_bounds__(TEAM >= 256 ? TEAM : 256)
    row_kernel(const TI* __restrict__ x, TO* __restrict__ y, int64_t rows, int64_t n) {
  constexpr int kTeamsPerBlock = TEAM >= 256 ? 1 : 256 / TEAM;
  // groups in flight per thread: a 1024-thread team has 64 registers a thread,
  // so it takes one at a time (the fold order -- a thread's groups in
  // increasing index -- does not depend on this)
  constexpr int UNR = TEAM >= 1024 ? 1 : kUnroll;
  __shared__ float scratch[kTeamsPerBlock][TEAM / 32 + 1];
  const int team = threadIdx.x / TEAM;
  const int t = threadIdx.x % TEAM;
  const int64_t groups = (n + 7) / 8;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * kTeamsPerBlock + team; r < rows;
       r += static_cast<int64_t>(gridDim.x) * kTeamsPerBlock) {
    const TI* row = x + r * n;
    if constexpr (OP == kMean || OP == kL2Norm) {
      float acc = 0.f;
      for (int64_t g0 = t; g0 < groups; g0 += UNR * TEAM) {
        float v[UNR][8];
#pragma unroll
        for (int u = 0; u < UNR; ++u)
          if (g0 + u * TEAM < groups) load_group(row, g0 + u * TEAM, n, v[u], 0.f);
#pragma unroll
        for (int u = 0; u < UNR; ++u)
          if (g0 + u * TEAM < groups) {
#pragma unroll
            for (int j = 0; j < 8; ++j) acc += (OP == kL2Norm) ? v[u][j] * v[u][j] : v[u][j];
          }
      }
      const float s = team_reduce<TEAM, false>(acc, scratch[team]);
      if (t == 0) {
        const float out = (OP == kMean) ? s / static_cast<float>(n) : sqrtf(s);
        y[r] = from_f32<TO>(out);
      }
    } else {
      float mx = -INFINITY;
      for (int64_t g0 = t; g0 < groups; g0 += UNR * TEAM) {
        float v[UNR][8];
#pragma unroll
        for (int u = 0; u < UNR; ++u)
          if (g0 + u * TEAM < groups) load_group(row, g0 + u * TEAM, n, v[u], -INFINITY);
#pragma unroll
        for (int u = 0; u < UNR; ++u)
          if (g0 + u * TEAM < groups) {
#pragma unroll
            for (int j = 0; j < 8; ++j) mx = fmaxf(mx, v[u][j]);
          }
      }
      mx = team_reduce<TEAM, true>(mx, scratch[team]);
      float den = 0.f;
      for (int64_t g0 = t; g0 < groups; g0 += UNR * TEAM) {
        float v[UNR][8];
#pragma unroll
        for (int u = 0; u < UNR; ++u)
          if (g0 + u * TEAM < groups) load_group(row, g0 + u * TEAM, n, v[u], -INFINITY);
#pragma unroll
        for (int u = 0; u < UNR; ++u) {
          const int64_t g = g0 + u * TEAM;
          if (g < groups) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              if (g * 8 + j < n) {
                if constexpr (OP == kSoftmax)
                  den += (mx == -INFINITY) ? 0.f : __expf(v[u][j] - mx);
                else
                  den += __expf(v[u][j] - mx);
              }
            }
          }
        }
      }
      den = team_reduce<TEAM, false>(den, scratch[team]);
      TO* out = y + r * n;
      const float inv = den != 0.f ? 1.f / den : 0.f;
      const float lse = (OP == kLogSoftmax) ? logf(den) : 0.f;
      for (int64_t g0 = t; g0 < groups; g0 += UNR * TEAM) {
        float v[UNR][8];
#pragma unroll
        for (int u = 0; u < UNR; ++u)
          if (g0 + u * TEAM < groups) load_group(row, g0 + u * TEAM, n, v[u], -INFINITY);
#pragma unroll
        for (int u = 0; u < UNR; ++u) {
          const int64_t g = g0 + u * TEAM;
          if (g < groups) {
            float o[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              if constexpr (OP == kSoftmax)
                o[j] = ((mx == -INFINITY) ? 0.f : __expf(v[u][j] - mx)) * inv;
              else
                o[j] = v[u][j] - mx - lse;
            }
            store_group(out, g, n, o);
          }
        }
      }
    }
  }
}

// Register-resident softmax / log-softmax for rows of up to TEAM * 8 * RMAX
// elements (RMAX groups of 8 per thread, the smallest power of two that holds
// the row): the row is read from HBM once and written once.  The element to
// thread assignment (8-element group g -> thread g % TEAM) and the reduction
// tree are the same as in row_kernel, so results do not depend on which of the
// two kernels a row length selects.
template <typename TI, typename TO, bool LOG, int TEAM, int RMAX>
__global__ void __launch_bounds__(TEAM >= 128 ? TEAM : 256)
    row_softmax_reg_kernel(const TI* __restrict__ x, TO* __restrict__ y, int64_t rows, int64_t n) {
  constexpr int kTeamsPerBlock = TEAM >= 128 ? 1 : 256 / TEAM;
  __shared__ float scratch[kTeamsPerBlock][TEAM / 32 + 1];
  const int team = threadIdx.x / TEAM;
  const int t = threadIdx.x % TEAM;
  const int64_t groups = (n + 7) / 8;
  // Rows are software-pipelined: the next row's groups are loaded into
  // registers before the current row's reductions, so their latency overlaps
  // the current row's work.
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kTeamsPerBlock;
  auto load_row = [&](int64_t r, float (&v)[RMAX][8]) {
    const TI* row = x + r * n;
#pragma unroll
    for (int q = 0; q < RMAX; ++q) {
      const int64_t g = t + static_cast<int64_t>(q) * TEAM;
      if (g < groups) {
        load_group(row, g, n, v[q], -INFINITY);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[q][j] = -INFINITY;
      }
    }
  };
  int64_t r = static_cast<int64_t>(blockIdx.x) * kTeamsPerBlock + team;
  float v[RMAX][8];
  if (r < rows) load_row(r, v);
  for (; r < rows; r += stride) {
    float nv[RMAX][8];
    if (r + stride < rows) load_row(r + stride, nv);
    float mx = -INFINITY;
#pragma unroll
    for (int q = 0; q < RMAX; ++q)
#pragma unroll
      for (int j = 0; j < 8; ++j) mx = fmaxf(mx, v[q][j]);
    mx = team_reduce<TEAM, true>(mx, scratch[team]);
    float den = 0.f;
#pragma unroll
    for (int q = 0; q < RMAX; ++q) {
      const int64_t g = t + static_cast<int64_t>(q) * TEAM;
      if (g < groups) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (g * 8 + j < n) {
            float e;
            if (LOG)
              e = __expf(v[q][j] - mx);
            else
              e = (mx == -INFINITY) ? 0.f : __expf(v[q][j] - mx);
            den += e;
            if (!LOG) v[q][j] = e;
          }
        }
      }
    }
    den = team_reduce<TEAM, false>(den, scratch[team]);
    TO* out = y + r * n;
    const float lse = LOG ? logf(den) : 0.f;
    const float inv = den != 0.f ? 1.f / den : 0.f;
#pragma unroll
    for (int q = 0; q < RMAX; ++q) {
      const int64_t g = t + static_cast<int64_t>(q) * TEAM;
      if (g < groups) {
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = LOG ? (v[q][j] - mx - lse) : v[q][j] * inv;
        store_group(out, g, n, o);
      }
    }
#pragma unroll
    for (int q = 0; q < RMAX; ++q)
#pragma unroll
      for (int j = 0; j < 8; ++j) v[q][j] = nv[q][j];
  }
}

// Fast path of row_softmax_reg_kernel for rows made of whole, 16-byte
// aligned groups (n % 8 == 0, aligned bases): no per-element bounds tests,
// 32-bit indices, exponentials as ex2(x * log2e - max * log2e) with one FFMA.
// Same element-to-thread assignment and reduction trees as the general
// kernels; the next row is prefetched into registers before the current
// row's reductions.
template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]) {
  if constexpr (sizeof(T) == 2) {
    const uint4 w = *reinterpret_cast<const uint4*>(p);
    const T* e = reinterpret_cast<const T*>(&w);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = to_f32(e[j]);
  } else {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
}

template <typename T>
__device__ __forceinline__ void store8(T* p, const float (&o)[8]) {
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
}

__device__ __forceinline__ float ex2f_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename TI, typename TO, bool LOG, int TEAM, int RMAX>
__global__ void __launch_bounds__(TEAM >= 128 ? TEAM : 256)
    row_softmax_fast_kernel(const TI* __restrict__ x, TO* __restrict__ y, int64_t rows, int n) {
  constexpr int kTeamsPerBlock = TEAM >= 128 ? 1 : 256 / TEAM;
  __shared__ float scratch[kTeamsPerBlock][TEAM / 32 + 1];
  const int team = threadIdx.x / TEAM;
  const int t = threadIdx.x % TEAM;
  const int groups = n >> 3;
  const float kLog2e = 1.4426950408889634f;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kTeamsPerBlock;
  auto load_row = [&](int64_t r, float (&v)[RMAX][8]) {
    const TI* row = x + r * n;
#pragma unroll
    for (int q = 0; q < RMAX; ++q) {
      const int g = t + q * TEAM;
      if (g < groups) {
        load8(row + g * 8, v[q]);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[q][j] = -INFINITY;
      }
    }
  };
  int64_t r = static_cast<int64_t>(blockIdx.x) * kTeamsPerBlock + team;
  float v[RMAX][8];
  if (r < rows) load_row(r, v);
  for (; r < rows; r += stride) {
    float nv[RMAX][8];
    if (r + stride < rows) load_row(r + stride, nv);
    float mx = -INFINITY;
#pragma unroll
    for (int q = 0; q < RMAX; ++q)
#pragma unroll
      for (int j = 0; j < 8; ++j) mx = fmaxf(mx, v[q][j]);
    mx = team_reduce<TEAM, true>(mx, scratch[team]);
    const float ml = (!LOG && mx == -INFINITY) ? 0.f : mx * kLog2e;
    float den = 0.f;
#pragma unroll
    for (int q = 0; q < RMAX; ++q) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float e = ex2f_approx(fmaf(v[q][j], kLog2e, -ml));
        den += e;  // groups past the row end hold -inf: e = 0
        if (!LOG) v[q][j] = e;
      }
    }
    den = team_reduce<TEAM, false>(den, scratch[team]);
    TO* out = y + r * n;
    const float lse = LOG ? logf(den) : 0.f;
    const float inv = den != 0.f ? 1.f / den : 0.f;
#pragma unroll
    for (int q = 0; q < RMAX; ++q) {
      const int g = t + q * TEAM;
      if (g < groups) {
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = LOG ? (v[q][j] - mx - lse) : v[q][j] * inv;
        store8(out + g * 8, o);
      }
    }
#pragma unroll
    for (int q = 0; q < RMAX; ++q)
#pragma unroll
      for (int j = 0; j < 8; ++j) v[q][j] = nv[q][j];
  }
}

// Softmax / log-softmax of long rows (vocabulary-sized) by a cluster of CS
// CTAs of kClusterTeam threads per row.  CTA c of the cluster owns the
// contiguous groups [c*gpc, (c+1)*gpc) (gpc = ceil(groups / CS)) and keeps them
// in registers: thread t holds local groups t, t + kClusterTeam, ... (at most
// RMAX).  The row maximum and the sum of exponentials are combined across the
// cluster through distributed shared memory: every CTA writes its partial into
// slot c of every CTA, and after the cluster barrier each CTA folds the CS
// slots in increasing c.  CS, gpc and the trees depend on n only.
constexpr int kClusterTeam = 512;

// RAW (16-bit input, n % 8 == 0, 16-byte aligned rows): the groups stay in
// registers as their raw 16-byte words (half the registers of floats, two
// CTAs per SM) and are widened at each use; softmax recomputes the same
// exponential for the output instead of keeping it.  Every value computed is
// the one the float form computes, so the two forms give the same bits.
template <typename TI, typename TO, bool LOG, int CS, int RMAX>
__global__ void __launch_bounds__(kClusterTeam, 2)
    row_softmax_cluster_raw_kernel(const TI* __restrict__ x, TO* __restrict__ y, int64_t n) {
  constexpr int TEAM = kClusterTeam;
  __shared__ float scratch[TEAM / 32 + 1];
  __shared__ float part_max[CS];
  __shared__ float part_sum[CS];
  const int t = threadIdx.x;
  const uint32_t rank = cluster_ctarank();
  const int64_t r = blockIdx.x / CS;
  // rows are at most kMaxClusterRow long: group indices fit in int
  const int groups = static_cast<int>(n / 8);
  const int gpc = (groups + CS - 1) / CS;
  const int g_lo = static_cast<int>(rank) * gpc;
  const int cnt = min(gpc, groups - g_lo);  // groups of this CTA
  const uint4* row = reinterpret_cast<const uint4*>(x + r * n) + g_lo;
  uint4 w[RMAX];
  float mx = -INFINITY;
#pragma unroll
  for (int q = 0; q < RMAX; ++q)
    if (t + q * TEAM < cnt) w[q] = row[t + q * TEAM];
#pragma unroll
  for (int q = 0; q < RMAX; ++q) {
    if (t + q * TEAM < cnt) {
      const TI* e = reinterpret_cast<const TI*>(&w[q]);
#pragma unroll
      for (int j = 0; j < 8; ++j) mx = fmaxf(mx, to_f32(e[j]));
    }
  }
  mx = team_reduce<TEAM, true>(mx, scratch);
  if (t < CS) {
    const uint32_t dst = mapa_shared(static_cast<uint32_t>(__cvta_generic_to_shared(&part_max[rank])),
                                     static_cast<uint32_t>(t));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(dst), "f"(mx) : "memory");
  }
  cluster_sync_all();
  mx = part_max[0];
#pragma unroll
  for (int c = 1; c < CS; ++c) mx = fmaxf(mx, part_max[c]);
  float den = 0.f;
#pragma unroll
  for (int q = 0; q < RMAX; ++q) {
    if (t + q * TEAM < cnt) {
      const TI* e = reinterpret_cast<const TI*>(&w[q]);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (LOG)
          den += __expf(to_f32(e[j]) - mx);
        else
          den += (mx == -INFINITY) ? 0.f : __expf(to_f32(e[j]) - mx);
      }
    }
  }
  den = team_reduce<TEAM, false>(den, scratch);
  if (t < CS) {
    const uint32_t dst = mapa_shared(static_cast<uint32_t>(__cvta_generic_to_shared(&part_sum[rank])),
                                     static_cast<uint32_t>(t));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(dst), "f"(den) : "memory");
  }
  cluster_sync_all();
  den = part_sum[0];
#pragma unroll
  for (int c = 1; c < CS; ++c) den += part_sum[c];
  TO* out = y + r * n + static_cast<int64_t>(g_lo) * 8;
  const float lse = LOG ? logf(den) : 0.f;
  const float inv = den != 0.f ? 1.f / den : 0.f;
#pragma unroll
  for (int q = 0; q < RMAX; ++q) {
    const int gl = t + q * TEAM;
    if (gl < cnt) {
      const TI* e = reinterpret_cast<const TI*>(&w[q]);
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float v = to_f32(e[j]);
        if (LOG)
          o[j] = v - mx - lse;
        else
          o[j] = ((mx == -INFINITY) ? 0.f : __expf(v - mx)) * inv;
      }
      store_group(out, gl, n - static_cast<int64_t>(g_lo) * 8, o);
    }
  }
}

template <typename TI, typename TO, bool LOG, int CS, int RMAX>
__global__ void __launch_bounds__(kClusterTeam)
    row_softmax_cluster_kernel(const TI* __restrict__ x, TO* __restrict__ y, int64_t n) {
  constexpr int TEAM = kClusterTeam;
  __shared__ float scratch[TEAM / 32 + 1];
  __shared__ float part_max[CS];
  __shared__ float part_sum[CS];
  const int t = threadIdx.x;
  const uint32_t rank = cluster_ctarank();
  const int64_t r = blockIdx.x / CS;
  const int64_t groups = (n + 7) / 8;
  const int64_t gpc = (groups + CS - 1) / CS;
  const int64_t g_lo = static_cast<int64_t>(rank) * gpc;
  const int64_t g_hi = g_lo + gpc < groups ? g_lo + gpc : groups;
  const TI* row = x + r * n;
  float v[RMAX][8];
  float mx = -INFINITY;
#pragma unroll
  for (int q = 0; q < RMAX; ++q) {
    const int64_t g = g_lo + t + static_cast<int64_t>(q) * TEAM;
    if (g < g_hi) {
      load_group(row, g, n, v[q], -INFINITY);
#pragma unroll
      for (int j = 0; j < 8; ++j) mx = fmaxf(mx, v[q][j]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[q][j] = -INFINITY;
    }
  }
  mx = team_reduce<TEAM, true>(mx, scratch);
  if (t < CS) {
    const uint32_t dst = mapa_shared(static_cast<uint32_t>(__cvta_generic_to_shared(&part_max[rank])),
                                     static_cast<uint32_t>(t));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(dst), "f"(mx) : "memory");
  }
  cluster_sync_all();
  mx = part_max[0];
#pragma unroll
  for (int c = 1; c < CS; ++c) mx = fmaxf(mx, part_max[c]);
  float den = 0.f;
#pragma unroll
  for (int q = 0; q < RMAX; ++q) {
    const int64_t g = g_lo + t + static_cast<int64_t>(q) * TEAM;
    if (g < g_hi) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (g * 8 + j < n) {
          float e;
          if (LOG)
            e = __expf(v[q][j] - mx);
          else
            e = (mx == -INFINITY) ? 0.f : __expf(v[q][j] - mx);
          den += e;
          if (!LOG) v[q][j] = e;
        }
      }
    }
  }
  den = team_reduce<TEAM, false>(den, scratch);
  if (t < CS) {
    const uint32_t dst = mapa_shared(static_cast<uint32_t>(__cvta_generic_to_shared(&part_sum[rank])),
                                     static_cast<uint32_t>(t));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(dst), "f"(den) : "memory");
  }
  cluster_sync_all();
  den = part_sum[0];
#pragma unroll
  for (int c = 1; c < CS; ++c) den += part_sum[c];
  TO* out = y + r * n;
  const float lse = LOG ? logf(den) : 0.f;
  const float inv = den != 0.f ? 1.f / den : 0.f;
#pragma unroll
  for (int q = 0; q < RMAX; ++q) {
    const int64_t g = g_lo + t + static_cast<int64_t>(q) * TEAM;
    if (g < g_hi) {
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = LOG ? (v[q][j] - mx - lse) : v[q][j] * inv;
      store_group(out, g, n, o);
    }
  }
}

// Column mode: one thread per (outer, inner) column, sequential over n.
template <typename TI, typename TO, int OP>
__global__ void __launch_bounds__(256)
    col_kernel(const TI* __restrict__ x, TO* __restrict__ y, int64_t outer, int64_t n,
               int64_t inner) {
  const int64_t cols = outer * inner;
  for (int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < cols;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t o = c / inner, i = c - o * inner;
    const TI* base = x + o * n * inner + i;
    if constexpr (OP == kMean || OP == kL2Norm) {
      float acc = 0.f;
#pragma unroll 8
      for (int64_t j = 0; j < n; ++j) {
        const float v = to_f32(base[j * inner]);
        acc += (OP == kL2Norm) ? v * v : v;
      }
      y[c] = from_f32<TO>((OP == kMean) ? acc / static_cast<float>(n) : sqrtf(acc));
    } else {
      float mx = -INFINITY;
      for (int64_t j = 0; j < n; ++j) mx = fmaxf(mx, to_f32(base[j * inner]));
      float den = 0.f;
      for (int64_t j = 0; j < n; ++j) {
        const float v = to_f32(base[j * inner]);
        if constexpr (OP == kSoftmax)
          den += (mx == -INFINITY) ? 0.f : __expf(v - mx);
        else
          den += __expf(v - mx);
      }
      TO* out = y + o * n * inner + i;
      if constexpr (OP == kSoftmax) {
        const float inv = den != 0.f ? 1.f / den : 0.f;
        for (int64_t j = 0; j < n; ++j) {
          const float v = to_f32(base[j * inner]);
          const float e = (mx == -INFINITY) ? 0.f : __expf(v - mx);
          out[j * inner] = from_f32<TO>(e * inv);
        }
      } else {
        const float lse = logf(den);
        for (int64_t j = 0; j < n; ++j) out[j * inner] = from_f32<TO>(to_f32(base[j * inner]) - mx - lse);
      }
    }
  }
}


// Column mode, vectorised: one thread owns 8 adjacent columns (16-byte loads
// for 2-byte types) and keeps 8 independent running values, each folded over
// n in increasing order exactly as col_kernel folds a single column.
template <typename TI, typename TO, int OP>
__global__ void __launch_bounds__(256)
    col_kernel_vec8(const TI* __restrict__ x, TO* __restrict__ y, int64_t outer, int64_t n,
                    int64_t inner) {
  static_assert(sizeof(TI) == 2, "vector path is for 2-byte inputs");
  const int64_t vecs = outer * (inner / 8);
  for (int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < vecs;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t o = c / (inner / 8), i0 = (c - o * (inner / 8)) * 8;
    const TI* base = x + o * n * inner + i0;
    float acc[8];
    if constexpr (OP == kMean || OP == kL2Norm) {
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] = 0.f;
#pragma unroll 8
      for (int64_t j = 0; j < n; ++j) {
        const uint4 w = *reinterpret_cast<const uint4*>(base + j * inner);
        const TI* e = reinterpret_cast<const TI*>(&w);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float v = to_f32(e[k]);
          acc[k] += (OP == kL2Norm) ? v * v : v;
        }
      }
      TO* out = y + o * inner + i0;
#pragma unroll
      for (int k = 0; k < 8; ++k)
        out[k] = from_f32<TO>((OP == kMean) ? acc[k] / static_cast<float>(n) : sqrtf(acc[k]));
    } else {
      float mx[8], den[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        mx[k] = -INFINITY;
        den[k] = 0.f;
      }
#pragma unroll 8
      for (int64_t j = 0; j < n; ++j) {
        const uint4 w = *reinterpret_cast<const uint4*>(base + j * inner);
        const TI* e = reinterpret_cast<const TI*>(&w);
#pragma unroll
        for (int k = 0; k < 8; ++k) mx[k] = fmaxf(mx[k], to_f32(e[k]));
      }
#pragma unroll 8
      for (int64_t j = 0; j < n; ++j) {
        const uint4 w = *reinterpret_cast<const uint4*>(base + j * inner);
        const TI* e = reinterpret_cast<const TI*>(&w);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float v = to_f32(e[k]);
          if constexpr (OP == kSoftmax)
            den[k] += (mx[k] == -INFINITY) ? 0.f : __expf(v - mx[k]);
          else
            den[k] += __expf(v - mx[k]);
        }
      }
      TO* out = y + o * n * inner + i0;
#pragma unroll 8
      for (int64_t j = 0; j < n; ++j) {
        const uint4 w = *reinterpret_cast<const uint4*>(base + j * inner);
        const TI* e = reinterpret_cast<const TI*>(&w);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float v = to_f32(e[k]);
          float r;
          if constexpr (OP == kSoftmax) {
            const float inv = den[k] != 0.f ? 1.f / den[k] : 0.f;
            r = ((mx[k] == -INFINITY) ? 0.f : __expf(v - mx[k])) * inv;
          } else {
            r = v - mx[k] - logf(den[k]);
          }
          out[j * inner + k] = from_f32<TO>(r);
        }
      }
    }
  }
}

}  // namespace bio

namespace {

// Team size of row mode: a function of the row length only.
int team_for(int64_t n) {
  if (n <= 2048) return 32;
  if (n <= 32768) return 256;
  return 1024;
}

// Rows of (16384, kMaxClusterRow] elements: cluster softmax, CS CTAs per row.
constexpr int kMaxClusterRow = 8 * bio::kClusterTeam * 8 * 8;

template <typename TI, typename TO, bool LOG, int CS, int RMAX>
int launch_cluster_case(const TI* x, TO* y, int64_t rows, int64_t n, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(rows * CS));
  cfg.blockDim = dim3(bio::kClusterTeam);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CS;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if constexpr (sizeof(TI) == 2) {
    if (n % 8 == 0 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0)
      return bio_host::launch_status(cudaLaunchKernelEx(
          &cfg, bio::row_softmax_cluster_raw_kernel<TI, TO, LOG, CS, RMAX>, x, y, n));
  }
  return bio_host::launch_status(
      cudaLaunchKernelEx(&cfg, bio::row_softmax_cluster_kernel<TI, TO, LOG, CS, RMAX>, x, y, n));
}

template <typename TI, typename TO, bool LOG>
int launch_cluster_softmax(const TI* x, TO* y, int64_t rows, int64_t n, cudaStream_t stream) {
  const int cs = n <= 4 * 16384 ? 2 : (n <= 8 * 16384 ? 4 : 8);
  const int64_t groups = (n + 7) / 8;
  const int64_t gpc = (groups + cs - 1) / cs;
  const int64_t per = (gpc + bio::kClusterTeam - 1) / bio::kClusterTeam;
  const int rmax = per <= 1 ? 1 : (per <= 2 ? 2 : (per <= 4 ? 4 : 8));
#define BIO_CL_CASE(C, R) \
  if (cs == C && rmax == R) return launch_cluster_case<TI, TO, LOG, C, R>(x, y, rows, n, stream);
  BIO_CL_CASE(2, 4)
  BIO_CL_CASE(2, 8)
  BIO_CL_CASE(4, 8)
  BIO_CL_CASE(8, 8)
#undef BIO_CL_CASE
  return BIO_ERR_ARG;
}

template <typename TI, typename TO, int OP>
int launch_rows(const void* x, void* y, int64_t outer, int64_t n, int64_t inner,
                cudaStream_t stream, int sms) {
  const TI* xi = static_cast<const TI*>(x);
  TO* yo = static_cast<TO*>(y);
  if (inner == 1) {
    const int team = team_for(n);
    const int64_t per_block = team >= 256 ? 1 : 256 / team;
    int64_t blocks = (outer + per_block - 1) / per_block;
    const int64_t cap = static_cast<int64_t>(sms) * 64;
    if (blocks > cap) blocks = cap;
    const unsigned g = static_cast<unsigned>(blocks);
    if ((OP == bio::kSoftmax || OP == bio::kLogSoftmax) && n <= 256 * 64) {
      // register-resident rows: one warp (n <= 2048) or one 256-thread CTA
      // per row; the team is a function of n
      const int steam = n <= 2048 ? 32 : 256;
      constexpr bool kLog = OP == bio::kLogSoftmax;
      const int64_t per = (n + 8 * steam - 1) / (8 * steam);  // groups per thread
      const int rmax = per <= 1 ? 1 : (per <= 2 ? 2 : (per <= 4 ? 4 : 8));
      const int threads = steam >= 128 ? steam : 256;
      const int64_t rows_per_block = steam >= 128 ? 1 : 256 / steam;
      int64_t sblocks = (outer + rows_per_block - 1) / rows_per_block;
      const int64_t scap = static_cast<int64_t>(sms) * (2048 / threads) * 8;
      if (sblocks > scap) sblocks = scap;
      const unsigned sg = static_cast<unsigned>(sblocks);
      const bool fast = (n % 8) == 0 && n <= 2147483647 &&
                        (reinterpret_cast<uintptr_t>(x) & 15u) == 0 &&
                        (reinterpret_cast<uintptr_t>(y) & 15u) == 0 &&
                        ((n * static_cast<int64_t>(sizeof(TI))) % 16) == 0 &&
                        ((n * static_cast<int64_t>(sizeof(TO))) % 16) == 0;
#define BIO_FAST_CASE(TM, R)                                                                   \
  if (fast && steam == TM && rmax == R) {                                                      \
    bio::row_softmax_fast_kernel<TI, TO, kLog, TM, R><<<sg, threads, 0, stream>>>(            \
        xi, yo, outer, static_cast<int>(n));                                                   \
    return bio_host::launch_status(cudaGetLastError());                                        \
  }
      BIO_FAST_CASE(32, 1)
      BIO_FAST_CASE(32, 2)
      BIO_FAST_CASE(32, 4)
      BIO_FAST_CASE(32, 8)
      BIO_FAST_CASE(256, 2)
      BIO_FAST_CASE(256, 4)
      BIO_FAST_CASE(256, 8)
#undef BIO_FAST_CASE
#define BIO_REG_CASE(TM, R)                                                                   \
  if (steam == TM && rmax == R) {                                                             \
    bio::row_softmax_reg_kernel<TI, TO, kLog, TM, R><<<sg, threads, 0, stream>>>(xi, yo, outer, \
                                                                                 n);          \
    return bio_host::launch_status(cudaGetLastError());                                       \
  }
      BIO_REG_CASE(32, 1)
      BIO_REG_CASE(32, 2)
      BIO_REG_CASE(32, 4)
      BIO_REG_CASE(32, 8)
      BIO_REG_CASE(256, 1)
      BIO_REG_CASE(256, 2)
      BIO_REG_CASE(256, 4)
      BIO_REG_CASE(256, 8)
#undef BIO_REG_CASE
    }
    if ((OP == bio::kSoftmax || OP == bio::kLogSoftmax) && n > 256 * 64 &&
        n <= static_cast<int64_t>(kMaxClusterRow) && outer <= (int64_t{1} << 27)) {
      return launch_cluster_softmax<TI, TO, OP == bio::kLogSoftmax>(xi, yo, outer, n, stream);
    }
    switch (team) {
      case 32: bio::row_kernel<TI, TO, OP, 32><<<g, 256, 0, stream>>>(xi, yo, outer, n); break;
      case 256: bio::row_kernel<TI, TO, OP, 256><<<g, 256, 0, stream>>>(xi, yo, outer, n); break;
      default: bio::row_kernel<TI, TO, OP, 1024><<<g, 1024, 0, stream>>>(xi, yo, outer, n); break;
    }
  } else {
    if constexpr (sizeof(TI) == 2) {
      if (inner % 8 == 0 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0) {
        const int64_t vecs = outer * (inner / 8);
        int64_t blocks = (vecs + 255) / 256;
        const int64_t cap = static_cast<int64_t>(sms) * 64;
        if (blocks > cap) blocks = cap;
        bio::col_kernel_vec8<TI, TO, OP><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
            xi, yo, outer, n, inner);
        return bio_host::launch_status(cudaGetLastError());
      }
    }
    const int64_t cols = outer * inner;
    int64_t blocks = (cols + 255) / 256;
    const int64_t cap = static_cast<int64_t>(sms) * 64;
    if (blocks > cap) blocks = cap;
    bio::col_kernel<TI, TO, OP><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(xi, yo, outer,
                                                                                  n, inner);
  }
  return bio_host::launch_status(cudaGetLastError());
}

template <int OP, typename TI>
int dispatch_out(int dtype_out, const void* x, void* y, int64_t outer, int64_t n, int64_t inner,
                 cudaStream_t s, int sms) {
  switch (dtype_out) {
    case BIO_F32: return launch_rows<TI, float, OP>(x, y, outer, n, inner, s, sms);
    case BIO_F16: return launch_rows<TI, __half, OP>(x, y, outer, n, inner, s, sms);
    case BIO_BF16: return launch_rows<TI, __nv_bfloat16, OP>(x, y, outer, n, inner, s, sms);
    default: return BIO_ERR_DTYPE;
  }
}

template <int OP>
int dispatch(int dtype_in, int dtype_out, const void* x, void* y, int64_t outer, int64_t n,
             int64_t inner, cudaStream_t s, int sms) {
  switch (dtype_in) {
    case BIO_F32: return dispatch_out<OP, float>(dtype_out, x, y, outer, n, inner, s, sms);
    case BIO_F16: return dispatch_out<OP, __half>(dtype_out, x, y, outer, n, inner, s, sms);
    case BIO_BF16: return dispatch_out<OP, __nv_bfloat16>(dtype_out, x, y, outer, n, inner, s, sms);
    default: return BIO_ERR_DTYPE;
  }
}

int check_common(const void* x, void* y, int64_t outer, int64_t n, int64_t inner, int device) {
  if (outer < 0 || n < 0 || inner < 0) return BIO_ERR_SHAPE;
  if (outer * inner == 0) return BIO_OK;
  if (x == nullptr || y == nullptr) return BIO_ERR_ARG;
  return bio_host::ensure_device(device);
}

}  // namespace

extern "C" {

int bio_softmax(int32_t dtype_in, int32_t dtype_out, const void* x, void* y, int64_t outer,
                int64_t n, int64_t inner, int32_t log_softmax, int32_t device, void* stream) {
  int st = check_common(x, y, outer, n, inner, device);
  if (st != BIO_OK || outer * inner == 0 || n == 0) return st;
  const int sms = bio_host::sm_count(device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (log_softmax) {
    // same dtype, or fp32 out (aten::_log_softmax with half_to_float)
    if (dtype_out != dtype_in && dtype_out != BIO_F32) return BIO_ERR_DTYPE;
    return dispatch<bio::kLogSoftmax>(dtype_in, dtype_out, x, y, outer, n, inner, s, sms);
  }
  return dispatch<bio::kSoftmax>(dtype_in, dtype_out, x, y, outer, n, inner, s, sms);
}

int bio_reduce(int32_t kind, int32_t dtype_in, int32_t dtype_out, const void* x, void* y,
               int64_t outer, int64_t n, int64_t inner, int32_t device, void* stream) {
  int st = check_common(x, y, outer, n, inner, device);
  if (st != BIO_OK || outer * inner == 0) return st;
  const int sms = bio_host::sm_count(device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (kind) {
    case BIO_REDUCE_MEAN:
      return dispatch<bio::kMean>(dtype_in, dtype_out, x, y, outer, n, inner, s, sms);
    case BIO_REDUCE_L2NORM:
      return dispatch<bio::kL2Norm>(dtype_in, dtype_out, x, y, outer, n, inner, s, sms);
    default: return BIO_ERR_ARG;
  }
}

}  // extern "C"
