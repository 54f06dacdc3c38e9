// Deterministic token-choice MoE pieces that sit between the expert GEMMs.
//
// * bio_silu_mul: act = silu(gate) * up, elementwise, with the rounding steps
//   of the reference's stock ops (silu result rounded to the dtype, then the
//   product rounded).
// * bio_moe_route_sum: out[t] = sum over slots j = 0..k-1, left to right, of
//   y[sel[t, j], t, :] * w[t, j]; every product and every partial sum is
//   rounded to the dtype like the reference's gather / multiply / add chain.
//   No atomics: one thread owns one (token, column) output.  Expert indices
//   outside [0, E) raise BIO_DEV_INDEX in the status word (instead of the
//   reference's device-side assert) and zero that output row.
//
// Reference: batch_invariant_ops/moe.py:67-92.
#include "bio_common.cuh"

namespace bio {

template <typename T>
__global__ void silu_mul_kernel(const T* __restrict__ gate, const T* __restrict__ up,
                                T* __restrict__ out, int64_t total) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float g = to_f32(gate[i]);
    const float s = round_to<T>(g / (1.f + expf(-g)));
    out[i] = from_f32<T>(s * to_f32(up[i]));
  }
}

// Same arithmetic, 16 bytes of elements per thread (aligned, n % V == 0).
template <typename T>
__global__ void silu_mul_vec_kernel(const T* __restrict__ gate, const T* __restrict__ up,
                                    T* __restrict__ out, int64_t nvec) {
  constexpr int V = 16 / sizeof(T);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < nvec;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    T g[V], u[V], o[V];
    *reinterpret_cast<uint4*>(g) = reinterpret_cast<const uint4*>(gate)[i];
    *reinterpret_cast<uint4*>(u) = reinterpret_cast<const uint4*>(up)[i];
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const float x = to_f32(g[j]);
      const float sv = round_to<T>(x / (1.f + expf(-x)));
      o[j] = from_f32<T>(sv * to_f32(u[j]));
    }
    reinterpret_cast<uint4*>(out)[i] = *reinterpret_cast<const uint4*>(o);
  }
}

template <typename T, typename WT>
__global__ void route_sum_kernel(const T* __restrict__ y, const WT* __restrict__ w,
                                 const int64_t* __restrict__ sel, T* __restrict__ out,
                                 int64_t experts, int64_t tokens, int64_t top_k, int64_t hidden,
                                 int* status) {
  const int64_t total = tokens * hidden;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / hidden, c = i - t * hidden;
    bool ok = true;
    float acc = 0.f;
    for (int64_t j = 0; j < top_k; ++j) {
      const int64_t e = sel[t * top_k + j];
      if (e < 0 || e >= experts) {
        ok = false;
        break;
      }
      const float wt = round_to<T>(to_f32(w[t * top_k + j]));
      const float r = round_to<T>(to_f32(y[(e * tokens + t) * hidden + c]) * wt);
      acc = (j == 0) ? r : round_to<T>(acc + r);
    }
    if (!ok) {
      if (c == 0) raise_status(status, BIO_DEV_INDEX);
      acc = 0.f;
    }
    out[i] = from_f32<T>(acc);
  }
}

// ---------------------------------------------------------------- sparse path
// Route plan: the slots (t, j) of a [tokens, top_k] selection sorted by
// expert, stably (ascending slot index within an expert), by a counting sort
// with no atomics on positions:
//   1. count: block b histograms its kPlanChunk (256) slots per expert (shared
//      atomics: counts do not depend on their order)
//   2. scan:  per expert, exclusive prefix over blocks, then over experts ->
//      seg[e] and each (block, expert) start position
//   3. place: one warp per block walks its slots in order, 32 at a time;
//      lanes with the same expert rank themselves with __match_any_sync
// Outputs (int32): seg[E + 1] (rows of expert e: [seg[e], seg[e+1])),
// slot_row[S] (sorted row of slot i, -1 for an invalid expert id) and
// row_token[S] (token of sorted row r; rows >= seg[E] unused).
constexpr int kPlanChunk = 256;

__global__ void moe_count_kernel(const int64_t* __restrict__ sel, int64_t slots, int experts,
                                 int* __restrict__ blockcnt, int* status) {
  extern __shared__ int hist[];
  for (int e = threadIdx.x; e < experts; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  const int64_t i0 = static_cast<int64_t>(blockIdx.x) * kPlanChunk;
  const int64_t i1 = min(i0 + kPlanChunk, slots);
  bool bad = false;
  for (int64_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
    const int64_t e = sel[i];
    if (e >= 0 && e < experts)
      atomicAdd(&hist[e], 1);
    else
      bad = true;
  }
  if (bad) raise_status(status, BIO_DEV_INDEX);
  __syncthreads();
  for (int e = threadIdx.x; e < experts; e += blockDim.x)
    blockcnt[static_cast<int64_t>(blockIdx.x) * experts + e] = hist[e];
}

// One block of 1024 threads; experts <= 1024.
__global__ void __launch_bounds__(1024) moe_scan_kernel(int* __restrict__ blockcnt, int nblocks,
                                                        int experts, int* __restrict__ seg) {
  __shared__ int warp_sum[32];
  const int e = threadIdx.x;
  int run = 0;
  if (e < experts) {
    // eight loads in flight per step
    for (int b0 = 0; b0 < nblocks; b0 += 8) {
      int v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        v[j] = b0 + j < nblocks ? blockcnt[static_cast<int64_t>(b0 + j) * experts + e] : 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (b0 + j < nblocks) blockcnt[static_cast<int64_t>(b0 + j) * experts + e] = run;
        run += v[j];
      }
    }
  }
  // exclusive scan of the per-expert totals across the block
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = run;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += v;
  }
  if (lane == 31) warp_sum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = warp_sum[lane];
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, w, d);
      if (lane >= d) w += v;
    }
    warp_sum[lane] = w;  // inclusive over warps
  }
  __syncthreads();
  const int base = (warp > 0 ? warp_sum[warp - 1] : 0) + incl - run;
  if (e < experts) {
    seg[e] = base;
    for (int b = 0; b < nblocks; ++b) blockcnt[static_cast<int64_t>(b) * experts + e] += base;
  }
  if (threadIdx.x == 0) seg[experts] = warp_sum[31];
}

// One warp per block of kPlanChunk slots.
__global__ void __launch_bounds__(32) moe_place_kernel(const int64_t* __restrict__ sel,
                                                       int64_t slots, int top_k, int experts,
                                                       const int* __restrict__ blockcnt,
                                                       int* __restrict__ slot_row,
                                                       int* __restrict__ row_token) {
  extern __shared__ int next[];
  const int lane = threadIdx.x;
  for (int e = lane; e < experts; e += 32)
    next[e] = blockcnt[static_cast<int64_t>(blockIdx.x) * experts + e];
  __syncwarp();
  const int64_t i0 = static_cast<int64_t>(blockIdx.x) * kPlanChunk;
  const int64_t i1 = min(i0 + kPlanChunk, slots);
  int ev[kPlanChunk / 32];  // all of this lane's ids loaded up front
#pragma unroll
  for (int s = 0; s < kPlanChunk / 32; ++s) {
    const int64_t i = i0 + s * 32 + lane;
    int e = -1;
    if (i < i1) {
      const int64_t v = sel[i];
      e = (v >= 0 && v < experts) ? static_cast<int>(v) : -1;
    }
    ev[s] = e;
  }
#pragma unroll
  for (int s = 0; s < kPlanChunk / 32; ++s) {
    const int64_t i = i0 + s * 32 + lane;
    const int e = ev[s];
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    int pos = -1;
    if (e >= 0) pos = next[e] + rank;
    __syncwarp();
    if (e >= 0 && rank == 0) next[e] += __popc(peers);
    __syncwarp();
    if (i < i1) {
      slot_row[i] = pos;
      if (pos >= 0) row_token[pos] = static_cast<int>(i / top_k);
    }
  }
}

// x_sorted[r, :] = x[row_token[r], :] for r < seg[E]; 16-byte vectors when
// VEC (hidden bytes and both bases 16-byte aligned).
template <bool VEC, typename T>
__global__ void moe_gather_kernel(const T* __restrict__ x, int64_t hidden,
                                  const int* __restrict__ seg_end,
                                  const int* __restrict__ row_token, T* __restrict__ xs,
                                  int64_t max_rows) {
  const int64_t rows = min(static_cast<int64_t>(*seg_end), max_rows);
  const int64_t per = VEC ? hidden * static_cast<int64_t>(sizeof(T)) / 16 : hidden;
  const int64_t total = rows * per;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / per, c = i - r * per;
    const int64_t t = row_token[r];
    if constexpr (VEC) {
      reinterpret_cast<uint4*>(xs + r * hidden)[c] =
          reinterpret_cast<const uint4*>(x + t * hidden)[c];
    } else {
      xs[r * hidden + c] = x[t * hidden + c];
    }
  }
}

// Sparse route sum: the same per-element chain as route_sum_kernel (weight
// rounded to T, product rounded, partial sums rounded, slots left to right),
// reading route j of token t from sorted row slot_row[t * top_k + j].  VEC:
// 16 bytes of columns per thread (16-byte aligned rows).
template <bool VEC, typename T, typename WT>
__global__ void route_sum_sorted_kernel(const T* __restrict__ ys, const WT* __restrict__ w,
                                        const int* __restrict__ slot_row, T* __restrict__ out,
                                        int64_t tokens, int top_k, int64_t hidden) {
  constexpr int V = VEC ? static_cast<int>(16 / sizeof(T)) : 1;
  const int64_t per = hidden / V;
  const int64_t total = tokens * per;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / per, c = (i - t * per) * V;
    bool ok = true;
    float acc[V];
#pragma unroll
    for (int q = 0; q < V; ++q) acc[q] = 0.f;
    for (int j = 0; j < top_k; ++j) {
      const int r = slot_row[t * top_k + j];
      if (r < 0) {
        ok = false;
        break;
      }
      const float wt = round_to<T>(to_f32(w[t * top_k + j]));
      const T* src = ys + static_cast<int64_t>(r) * hidden + c;
      T vals[V];
      if constexpr (VEC) {
        *reinterpret_cast<uint4*>(vals) = *reinterpret_cast<const uint4*>(src);
      } else {
        vals[0] = src[0];
      }
#pragma unroll
      for (int q = 0; q < V; ++q) {
        const float prod = round_to<T>(to_f32(vals[q]) * wt);
        acc[q] = (j == 0) ? prod : round_to<T>(acc[q] + prod);
      }
    }
    T res[V];
#pragma unroll
    for (int q = 0; q < V; ++q) res[q] = from_f32<T>(ok ? acc[q] : 0.f);
    if constexpr (VEC) {
      *reinterpret_cast<uint4*>(out + t * hidden + c) = *reinterpret_cast<const uint4*>(res);
    } else {
      out[t * hidden + c] = res[0];
    }
  }
}

}  // namespace bio

namespace {

unsigned grid_for(int64_t total) {
  int64_t b = (total + 255) / 256;
  if (b > 65536 * 4) b = 65536 * 4;
  return static_cast<unsigned>(b < 1 ? 1 : b);
}

template <typename T>
int launch_route(const void* y, int32_t w_dtype, const void* w, const int64_t* sel, void* out,
                 int64_t e, int64_t t, int64_t k, int64_t d, int* status, cudaStream_t s) {
  const unsigned g = grid_for(t * d);
  switch (w_dtype) {
    case BIO_F32:
      bio::route_sum_kernel<T, float><<<g, 256, 0, s>>>(static_cast<const T*>(y),
                                                        static_cast<const float*>(w), sel,
                                                        static_cast<T*>(out), e, t, k, d, status);
      break;
    case BIO_F16:
      bio::route_sum_kernel<T, __half><<<g, 256, 0, s>>>(static_cast<const T*>(y),
                                                         static_cast<const __half*>(w), sel,
                                                         static_cast<T*>(out), e, t, k, d, status);
      break;
    case BIO_BF16:
      bio::route_sum_kernel<T, __nv_bfloat16><<<g, 256, 0, s>>>(
          static_cast<const T*>(y), static_cast<const __nv_bfloat16*>(w), sel,
          static_cast<T*>(out), e, t, k, d, status);
      break;
    default: return BIO_ERR_DTYPE;
  }
  return bio_host::launch_status(cudaGetLastError());
}

// int32 workspace of the route plan: seg[E + 1] | slot_row[S] | row_token[S]
// | per-block counts[nblocks * E]
struct PlanLayout {
  int64_t slots, nblocks, ints;
  int64_t seg, slot_row, row_token, blockcnt;  // offsets in int32 elements
};

bool plan_layout(int64_t experts, int64_t tokens, int64_t top_k, PlanLayout* l) {
  if (experts < 1 || experts > 1024 || tokens < 0 || top_k < 0) return false;
  if (top_k > 0 && tokens > 2147483647 / top_k) return false;
  l->slots = tokens * top_k;
  l->nblocks = (l->slots + bio::kPlanChunk - 1) / bio::kPlanChunk;
  l->seg = 0;
  l->slot_row = experts + 1;
  l->row_token = l->slot_row + l->slots;
  l->blockcnt = l->row_token + l->slots;
  l->ints = l->blockcnt + l->nblocks * experts;
  return true;
}

template <typename T>
int launch_gather(const void* x, int64_t hidden, const int* ws, const PlanLayout& l,
                  int64_t experts, void* xs, cudaStream_t s) {
  const int64_t bytes = hidden * static_cast<int64_t>(sizeof(T));
  const bool vec = bytes % 16 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(xs) & 15) == 0;
  const int64_t per = vec ? bytes / 16 : hidden;
  const unsigned g = grid_for(l.slots * per);
  if (vec)
    bio::moe_gather_kernel<true, T><<<g, 256, 0, s>>>(static_cast<const T*>(x), hidden,
                                                      ws + l.seg + experts, ws + l.row_token,
                                                      static_cast<T*>(xs), l.slots);
  else
    bio::moe_gather_kernel<false, T><<<g, 256, 0, s>>>(static_cast<const T*>(x), hidden,
                                                       ws + l.seg + experts, ws + l.row_token,
                                                       static_cast<T*>(xs), l.slots);
  return bio_host::launch_status(cudaGetLastError());
}

template <typename T, typename WT>
int launch_route_sorted_w(const void* ys, const void* w, const int* slot_row, void* out,
                          int64_t t, int64_t k, int64_t d, cudaStream_t s) {
  constexpr int64_t V = 16 / sizeof(T);
  const bool vec = d % V == 0 && (reinterpret_cast<uintptr_t>(ys) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(out) & 15) == 0;
  if (vec)
    bio::route_sum_sorted_kernel<true, T, WT><<<grid_for(t * (d / V)), 256, 0, s>>>(
        static_cast<const T*>(ys), static_cast<const WT*>(w), slot_row, static_cast<T*>(out), t,
        static_cast<int>(k), d);
  else
    bio::route_sum_sorted_kernel<false, T, WT><<<grid_for(t * d), 256, 0, s>>>(
        static_cast<const T*>(ys), static_cast<const WT*>(w), slot_row, static_cast<T*>(out), t,
        static_cast<int>(k), d);
  return bio_host::launch_status(cudaGetLastError());
}

template <typename T>
int launch_route_sorted(const void* ys, int32_t w_dtype, const void* w, const int* slot_row,
                        void* out, int64_t t, int64_t k, int64_t d, cudaStream_t s) {
  switch (w_dtype) {
    case BIO_F32: return launch_route_sorted_w<T, float>(ys, w, slot_row, out, t, k, d, s);
    case BIO_F16: return launch_route_sorted_w<T, __half>(ys, w, slot_row, out, t, k, d, s);
    case BIO_BF16:
      return launch_route_sorted_w<T, __nv_bfloat16>(ys, w, slot_row, out, t, k, d, s);
    default: return BIO_ERR_DTYPE;
  }
}

}  // namespace

extern "C" {

int64_t bio_moe_plan_workspace(int64_t experts, int64_t tokens, int64_t top_k) {
  PlanLayout l;
  if (!plan_layout(experts, tokens, top_k, &l)) return 0;
  return (l.ints * 4 + 255) / 256 * 256;
}

int bio_moe_plan(const int64_t* selected_experts, int64_t experts, int64_t tokens,
                 int64_t top_k, void* workspace, int64_t workspace_bytes, int32_t device,
                 void* stream) {
  PlanLayout l;
  if (!plan_layout(experts, tokens, top_k, &l)) return BIO_ERR_SHAPE;
  if (workspace == nullptr || (l.slots > 0 && selected_experts == nullptr)) return BIO_ERR_ARG;
  if (workspace_bytes < l.ints * 4) return BIO_ERR_SCRATCH;
  if ((reinterpret_cast<uintptr_t>(workspace) & 3) != 0) return BIO_ERR_ALIGN;
  int st = bio_host::ensure_device(device);
  if (st != BIO_OK) return st;
  int* ws = static_cast<int*>(workspace);
  int* status = bio_host::status_word(device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int e = static_cast<int>(experts);
  const size_t hist_bytes = static_cast<size_t>(e) * sizeof(int);
  if (l.nblocks > 0) {
    bio::moe_count_kernel<<<static_cast<unsigned>(l.nblocks), 256, hist_bytes, s>>>(
        selected_experts, l.slots, e, ws + l.blockcnt, status);
    st = bio_host::launch_status(cudaGetLastError());
    if (st != BIO_OK) return st;
  }
  bio::moe_scan_kernel<<<1, 1024, 0, s>>>(ws + l.blockcnt, static_cast<int>(l.nblocks), e,
                                          ws + l.seg);
  st = bio_host::launch_status(cudaGetLastError());
  if (st != BIO_OK || l.nblocks == 0) return st;
  bio::moe_place_kernel<<<static_cast<unsigned>(l.nblocks), 32, hist_bytes, s>>>(
      selected_experts, l.slots, static_cast<int>(top_k), e, ws + l.blockcnt, ws + l.slot_row,
      ws + l.row_token);
  return bio_host::launch_status(cudaGetLastError());
}

int bio_moe_gather_rows(int32_t dtype, const void* x, int64_t hidden, const void* plan,
                        int64_t experts, int64_t tokens, int64_t top_k, void* x_sorted,
                        int32_t device, void* stream) {
  PlanLayout l;
  if (!plan_layout(experts, tokens, top_k, &l) || hidden < 0) return BIO_ERR_SHAPE;
  if (l.slots == 0 || hidden == 0) return BIO_OK;
  if (x == nullptr || plan == nullptr || x_sorted == nullptr) return BIO_ERR_ARG;
  int st = bio_host::ensure_device(device);
  if (st != BIO_OK) return st;
  const int* ws = static_cast<const int*>(plan);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case BIO_F32: return launch_gather<float>(x, hidden, ws, l, experts, x_sorted, s);
    case BIO_F16: return launch_gather<__half>(x, hidden, ws, l, experts, x_sorted, s);
    case BIO_BF16: return launch_gather<__nv_bfloat16>(x, hidden, ws, l, experts, x_sorted, s);
    default: return BIO_ERR_DTYPE;
  }
}

int bio_moe_route_sum_sorted(int32_t dtype, const void* y_sorted, int32_t w_dtype,
                             const void* routing_weights, const void* plan, void* out,
                             int64_t experts, int64_t tokens, int64_t top_k, int64_t hidden,
                             int32_t device, void* stream) {
  PlanLayout l;
  if (!plan_layout(experts, tokens, top_k, &l) || hidden < 0) return BIO_ERR_SHAPE;
  if (tokens * hidden == 0) return BIO_OK;
  if (out == nullptr || (top_k > 0 && (y_sorted == nullptr || routing_weights == nullptr ||
                                       plan == nullptr)))
    return BIO_ERR_ARG;
  int st = bio_host::ensure_device(device);
  if (st != BIO_OK) return st;
  const int* slot_row = static_cast<const int*>(plan) + l.slot_row;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case BIO_F32:
      return launch_route_sorted<float>(y_sorted, w_dtype, routing_weights, slot_row, out,
                                        tokens, top_k, hidden, s);
    case BIO_F16:
      return launch_route_sorted<__half>(y_sorted, w_dtype, routing_weights, slot_row, out,
                                         tokens, top_k, hidden, s);
    case BIO_BF16:
      return launch_route_sorted<__nv_bfloat16>(y_sorted, w_dtype, routing_weights, slot_row,
                                                out, tokens, top_k, hidden, s);
    default: return BIO_ERR_DTYPE;
  }
}

int bio_silu_mul(int32_t dtype, const void* gate, const void* up, void* out, int64_t n,
                 int32_t device, void* stream) {
  if (n < 0) return BIO_ERR_SHAPE;
  if (n == 0) return BIO_OK;
  if (gate == nullptr || up == nullptr || out == nullptr) return BIO_ERR_ARG;
  int st = bio_host::ensure_device(device);
  if (st != BIO_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool aligned = ((reinterpret_cast<uintptr_t>(gate) | reinterpret_cast<uintptr_t>(up) |
                         reinterpret_cast<uintptr_t>(out)) & 15u) == 0;
  const int64_t per = dtype == BIO_F32 ? 4 : 8;
  if (aligned && n % per == 0 && (dtype == BIO_F32 || dtype == BIO_F16 || dtype == BIO_BF16)) {
    const int64_t nvec = n / per;
    const unsigned g = grid_for(nvec);
    switch (dtype) {
      case BIO_F32:
        bio::silu_mul_vec_kernel<float><<<g, 256, 0, s>>>(static_cast<const float*>(gate),
                                                          static_cast<const float*>(up),
                                                          static_cast<float*>(out), nvec);
        break;
      case BIO_F16:
        bio::silu_mul_vec_kernel<__half><<<g, 256, 0, s>>>(static_cast<const __half*>(gate),
                                                           static_cast<const __half*>(up),
                                                           static_cast<__half*>(out), nvec);
        break;
      default:
        bio::silu_mul_vec_kernel<__nv_bfloat16><<<g, 256, 0, s>>>(
            static_cast<const __nv_bfloat16*>(gate), static_cast<const __nv_bfloat16*>(up),
            static_cast<__nv_bfloat16*>(out), nvec);
        break;
    }
    return bio_host::launch_status(cudaGetLastError());
  }
  switch (dtype) {
    case BIO_F32:
      bio::silu_mul_kernel<float><<<grid_for(n), 256, 0, s>>>(
          static_cast<const float*>(gate), static_cast<const float*>(up), static_cast<float*>(out), n);
      break;
    case BIO_F16:
      bio::silu_mul_kernel<__half><<<grid_for(n), 256, 0, s>>>(
          static_cast<const __half*>(gate), static_cast<const __half*>(up), static_cast<__half*>(out), n);
      break;
    case BIO_BF16:
      bio::silu_mul_kernel<__nv_bfloat16><<<grid_for(n), 256, 0, s>>>(
          static_cast<const __nv_bfloat16*>(gate), static_cast<const __nv_bfloat16*>(up),
          static_cast<__nv_bfloat16*>(out), n);
      break;
    default: return BIO_ERR_DTYPE;
  }
  return bio_host::launch_status(cudaGetLastError());
}

int bio_moe_route_sum(int32_t dtype, const void* expert_out, int32_t w_dtype,
                      const void* routing_weights, const int64_t* selected_experts, void* out,
                      int64_t experts, int64_t tokens, int64_t top_k, int64_t hidden,
                      int32_t device, void* stream) {
  if (experts < 1 || tokens < 0 || top_k < 0 || hidden < 0) return BIO_ERR_SHAPE;
  if (tokens * hidden == 0) return BIO_OK;
  if (out == nullptr || (top_k > 0 && (expert_out == nullptr || routing_weights == nullptr ||
                                       selected_experts == nullptr)))
    return BIO_ERR_ARG;
  int st = bio_host::ensure_device(device);
  if (st != BIO_OK) return st;
  int* status = bio_host::status_word(device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case BIO_F32:
      return launch_route<float>(expert_out, w_dtype, routing_weights, selected_experts, out,
                                 experts, tokens, top_k, hidden, status, s);
    case BIO_F16:
      return launch_route<__half>(expert_out, w_dtype, routing_weights, selected_experts, out,
                                  experts, tokens, top_k, hidden, status, s);
    case BIO_BF16:
      return launch_route<__nv_bfloat16>(expert_out, w_dtype, routing_weights, selected_experts,
                                         out, experts, tokens, top_k, hidden, status, s);
    default: return BIO_ERR_DTYPE;
  }
}

}  // extern "C"
