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

}  // namespace

extern "C" {

int bio_silu_mul(int32_t dtype, const void* gate, const void* up, void* out, int64_t n,
                 int32_t device, void* stream) {
  if (n < 0) return BIO_ERR_SHAPE;
  if (n == 0) return BIO_OK;
  if (gate == nullptr || up == nullptr || out == nullptr) return BIO_ERR_ARG;
  int st = bio_host::ensure_device(device);
  if (st != BIO_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
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
