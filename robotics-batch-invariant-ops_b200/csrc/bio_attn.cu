// Fused batch-invariant attention (dense SDPA and sequence-packed varlen).
//
// One warp owns one (sequence, head, query row).  Keys are visited in fixed
// blocks of 32 in increasing order: lane j computes the score of key j of the
// block (sequential fp32 dot product over d), the block maximum and the sum of
// exponentials use a fixed xor-shuffle tree, and lane t accumulates output
// columns dv = t, t+32, ... as o = o * corr + sum_j p_j * v[j][dv] with j in
// order (online softmax).  Nothing depends on how many sequences, heads or
// rows are in the launch, so every query row is batch invariant.
//
// Masks: causal (top-left, or bottom-right for varlen), boolean keep-masks and
// additive float masks, broadcast through strides (0 = broadcast).  A row
// whose keys are all masked (or whose KV range is empty) produces zeros, like
// the reference's softmax edge rule.  Grouped-query attention reads KV head
// h / (H / Hkv) directly (no repeat_interleave copy).
//
// Varlen: the sequence of a packed query token is found on the device by a
// binary search of cu_seqlens_q; tokens outside every sequence are written as
// zeros; invalid offsets raise BIO_DEV_INDEX in the status word (no host
// synchronisation).
//
// Reference: scaled_dot_product_attention_batch_invariant
// (batch_invariant_ops.py:1148-1213) and
// varlen_scaled_dot_product_attention_batch_invariant (:1216-1344).
#include "bio_common.cuh"

namespace bio {

constexpr int kAttnWarps = 8;
constexpr int kMaxHeadDim = 256;

struct AttnParams {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  // strides in elements: [batch][head][token][dim]
  int64_t q_sb, q_sh, q_st;
  int64_t k_sb, k_sh, k_st;
  int64_t v_sb, v_sh, v_st;
  int64_t o_sb, o_sh, o_st;
  int64_t batch, heads, kv_heads;
  int64_t lq, lk;  // dense lengths (varlen: total packed tokens)
  int d, dv;
  float scale;
  int causal;      // 0 none, 1 top-left, 2 bottom-right, 3 equal-lengths-required
  const void* mask;
  int64_t m_sb, m_sh, m_sq, m_sk;
  // varlen
  const void* cu_q;
  const void* cu_k;
  int cu_is64;
  int64_t nseq;
  int* status;
};

__device__ __forceinline__ int64_t load_off(const void* p, int is64, int64_t i) {
  return is64 ? static_cast<const int64_t*>(p)[i] : static_cast<int64_t>(static_cast<const int*>(p)[i]);
}

template <typename MT>
__device__ __forceinline__ float mask_value(const MT* m, int64_t idx) {
  return to_f32(m[idx]);
}

__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return __shfl_sync(0xffffffffu, v, 0);
}

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return __shfl_sync(0xffffffffu, v, 0);
}

template <typename T, int MASK, typename MT, bool VARLEN>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_kernel(const AttnParams p) {
  __shared__ float qs[kAttnWarps][kMaxHeadDim];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t total_rows = VARLEN ? p.lq * p.heads : p.batch * p.heads * p.lq;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kAttnWarps + warp;
  if (row >= total_rows) return;

  int64_t b, h, i, lq, lk, q_tok, k_tok0;
  T* out_row;
  if constexpr (VARLEN) {
    const int64_t t = row / p.heads;
    h = row - t * p.heads;
    out_row = static_cast<T*>(p.o) + t * p.o_st + h * p.o_sh;
    // binary search: largest s with cu_q[s] <= t, s < nseq
    int64_t lo = 0, hi = p.nseq;  // answer in [0, nseq)
    const int64_t last = load_off(p.cu_q, p.cu_is64, p.nseq);
    bool covered = t < last;
    while (covered && hi - lo > 1) {
      const int64_t mid = (lo + hi) >> 1;
      if (load_off(p.cu_q, p.cu_is64, mid) <= t) lo = mid; else hi = mid;
    }
    b = lo;
    int64_t qs0 = 0, qs1 = 0, ks0 = 0, ks1 = 0;
    if (covered) {
      qs0 = load_off(p.cu_q, p.cu_is64, b);
      qs1 = load_off(p.cu_q, p.cu_is64, b + 1);
      ks0 = load_off(p.cu_k, p.cu_is64, b);
      ks1 = load_off(p.cu_k, p.cu_is64, b + 1);
      const bool bad = qs0 > t || qs1 <= t || qs1 > p.lq || ks1 < ks0 || ks0 < 0 || ks1 > p.lk ||
                       load_off(p.cu_q, p.cu_is64, 0) != 0 || load_off(p.cu_k, p.cu_is64, 0) != 0;
      if (bad) {
        if (lane == 0) raise_status(p.status, BIO_DEV_INDEX);
        covered = false;
      }
    }
    if (covered && p.causal == 3 && (qs1 - qs0) != (ks1 - ks0)) {
      if (lane == 0) raise_status(p.status, BIO_DEV_INDEX);
      covered = false;
    }
    if (!covered) {
      for (int c = lane; c < p.dv; c += 32) out_row[c] = from_f32<T>(0.f);
      return;
    }
    i = t - qs0;
    lq = qs1 - qs0;
    lk = ks1 - ks0;
    q_tok = t;
    k_tok0 = ks0;
  } else {
    i = row % p.lq;
    const int64_t bh = row / p.lq;
    h = bh % p.heads;
    b = bh / p.heads;
    lq = p.lq;
    lk = p.lk;
    q_tok = i;
    k_tok0 = 0;
    out_row = static_cast<T*>(p.o) + b * p.o_sb + h * p.o_sh + i * p.o_st;
  }
  const int64_t hk = h / (p.heads / p.kv_heads);
  const T* qrow = static_cast<const T*>(p.q) + (VARLEN ? 0 : b * p.q_sb) + h * p.q_sh + q_tok * p.q_st;
  const T* kbase = static_cast<const T*>(p.k) + (VARLEN ? 0 : b * p.k_sb) + hk * p.k_sh + k_tok0 * p.k_st;
  const T* vbase = static_cast<const T*>(p.v) + (VARLEN ? 0 : b * p.v_sb) + hk * p.v_sh + k_tok0 * p.v_st;

  for (int c = lane; c < p.d; c += 32) qs[warp][c] = to_f32(qrow[c]);
  __syncwarp();

  // causal limit: keys j <= i + shift are visible
  int64_t kend = lk;
  if (p.causal == 1 || p.causal == 3) kend = min(lk, i + 1);
  if (p.causal == 2) kend = min(lk, i + (lk - lq) + 1);
  if (kend < 0) kend = 0;

  float m = -INFINITY, l = 0.f;
  float o[kMaxHeadDim / 32];
#pragma unroll
  for (int t = 0; t < kMaxHeadDim / 32; ++t) o[t] = 0.f;

  const MT* mrow = nullptr;
  if constexpr (MASK != 0) {
    mrow = static_cast<const MT*>(p.mask) + b * p.m_sb + h * p.m_sh + i * p.m_sq;
  }

  for (int64_t j0 = 0; j0 < kend; j0 += 32) {
    const int64_t j = j0 + lane;
    float s = -INFINITY;
    if (j < kend) {
      const T* krow = kbase + j * p.k_st;
      float acc = 0.f;
      for (int c = 0; c < p.d; ++c) acc += qs[warp][c] * to_f32(krow[c]);
      s = acc * p.scale;
      if constexpr (MASK == 1) {
        if (!mrow[j * p.m_sk]) s = -INFINITY;
      } else if constexpr (MASK == 2) {
        s += mask_value(mrow, j * p.m_sk);
      }
    }
    const float bm = warp_max_f(s);
    const float m_new = fmaxf(m, bm);
    if (m_new == -INFINITY) continue;  // every key so far is masked
    const float corr = (m == -INFINITY) ? 0.f : expf(m - m_new);
    const float pj = (s == -INFINITY) ? 0.f : expf(s - m_new);
    l = l * corr + warp_sum_f(pj);
    const int nk = static_cast<int>(min(static_cast<int64_t>(32), kend - j0));
#pragma unroll
    for (int t = 0; t < kMaxHeadDim / 32; ++t) o[t] *= corr;
    for (int jj = 0; jj < nk; ++jj) {
      const float pv = __shfl_sync(0xffffffffu, pj, jj);
      const T* vrow = vbase + (j0 + jj) * p.v_st;
#pragma unroll
      for (int t = 0; t < kMaxHeadDim / 32; ++t) {
        const int c = lane + 32 * t;
        if (c < p.dv) o[t] += pv * to_f32(vrow[c]);
      }
    }
    m = m_new;
  }
#pragma unroll
  for (int t = 0; t < kMaxHeadDim / 32; ++t) {
    const int c = lane + 32 * t;
    if (c < p.dv) out_row[c] = from_f32<T>(l > 0.f ? o[t] / l : 0.f);
  }
}

}  // namespace bio

namespace {

template <typename T, int MASK, typename MT>
int launch_attn(const bio::AttnParams& p, bool varlen, cudaStream_t s) {
  const int64_t rows = varlen ? p.lq * p.heads : p.batch * p.heads * p.lq;
  if (rows == 0) return BIO_OK;
  const int64_t blocks = (rows + bio::kAttnWarps - 1) / bio::kAttnWarps;
  if (blocks > 2147483647) return BIO_ERR_SHAPE;
  const unsigned g = static_cast<unsigned>(blocks);
  if (varlen)
    bio::attn_kernel<T, MASK, MT, true><<<g, bio::kAttnWarps * 32, 0, s>>>(p);
  else
    bio::attn_kernel<T, MASK, MT, false><<<g, bio::kAttnWarps * 32, 0, s>>>(p);
  return bio_host::launch_status(cudaGetLastError());
}

template <typename T>
int dispatch_mask(const bio::AttnParams& p, int mask_kind, int mask_dtype, bool varlen,
                  cudaStream_t s) {
  switch (mask_kind) {
    case BIO_MASK_NONE: return launch_attn<T, 0, uint8_t>(p, varlen, s);
    case BIO_MASK_BOOL: return launch_attn<T, 1, uint8_t>(p, varlen, s);
    case BIO_MASK_ADD:
      switch (mask_dtype) {
        case BIO_F32: return launch_attn<T, 2, float>(p, varlen, s);
        case BIO_F16: return launch_attn<T, 2, __half>(p, varlen, s);
        case BIO_BF16: return launch_attn<T, 2, __nv_bfloat16>(p, varlen, s);
        default: return BIO_ERR_DTYPE;
      }
    default: return BIO_ERR_ARG;
  }
}

int run_attention(const bio_attn_args* a, bool varlen, void* stream) {
  if (a == nullptr) return BIO_ERR_ARG;
  if (a->d < 1 || a->dv < 1 || a->d > bio::kMaxHeadDim || a->dv > bio::kMaxHeadDim)
    return BIO_ERR_SHAPE;
  if (a->heads < 1 || a->kv_heads < 1 || a->heads % a->kv_heads) return BIO_ERR_SHAPE;
  if (a->batch < 0 || a->lq < 0 || a->lk < 0) return BIO_ERR_SHAPE;
  if (a->causal < 0 || a->causal > 3) return BIO_ERR_ARG;
  if (a->mask_kind != BIO_MASK_NONE && a->mask == nullptr) return BIO_ERR_ARG;
  if (varlen && (a->cu_q == nullptr || a->cu_k == nullptr || a->nseq < 0)) return BIO_ERR_ARG;
  const int64_t rows = varlen ? a->lq * a->heads : a->batch * a->heads * a->lq;
  if (rows == 0) return BIO_OK;
  if (a->q == nullptr || a->o == nullptr || (a->lk > 0 && (a->k == nullptr || a->v == nullptr)))
    return BIO_ERR_ARG;
  int st = bio_host::ensure_device(a->device);
  if (st != BIO_OK) return st;
  bio::AttnParams p;
  p.q = a->q; p.k = a->k; p.v = a->v; p.o = a->o;
  p.q_sb = a->q_sb; p.q_sh = a->q_sh; p.q_st = a->q_st;
  p.k_sb = a->k_sb; p.k_sh = a->k_sh; p.k_st = a->k_st;
  p.v_sb = a->v_sb; p.v_sh = a->v_sh; p.v_st = a->v_st;
  p.o_sb = a->o_sb; p.o_sh = a->o_sh; p.o_st = a->o_st;
  p.batch = a->batch; p.heads = a->heads; p.kv_heads = a->kv_heads;
  p.lq = a->lq; p.lk = a->lk; p.d = a->d; p.dv = a->dv;
  p.scale = a->scale; p.causal = a->causal;
  p.mask = a->mask; p.m_sb = a->m_sb; p.m_sh = a->m_sh; p.m_sq = a->m_sq; p.m_sk = a->m_sk;
  p.cu_q = a->cu_q; p.cu_k = a->cu_k; p.cu_is64 = a->cu_is64; p.nseq = a->nseq;
  p.status = bio_host::status_word(a->device);
  if (a->dtype != BIO_F32) return bio_host::attn_tc_launch(a, varlen, stream);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (a->dtype) {
    case BIO_F32: return dispatch_mask<float>(p, a->mask_kind, a->mask_dtype, varlen, s);
    case BIO_F16: return dispatch_mask<__half>(p, a->mask_kind, a->mask_dtype, varlen, s);
    case BIO_BF16: return dispatch_mask<__nv_bfloat16>(p, a->mask_kind, a->mask_dtype, varlen, s);
    default: return BIO_ERR_DTYPE;
  }
}

}  // namespace

extern "C" {

int bio_attention(const bio_attn_args* args, void* stream) {
  return run_attention(args, false, stream);
}

int bio_attention_varlen(const bio_attn_args* args, void* stream) {
  if (args != nullptr && args->mask_kind != BIO_MASK_NONE) return BIO_ERR_ARG;
  return run_attention(args, true, stream);
}

}  // extern "C"
