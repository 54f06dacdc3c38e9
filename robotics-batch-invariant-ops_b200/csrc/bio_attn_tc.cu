// Tensor-core fused attention for bf16 / fp16 (dense SDPA and varlen).
//
// One CTA owns 128 query rows of one (sequence, head).  Keys are visited in
// fixed blocks of BN from the first key of the sequence (BN = 128, or 64 for
// D = Dv = 256 so that a two-deep K/V ring fits in shared memory; BN is a
// function of the head dims only):
//   warp 0      TMA: Q tile once, then K and V tiles of each key block into a
//               ring (128-byte swizzle; V is read N-major for the PV product).
//   warp 1      MMA: S_j = Q K_j^T (tcgen05, M=128, N=128, fp32 in TMEM, two S
//               buffers so S_{j+1} overlaps the softmax of block j), then
//               O += P_j V_j (M=128, N=Dv, O accumulator resident in TMEM).
//   warps 2..5  softmax: thread r owns query row r (its TMEM lane), reads its
//               128 scores, applies scale and masks, keeps the running max m
//               and sum l in fp32 (sequential over the 128 columns, so the
//               order is fixed by the key index alone), writes P_j (rounded to
//               the input dtype) into shared memory, rescales its O row in TMEM
//               by exp(m_old - m_new) when the max moved, and finally stores
//               O / l.
// A row's arithmetic depends on its Q row, the sequence's K/V and the fixed
// block partition only -- never on the other rows, heads or sequences of the
// launch -- so every output row is batch invariant.  Fully masked rows and
// empty key ranges produce zeros.  Grouped-query attention reads KV head
// h / (H / Hkv) directly.
//
// Varlen: a one-thread plan kernel turns cu_seqlens_q into per-sequence
// q-block offsets on the device; each CTA finds its (sequence, q-block) by
// binary search, so there is no host synchronisation.  K/V rows of a partial
// last block that belong to the next sequence are zeroed in shared memory
// before the PV product, so neighbouring sequences cannot leak in even when
// they hold non-finite values.
//
// Reference: scaled_dot_product_attention_batch_invariant
// (batch_invariant_ops.py:1148-1213), varlen_scaled_dot_product_attention_batch_invariant
// (:1216-1344).
#include <mutex>

#include "bio_common.cuh"

namespace bio {

constexpr int kAtBM = 128;
constexpr int kAtBN = 128;

struct AttnTcParams {
  int64_t heads, kv_heads;
  int64_t lq, lk;  // dense lengths; varlen: packed token counts
  int d, dv;
  float scale;
  int causal;
  const void* mask;
  int mask_kind;  // 0 none, 1 bool, 2 f32, 3 f16, 4 bf16 additive
  int64_t m_sb, m_sh, m_sq, m_sk;
  void* o;
  int64_t o_sb, o_sh, o_st;
  int varlen;
  const void* cu_q;
  const void* cu_k;
  int cu_is64;
  int64_t nseq;
  const int* blk_start;
  const int* order;  // two-tile varlen: planned position -> sequence id
  // One-tile dense kernel, grouped-query packing (0 = off): a CTA's 128 rows
  // are pack_tok consecutive query tokens of each of the 128 / pack_tok query
  // heads that share KV head blockIdx.y (row r: head blockIdx.y * 128 /
  // pack_tok + r / pack_tok, token blockIdx.x * pack_tok + r % pack_tok).
  int pack_tok;
  int* status;
};

// Key block of the one-tile kernel for padded head dims (DP, DVP).
template <int DP, int DVP>
constexpr int at_block_n() { return (DP == 256 && DVP == 256) ? 64 : kAtBN; }

// Shared memory plan.  HALVES = 2 splits every query row between two softmax
// warps (BN/2 score columns each) that exchange partial max / sum through kX.
template <int DP, int DVP, int BN = at_block_n<DP, DVP>()>
struct AttnSmem {
  static constexpr uint32_t kQ = kAtBM * DP * 2;
  static constexpr uint32_t kK = BN * DP * 2;
  static constexpr uint32_t kV = BN * DVP * 2;
  static constexpr uint32_t kP = kAtBM * BN * 2;
  static constexpr uint32_t kBar = 256;
  static constexpr int kHalves = 2;
  static constexpr uint32_t kX = kHalves == 2 ? 2 * 2 * 128 * 4 : 0;
  static constexpr uint32_t kFixed = 1024 + kQ + kP + kBar + kX;
  static constexpr int kStages = (227u * 1024u - kFixed) / (kK + kV) >= 2 ? 2 : 1;
  static constexpr uint32_t kTotal = kFixed + kStages * (kK + kV);
  static constexpr int kThreads = 64 + 128 * kHalves;
};

__device__ __forceinline__ int64_t ld_off(const void* p, int is64, int64_t i) {
  return is64 ? static_cast<const int64_t*>(p)[i]
              : static_cast<int64_t>(static_cast<const int*>(p)[i]);
}

__device__ __forceinline__ float mask_add(const void* m, int kind, int64_t idx) {
  switch (kind) {
    case 2: return static_cast<const float*>(m)[idx];
    case 3: return __half2float(static_cast<const __half*>(m)[idx]);
    default: return __bfloat162float(static_cast<const __nv_bfloat16*>(m)[idx]);
  }
}

template <typename T>
__device__ __forceinline__ uint32_t pack_pair(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack_pair<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack_pair<__half>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// 2^x on the special-function unit (PTX ex2.approx).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Fixed binary trees over 32 values (the order depends only on the index).
__device__ __forceinline__ float tree_max32(const float (&v)[32]) {
  float t[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) t[j] = fmaxf(v[2 * j], v[2 * j + 1]);
#pragma unroll
  for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
    for (int j = 0; j < w; ++j) t[j] = fmaxf(t[2 * j], t[2 * j + 1]);
  return t[0];
}

__device__ __forceinline__ float tree_sum16(float (&t)[16]) {
#pragma unroll
  for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
    for (int j = 0; j < w; ++j) t[j] = t[2 * j] + t[2 * j + 1];
  return t[0];
}

// Unpack a rounded pair back to fp32 (exact).
template <typename T>
__device__ __forceinline__ void unpack_pair(uint32_t w, float& lo, float& hi);
template <>
__device__ __forceinline__ void unpack_pair<__nv_bfloat16>(uint32_t w, float& lo, float& hi) {
  lo = __uint_as_float(w << 16);
  hi = __uint_as_float(w & 0xFFFF0000u);
}
template <>
__device__ __forceinline__ void unpack_pair<__half>(uint32_t w, float& lo, float& hi) {
  __half2 h = *reinterpret_cast<__half2*>(&w);
  lo = __low2float(h);
  hi = __high2float(h);
}

template <typename T>
struct AtFmt;
template <>
struct AtFmt<__half> {
  static constexpr uint32_t v = 0;
};
template <>
struct AtFmt<__nv_bfloat16> {
  static constexpr uint32_t v = 1;
};

// try_wait with a suspend-time hint: a waiting warp is parked until the phase
// completes (or the hint elapses) instead of spinning on the issue slots that
// the softmax warps need.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(1000000u)
      : "memory");
  return ok != 0;
}

// Bounded wait (same contract as mbar_wait) built on the sleeping try_wait.
__device__ __forceinline__ bool at_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                        int* status) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait_sleep(a, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t i = 1; i < kWaitMaxIters; ++i) {
    if (mbar_try_wait_sleep(a, parity)) return true;
    if (*abort_flag) return false;
    if (global_timer_ns() - t0 > kWaitTimeoutNs) break;
  }
  *abort_flag = 1;
  raise_status(status, BIO_DEV_TIMEOUT);
  return false;
}

__device__ __forceinline__ bool at_wait_drain(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  const uint64_t t0 = global_timer_ns();
  for (uint32_t i = 0; i < kWaitMaxIters; ++i) {
    if (mbar_try_wait(a, parity)) return true;
    if ((i & 63u) == 63u && global_timer_ns() - t0 > kWaitTimeoutNs) return false;
  }
  return false;
}

template <int DP, int DVP, typename T>
__global__ void __launch_bounds__(AttnSmem<DP, DVP>::kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const AttnTcParams p) {
  using L = AttnSmem<DP, DVP>;
  constexpr int BN = at_block_n<DP, DVP>();  // keys per block
  constexpr int S = L::kStages;
  constexpr int HALVES = L::kHalves;
  constexpr int CPT = BN / 32 / HALVES;  // 32-column score chunks per softmax thread
  constexpr int kQChunks = DP / 64;
  constexpr int kVChunks = DVP / 64;
  constexpr uint32_t kKChunk = BN * 128;  // one 64-column chunk of a K block
  constexpr uint32_t kIdescS = idesc_f16(AtFmt<T>::v, kAtBM, BN, false, false);
  constexpr uint32_t kIdescO = idesc_f16(AtFmt<T>::v, kAtBM, DVP, false, true);
  constexpr uint32_t kOCol = 256;  // TMEM: S0 [0,128), S1 [128,256), O [256, 256+DVP)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // ---------------------------------------------------------------- work
  const int pt = p.varlen ? 0 : p.pack_tok;
  int64_t b = 0, h = blockIdx.y, q0, lq_seq, lk_seq, q_tok0, k_tok0;
  if (p.varlen) {
    const int64_t g = blockIdx.x;
    const int64_t total = p.blk_start[p.nseq];
    if (g >= total) return;
    int64_t lo = 0, hi = p.nseq;
    while (hi - lo > 1) {
      const int64_t mid = (lo + hi) >> 1;
      if (p.blk_start[mid] <= g) lo = mid; else hi = mid;
    }
    const int64_t s = lo;
    const int64_t qs0 = ld_off(p.cu_q, p.cu_is64, s), qs1 = ld_off(p.cu_q, p.cu_is64, s + 1);
    const int64_t ks0 = ld_off(p.cu_k, p.cu_is64, s), ks1 = ld_off(p.cu_k, p.cu_is64, s + 1);
    const bool bad = qs0 < 0 || qs1 > p.lq || ks0 < 0 || ks1 < ks0 || ks1 > p.lk ||
                     ld_off(p.cu_q, p.cu_is64, 0) != 0 || ld_off(p.cu_k, p.cu_is64, 0) != 0 ||
                     (p.causal == 3 && (qs1 - qs0) != (ks1 - ks0));
    if (bad) {
      if (threadIdx.x == 0) raise_status(p.status, BIO_DEV_INDEX);
      return;  // output rows stay zero (pre-zeroed by the caller)
    }
    q0 = (g - p.blk_start[s]) * kAtBM;
    lq_seq = qs1 - qs0;
    lk_seq = ks1 - ks0;
    q_tok0 = qs0 + q0;
    k_tok0 = ks0;
  } else {
    b = blockIdx.z;
    if (pt > 0) {
      q0 = static_cast<int64_t>(blockIdx.x) * pt;
      h = static_cast<int64_t>(blockIdx.y) * (kAtBM / pt);  // first query head of the tile
    } else {
      q0 = static_cast<int64_t>(blockIdx.x) * kAtBM;
    }
    lq_seq = p.lq;
    lk_seq = p.lk;
    q_tok0 = q0;
    k_tok0 = 0;
  }
  const int64_t hk = pt > 0 ? static_cast<int64_t>(blockIdx.y) : h / (p.heads / p.kv_heads);
  // query tokens of this tile that exist (each packed head has the same ones)
  const int64_t nrows = min(static_cast<int64_t>(pt > 0 ? pt : kAtBM), lq_seq - q0);
  const int64_t shift = (p.causal == 2) ? (lk_seq - lq_seq) : 0;
  int64_t kend_cta = lk_seq;
  if (p.causal != 0) kend_cta = min(lk_seq, q0 + nrows - 1 + shift + 1);
  if (kend_cta < 0) kend_cta = 0;
  const int nblk = static_cast<int>((kend_cta + BN - 1) / BN);

  // per-row head, token and output pointer (softmax warps)
  const int r = (warp & 3) * 32 + lane;
  const int rt = pt > 0 ? (r % pt) : r;              // token offset of row r in the tile
  const int64_t hrow = pt > 0 ? h + r / pt : h;      // query head of row r
  const int64_t i = q0 + rt;
  const bool row_valid = warp >= 2 && rt < nrows;
  T* out_row = nullptr;
  if (row_valid) {
    out_row = static_cast<T*>(p.o) + (p.varlen ? 0 : b * p.o_sb) + hrow * p.o_sh +
              (p.varlen ? (q_tok0 + r) : i) * p.o_st;
  }
  if (nblk == 0) {
    if (row_valid && warp < 6)
      for (int c = 0; c < p.dv; ++c) out_row[c] = from_f32<T>(0.f);
    return;
  }

  // ---------------------------------------------------------------- smem
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;
  uint8_t* sP = sQ + L::kQ;
  uint8_t* sK = sP + L::kP;
  uint8_t* sV = sK + S * L::kK;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + S * L::kV);
  uint64_t* q_full = bars + 0;
  // K and V of a stage have their own barriers: K_{j+1} is copied as soon
  // as S_j has consumed K_j, while softmax_j and PV_j still run
  uint64_t* k_full = bars + 1;       // [S]
  uint64_t* k_empty = bars + 3;      // [S]
  uint64_t* v_full = bars + 18;      // [S]
  uint64_t* v_empty = bars + 20;     // [S]
  uint64_t* s_full = bars + 5;       // [2]
  uint64_t* s_free = bars + 7;       // [2]
  uint64_t* p_ready = bars + 9;
  uint64_t* pv_done = bars + 10;
  uint64_t* mma_done = bars + 11;
  uint64_t* xbar = bars + 12;        // [4] pair exchange, one per TMEM lane quarter
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* xmax = reinterpret_cast<float*>(sV + S * L::kV + L::kBar);  // [2][128]
  float* xsum = xmax + 256;                                          // [2][128]

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < S; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_free[s], 4 * HALVES);
    }
    mbar_init(p_ready, 4 * HALVES);
    for (int q = 0; q < 4; ++q) mbar_init(&xbar[q], 64);
    mbar_init(pv_done, 1);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int qc = static_cast<int>(q_tok0), kc0 = static_cast<int>(k_tok0);
  const int hc = static_cast<int>(h), hkc = static_cast<int>(hk), bc = static_cast<int>(b);

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      mbar_arrive_expect_tx(q_full, L::kQ);
      for (int c = 0; c < kQChunks; ++c)
        tma_load_4d(sQ + c * 16384, &tmQ, q_full, c * 64, qc, hc, bc);
      int k_issued = 0, v_issued = 0;
      for (int jb = 0; jb < nblk; ++jb) {
        const int stage = jb % S;
        const uint32_t ph = static_cast<uint32_t>(jb / S) & 1u;
        const int row = kc0 + jb * BN;
        if (!at_wait(&k_empty[stage], ph ^ 1u, abort_flag, p.status)) break;
        mbar_arrive_expect_tx(&k_full[stage], L::kK);
        uint8_t* k_dst = sK + stage * L::kK;
        for (int c = 0; c < kQChunks; ++c)
          tma_load_4d(k_dst + c * kKChunk, &tmK, &k_full[stage], c * 64, row, hkc, bc);
        k_issued = jb + 1;
        if (!at_wait(&v_empty[stage], ph ^ 1u, abort_flag, p.status)) break;
        mbar_arrive_expect_tx(&v_full[stage], L::kV);
        uint8_t* v_dst = sV + stage * L::kV;
        for (int kcnk = 0; kcnk < BN / 64; ++kcnk)
          for (int nc = 0; nc < kVChunks; ++nc)
            tma_load_4d(v_dst + (kcnk * kVChunks + nc) * 8192, &tmV, &v_full[stage], nc * 64,
                        row + kcnk * 64, hkc, bc);
        v_issued = jb + 1;
      }
      // drain: Q and the last loads of each stage must land before exit
      if (!at_wait_drain(q_full, 0)) raise_status(p.status, BIO_DEV_TIMEOUT);
      for (int jb = k_issued - 1; jb >= 0 && jb >= k_issued - S; --jb) {
        if (!at_wait_drain(&k_full[jb % S], static_cast<uint32_t>(jb / S) & 1u))
          raise_status(p.status, BIO_DEV_TIMEOUT);
      }
      for (int jb = v_issued - 1; jb >= 0 && jb >= v_issued - S; --jb) {
        if (!at_wait_drain(&v_full[jb % S], static_cast<uint32_t>(jb / S) & 1u))
          raise_status(p.status, BIO_DEV_TIMEOUT);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA
      bool ok = at_wait(q_full, 0, abort_flag, p.status);
      auto issue_s = [&](int jb) -> bool {
        const int stage = jb % S;
        if (!at_wait(&k_full[stage], static_cast<uint32_t>(jb / S) & 1u, abort_flag, p.status))
          return false;
        const int sb = jb & 1;
        if (!at_wait(&s_free[sb], (static_cast<uint32_t>(jb >> 1) & 1u) ^ 1u, abort_flag,
                       p.status))
          return false;
        tc_fence_after();
        const uint32_t qa = smem_u32(sQ), ka = smem_u32(sK + stage * L::kK);
#pragma unroll
        for (int kk = 0; kk < DP / 16; ++kk) {
          const uint32_t qoff = (kk >> 2) * 16384 + (kk & 3) * 32;
          const uint32_t koff = (kk >> 2) * kKChunk + (kk & 3) * 32;
          umma_f16(tmem + static_cast<uint32_t>(sb * 128), smem_desc_sw128(qa + qoff, 16, 1024),
                   smem_desc_sw128(ka + koff, 16, 1024), kIdescS, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[sb]);
        umma_commit(&k_empty[stage]);  // K_jb is free once S_jb is done
        return true;
      };
      // S_{j+1} is issued before PV_j (its K copy overlaps softmax_j); the
      // softmax waits for PV_{j-1} before it rewrites P
      if (ok) ok = issue_s(0);
      for (int jb = 0; ok && jb < nblk; ++jb) {
        if (jb + 1 < nblk && !issue_s(jb + 1)) break;
        if (!at_wait(p_ready, static_cast<uint32_t>(jb) & 1u, abort_flag, p.status)) break;
        const int stage = jb % S;
        if (!at_wait(&v_full[stage], static_cast<uint32_t>(jb / S) & 1u, abort_flag, p.status))
          break;
        tc_fence_after();
        const uint32_t pa = smem_u32(sP), va = smem_u32(sV + stage * L::kV);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint32_t aoff = (kk >> 2) * 16384 + (kk & 3) * 32;
          const uint32_t boff = (kk >> 2) * (kVChunks * 8192) + (kk & 3) * 2048;
          umma_f16(tmem + kOCol, smem_desc_sw128(pa + aoff, 16, 1024),
                   smem_desc_sw128(va + boff, 8192, 1024), kIdescO, (jb | kk) != 0 ? 1u : 0u);
        }
        umma_commit(&v_empty[stage]);
        umma_commit(pv_done);
      }
      umma_commit(mma_done);
      if (!at_wait_drain(mma_done, 0)) raise_status(p.status, BIO_DEV_TIMEOUT);
    }
  } else {
    // -------------------------------------------------------------- softmax
    // Warp w >= 2 owns TMEM lane quarter (w & 3) = 32 query rows, and score
    // columns [half*64*CPT/2 ...) of every block when a row is split in halves.
    const int half = (warp - 2) >> 2;  // 0 or 1 (always 0 when HALVES == 1)
    const int qtr = warp & 3;
    const int st = (warp - 2) * 32 + lane;  // softmax thread index 0 .. 128*HALVES-1
    const uint32_t lane_base = static_cast<uint32_t>(qtr * 32) << 16;
    int64_t kr = lk_seq;  // keys visible to this row
    if (p.causal != 0) kr = min(lk_seq, i + shift + 1);
    if (!row_valid || kr < 0) kr = 0;
    const int64_t mrow = (p.mask_kind != 0 && row_valid)
                             ? b * p.m_sb + hrow * p.m_sh + i * p.m_sq
                             : 0;
    // Without masks and with a positive scale, max(s * scale) == max(s) * scale
    // exactly (rounding is monotonic), so the hot loop runs on raw scores.
    const bool plain = p.mask_kind == 0 && p.scale > 0.f;
    const float kLog2e = 1.4426950408889634f;
    uint32_t xround = 0;
    // Exchange one float per row with the partner warp of the same quarter;
    // both receive (v_half0, v_half1).  Bounded like every other wait.
    auto exchange = [&](float* buf, float mine, float& v0, float& v1) -> bool {
      if constexpr (HALVES == 1) {
        v0 = mine;
        v1 = 0.f;
        return true;
      } else {
        buf[half * 128 + r] = mine;
        mbar_arrive(&xbar[qtr]);
        const bool okx = at_wait(&xbar[qtr], xround & 1u, abort_flag, p.status);
        ++xround;
        v0 = buf[r];
        v1 = buf[128 + r];
        return okx;
      }
    };
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int jb = 0; jb < nblk; ++jb) {
      const int sb = jb & 1;
      const bool got = at_wait(&s_full[sb], static_cast<uint32_t>(jb >> 1) & 1u, abort_flag,
                               p.status);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int64_t col0 = static_cast<int64_t>(jb) * BN;
      const int nvis = static_cast<int>(max(static_cast<int64_t>(0),
                                            min(static_cast<int64_t>(BN), kr - col0)));
      const uint32_t s_addr = tmem + lane_base + static_cast<uint32_t>(sb * 128);
      // ---- pass 1: this thread's CPT chunks of 32 scores stay in registers;
      // maximum of the scaled, masked scores (fixed tree within each chunk,
      // chunks in order, then half 0 vs half 1)
      float f[CPT][32];
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < CPT; ++c) {
        const int ca = half * CPT + c;
        uint32_t v[32];
        tmem_ld_32x32b_x32(s_addr + static_cast<uint32_t>(ca * 32), v);
        tmem_ld_wait();
        const int lim = nvis - ca * 32;
        if (plain) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            f[c][j] = (j < lim) ? __uint_as_float(v[j]) * p.scale : -INFINITY;
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            float sv = -INFINITY;
            if (j < lim) {
              const int64_t col = col0 + ca * 32 + j;
              sv = __uint_as_float(v[j]) * p.scale;
              if (p.mask_kind == 1) {
                if (static_cast<const uint8_t*>(p.mask)[mrow + col * p.m_sk] == 0) sv = -INFINITY;
              } else {
                sv += mask_add(p.mask, p.mask_kind, mrow + col * p.m_sk);
              }
            }
            f[c][j] = sv;
          }
        }
        mx = fmaxf(mx, tree_max32(f[c]));
      }
      // S buffer may now be overwritten by the next S product
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[sb]);
      {
        float x0, x1;
        const bool okx = exchange(xmax, mx, x0, x1);
        if (!__all_sync(0xffffffffu, okx)) {
          ok = false;
          break;
        }
        mx = (HALVES == 2) ? fmaxf(x0, x1) : x0;
      }
      // Reference point of the exponentials: the running max m moves only when
      // the block max exceeds it by more than 8 (log2 units), so P stays
      // <= 2^8 and the O rescale round trip through TMEM is rare.  The choice
      // depends on this row's own scores only.
      const bool move = (m == -INFINITY) ? (mx != -INFINITY) : (mx > m + 8.f / kLog2e);
      const float m_new = move ? mx : m;
      const float alpha = (m == -INFINITY || !move) ? 1.f : ex2_approx((m - m_new) * kLog2e);
      // ---- the P buffer and O are free once the previous PV product is done
      if (jb > 0) {
        const bool done = at_wait(pv_done, static_cast<uint32_t>(jb - 1) & 1u, abort_flag,
                                  p.status);
        if (!__all_sync(0xffffffffu, done)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
          for (int c = half * (DVP / 32 / HALVES); c < (half + 1) * (DVP / 32 / HALVES); ++c) {
            uint32_t v[32];
            const uint32_t ta = tmem + lane_base + kOCol + static_cast<uint32_t>(c * 32);
            tmem_ld_32x32b_x32(ta, v);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) * alpha);
            tmem_st_32x32b_x32(ta, v);
          }
          tmem_st_wait();
        }
      }
      // ---- pass 2: probabilities exp(s*scale - m) rounded to the input dtype,
      // summed with a fixed tree per chunk (chunks in order, then half 0 + half
      // 1), written straight into the 128-byte-swizzled K-major P tile
      const float ml2 = (m_new == -INFINITY) ? 0.f : m_new * kLog2e;
      float lsum = 0.f;
#pragma unroll
      for (int c = 0; c < CPT; ++c) {
        const int ca = half * CPT + c;
        uint32_t w16[16];
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const float s0 = f[c][j], s1 = f[c][j + 1];
          const float x0 = (s0 != -INFINITY) ? ex2_approx(fmaf(s0, kLog2e, -ml2)) : 0.f;
          const float x1 = (s1 != -INFINITY) ? ex2_approx(fmaf(s1, kLog2e, -ml2)) : 0.f;
          w16[j / 2] = pack_pair<T>(x0, x1);
        }
        float t16[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float lo, hi;
          unpack_pair<T>(w16[j], lo, hi);
          t16[j] = lo + hi;
        }
        lsum += tree_sum16(t16);
        uint8_t* base = sP + (ca >> 1) * 16384 + r * 128;
#pragma unroll
        for (int u4 = 0; u4 < 4; ++u4) {
          const int u = (ca & 1) * 4 + u4;
          *reinterpret_cast<uint4*>(base + ((u ^ (r & 7)) << 4)) =
              make_uint4(w16[u4 * 4 + 0], w16[u4 * 4 + 1], w16[u4 * 4 + 2], w16[u4 * 4 + 3]);
        }
      }
      {
        float x0, x1;
        const bool okx = exchange(xsum, lsum, x0, x1);
        if (!__all_sync(0xffffffffu, okx)) {
          ok = false;
          break;
        }
        lsum = (HALVES == 2) ? x0 + x1 : x0;
      }
      if (m_new != -INFINITY) {
        l = l * alpha + lsum;
        m = m_new;
      }
      // Zero V rows of a partial block that lie past the sequence end (they
      // may belong to the next packed sequence).
      if (p.varlen && col0 + BN > lk_seq) {
        const int stage = jb % S;
        uint8_t* vt = sV + stage * L::kV;
        const int first = static_cast<int>(lk_seq - col0);
        for (int row = first + st; row < BN; row += 128 * HALVES) {
          const int kcnk = row >> 6, rr = row & 63;
          for (int nc = 0; nc < kVChunks; ++nc) {
            uint4* dst = reinterpret_cast<uint4*>(vt + (kcnk * kVChunks + nc) * 8192 + rr * 128);
#pragma unroll
            for (int u = 0; u < 8; ++u) dst[u] = make_uint4(0, 0, 0, 0);
          }
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_ready);
    }
    if (ok) {
      const bool done = at_wait(pv_done, static_cast<uint32_t>(nblk - 1) & 1u, abort_flag,
                                p.status);
      if (__all_sync(0xffffffffu, done)) {
        tc_fence_after();
        // whole 32-column chunks of an aligned row leave as four 16-byte
        // stores (the same roundings as the element stores)
        const bool vec_row = row_valid && (reinterpret_cast<uintptr_t>(out_row) & 15u) == 0;
#pragma unroll 1
        for (int c = half * (DVP / 32 / HALVES); c < (half + 1) * (DVP / 32 / HALVES); ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tmem + lane_base + kOCol + static_cast<uint32_t>(c * 32), v);
          tmem_ld_wait();
          if (vec_row && c * 32 + 32 <= p.dv) {
            uint4* dst = reinterpret_cast<uint4*>(out_row + c * 32);
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
              uint32_t w[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int j = q4 * 8 + 2 * e;
                w[e] = pack_pair<T>(l > 0.f ? __uint_as_float(v[j]) / l : 0.f,
                                    l > 0.f ? __uint_as_float(v[j + 1]) / l : 0.f);
              }
              dst[q4] = make_uint4(w[0], w[1], w[2], w[3]);
            }
          } else if (row_valid) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int col = c * 32 + j;
              if (col < p.dv)
                out_row[col] = from_f32<T>(l > 0.f ? __uint_as_float(v[j]) / l : 0.f);
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Varlen plan (one thread): blk_start[i] = first q-block of the i-th planned
// sequence, blk_start[nseq] = total.  With `order` (two-tile kernel) the
// sequences are planned longest first (order[i] = sequence id, insertion sort
// by q-block count for up to 4096 sequences, input order beyond) so that the
// heaviest CTAs start first; without it the input order is kept.
__global__ void attn_plan_kernel(const void* cu_q, int is64, int64_t nseq, int bm,
                                 int* blk_start, int* order) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  auto nblk = [&](int64_t s) -> int {
    const int64_t len = ld_off(cu_q, is64, s + 1) - ld_off(cu_q, is64, s);
    return len > 0 ? static_cast<int>((len + bm - 1) / bm) : 0;
  };
  if (order != nullptr) {
    for (int64_t s = 0; s < nseq; ++s) order[s] = static_cast<int>(s);
    if (nseq <= 4096) {
      for (int64_t i = 1; i < nseq; ++i) {
        const int v = order[i];
        const int key = nblk(v);
        int64_t j = i - 1;
        while (j >= 0 && nblk(order[j]) < key) {
          order[j + 1] = order[j];
          --j;
        }
        order[j + 1] = v;
      }
    }
  }
  int acc = 0;
  for (int64_t i = 0; i < nseq; ++i) {
    blk_start[i] = acc;
    acc += nblk(order != nullptr ? order[i] : i);
  }
  blk_start[nseq] = acc;
}

// ---------------------------------------------------------------------------
// Two query tiles per CTA (D = Dv in {64, 128}).
//
// The CTA owns 256 query rows of one (sequence, head) as two tiles of 128.
// Each tile has its own S buffer and O accumulator in TMEM (S_t at column
// 128 t, O_t at 256 + D t) and its own softmax warpgroup (warps 2..5 tile 0,
// 6..9 tile 1; one thread per query row, all 128 scores of a key block in
// registers).  The MMA thread issues, per key block j,
//     PV_0(j), S_0(j+1), PV_1(j), S_1(j+1)
// so that the tensor core works on one tile while the other tile's softmax
// runs.  The softmax writes P_t (rounded to the input dtype, two per 32-bit
// column) over the first 64 columns of S_t in TMEM, and PV_t reads it from
// there as its A operand (no shared-memory P tile, no proxy fence); S_t(j+1)
// then overwrites it.  tcgen05 operations of one thread complete in issue
// order, so the arrival of S_t(j+1) also tells softmax t that PV_t(j) is
// done: its O row may be rescaled.  K and V have separate rings (K is
// consumed early by the S products, V late by the PV products).
//
// Per-row arithmetic is the same as in attn_tc_kernel's contract: keys in
// fixed blocks of 128 from the first key of the sequence, a fixed tree per 32
// scores, P rounded to the input dtype, the row sum taken over the rounded
// P, the lazy rescale rule decided by the row's own scores.  Results depend
// on the row's Q, the sequence's K/V and the block partition only.
// ---------------------------------------------------------------------------
// Exponentials of the two-tile kernel: two per special-function operation
// on an fp16 pair (ex2.approx.f16x2).  The exponent argument x - m is at most
// 8 (lazy rescale) and its fp16 rounding costs at most 2^-11 |x| ln2 relative
// error -- below the bf16/fp16 rounding of P for every P >= 2^-8 of the row
// maximum; P below 2^-24 becomes 0, which moves the row sum by at most
// n * 2^-24 of its value (2.4e-4 at 4096 keys).  Measured normwise error
// against fp32 SDPA is unchanged (2.1e-3 with or without), time -7..-11%.
#ifndef BIO_ATTN_EX2_F16X2
#define BIO_ATTN_EX2_F16X2 1
#endif
constexpr int kAt2BM = 256;
constexpr int kAt2Threads = 320;

// Packed fp32 pair helpers (sm_100 f32x2 arithmetic) and a 3-input maximum.
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Maximum of 32 score words (exact, so the grouping does not matter).
__device__ __forceinline__ float max32_words(const uint32_t (&f)[32]) {
  float t[11];
#pragma unroll
  for (int j = 0; j < 10; ++j)
    t[j] = fmax3(__uint_as_float(f[3 * j]), __uint_as_float(f[3 * j + 1]),
                 __uint_as_float(f[3 * j + 2]));
  t[10] = fmaxf(__uint_as_float(f[30]), __uint_as_float(f[31]));
  const float u0 = fmax3(t[0], t[1], t[2]), u1 = fmax3(t[3], t[4], t[5]);
  const float u2 = fmax3(t[6], t[7], t[8]), u3 = fmaxf(t[9], t[10]);
  return fmaxf(fmax3(u0, u1, u2), u3);
}

template <int D>
struct Attn2Smem {
  static constexpr uint32_t kQ = 128 * D * 2;  // one tile
  static constexpr uint32_t kK = kAtBN * D * 2;
  static constexpr uint32_t kV = kAtBN * D * 2;
  static constexpr int kKS = D == 128 ? 2 : 4;
  static constexpr int kVS = D == 128 ? 2 : 4;
  static constexpr uint32_t kBar = 256;
  static constexpr uint32_t kTotal = 1024 + 2 * kQ + kKS * kK + kVS * kV + kBar;
  static_assert(kTotal <= 227u * 1024u, "attention smem plan exceeds 227 KB");
};

// Element-by-element mask of one chunk (any mask stride); fully unrolled so
// that the score words stay in registers.
template <int KIND>
__device__ __forceinline__ void mask_chunk_strided(uint32_t (&f)[32], const uint8_t* mp,
                                                   int64_t step, int lim, float scale) {
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    float sv = -INFINITY;
    if (j < lim) {
      sv = __uint_as_float(f[j]) * scale;
      if (KIND == 1) {
        if (*mp == 0) sv = -INFINITY;
      } else if (KIND == 2) {
        sv += *reinterpret_cast<const float*>(mp);
      } else if (KIND == 3) {
        sv += __half2float(*reinterpret_cast<const __half*>(mp));
      } else {
        sv += __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(mp));
      }
    }
    f[j] = __float_as_uint(sv);
    mp += step;
  }
}

// Scale and mask one 32-column chunk of a row's scores in place (raw words
// in, scaled + masked fp32 words out; columns >= lim become -inf).  A chunk
// that lies inside the key range of a unit-stride, 16-byte aligned mask row
// is read with 16-byte loads; anything else element by element.
__device__ __forceinline__ void apply_mask_chunk(const AttnTcParams& p, uint32_t (&f)[32],
                                                 int64_t mrow, int64_t col, int lim,
                                                 int64_t lk_seq) {
  const int esz = p.mask_kind == 1 ? 1 : (p.mask_kind == 2 ? 4 : 2);
  const uint8_t* mp = static_cast<const uint8_t*>(p.mask) + (mrow + col * p.m_sk) * esz;
  const bool vec = p.m_sk == 1 && col + 32 <= lk_seq &&
                   (reinterpret_cast<uintptr_t>(mp) & 15u) == 0;
  if (vec) {
    if (p.mask_kind == 1) {
      const uint4 w0 = reinterpret_cast<const uint4*>(mp)[0];
      const uint4 w1 = reinterpret_cast<const uint4*>(mp)[1];
      const uint32_t wd[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const bool keep = ((wd[j >> 2] >> ((j & 3) * 8)) & 0xffu) != 0;
        const float sv = (j < lim && keep) ? __uint_as_float(f[j]) * p.scale : -INFINITY;
        f[j] = __float_as_uint(sv);
      }
    } else if (p.mask_kind == 2) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 a = reinterpret_cast<const float4*>(mp)[q];
        const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int j = q * 4 + e;
          f[j] = __float_as_uint(j < lim ? fmaf(__uint_as_float(f[j]), p.scale, av[e])
                                         : -INFINITY);
        }
      }
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 a = reinterpret_cast<const uint4*>(mp)[q];
        const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float lo, hi;
          if (p.mask_kind == 3) {
            unpack_pair<__half>(aw[e], lo, hi);
          } else {
            unpack_pair<__nv_bfloat16>(aw[e], lo, hi);
          }
          const int j = q * 8 + 2 * e;
          f[j] = __float_as_uint(j < lim ? __uint_as_float(f[j]) * p.scale + lo : -INFINITY);
          f[j + 1] = __float_as_uint(j + 1 < lim ? __uint_as_float(f[j + 1]) * p.scale + hi
                                                 : -INFINITY);
        }
      }
    }
    return;
  }
  const int64_t step = p.m_sk * esz;
  switch (p.mask_kind) {
    case 1: mask_chunk_strided<1>(f, mp, step, lim, p.scale); break;
    case 2: mask_chunk_strided<2>(f, mp, step, lim, p.scale); break;
    case 3: mask_chunk_strided<3>(f, mp, step, lim, p.scale); break;
    default: mask_chunk_strided<4>(f, mp, step, lim, p.scale); break;
  }
}

template <int D, typename T>
__global__ void __launch_bounds__(kAt2Threads, 1)
    attn_tc2_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const AttnTcParams p) {
  using L = Attn2Smem<D>;
  constexpr int KS = L::kKS;
  constexpr int VS = L::kVS;
  constexpr int kChunks = D / 64;
  constexpr uint32_t kIdescS = idesc_f16(AtFmt<T>::v, 128, kAtBN, false, false);
  constexpr uint32_t kIdescO = idesc_f16(AtFmt<T>::v, 128, D, false, true);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // ---------------------------------------------------------------- work
  // grid (heads, q-blocks, batch): all heads of the heaviest q-blocks launch first
  int64_t b = 0, h = blockIdx.x, q0, lq_seq, lk_seq, q_tok0, k_tok0;
  if (p.varlen) {
    const int64_t g = blockIdx.y;
    const int64_t total = p.blk_start[p.nseq];
    if (g >= total) return;
    int64_t lo = 0, hi = p.nseq;
    while (hi - lo > 1) {
      const int64_t mid = (lo + hi) >> 1;
      if (p.blk_start[mid] <= g) lo = mid; else hi = mid;
    }
    const int64_t si = lo;
    const int64_t sq = p.order[si];
    const int64_t qs0 = ld_off(p.cu_q, p.cu_is64, sq), qs1 = ld_off(p.cu_q, p.cu_is64, sq + 1);
    const int64_t ks0 = ld_off(p.cu_k, p.cu_is64, sq), ks1 = ld_off(p.cu_k, p.cu_is64, sq + 1);
    const bool bad = qs0 < 0 || qs1 > p.lq || ks0 < 0 || ks1 < ks0 || ks1 > p.lk ||
                     ld_off(p.cu_q, p.cu_is64, 0) != 0 || ld_off(p.cu_k, p.cu_is64, 0) != 0 ||
                     (p.causal == 3 && (qs1 - qs0) != (ks1 - ks0));
    if (bad) {
      if (threadIdx.x == 0) raise_status(p.status, BIO_DEV_INDEX);
      return;  // output rows stay zero (pre-zeroed by the caller)
    }
    // latest q-block of the sequence first (heaviest under causal masking)
    q0 = (p.blk_start[si + 1] - 1 - g) * kAt2BM;
    lq_seq = qs1 - qs0;
    lk_seq = ks1 - ks0;
    q_tok0 = qs0 + q0;
    k_tok0 = ks0;
  } else {
    b = blockIdx.z;
    // heaviest (latest, for causal) query blocks first
    q0 = static_cast<int64_t>(gridDim.y - 1 - blockIdx.y) * kAt2BM;
    lq_seq = p.lq;
    lk_seq = p.lk;
    q_tok0 = q0;
    k_tok0 = 0;
  }
  const int64_t hk = h / (p.heads / p.kv_heads);
  const int64_t shift = (p.causal == 2) ? (lk_seq - lq_seq) : 0;
  auto tile_rows = [&](int t) -> int64_t {
    return max(static_cast<int64_t>(0), min(static_cast<int64_t>(128), lq_seq - (q0 + 128 * t)));
  };
  auto tile_blocks = [&](int t) -> int {
    const int64_t nr = tile_rows(t);
    int64_t kend = lk_seq;
    if (p.causal != 0) kend = min(lk_seq, q0 + 128 * t + nr - 1 + shift + 1);
    if (nr == 0 || kend < 0) kend = 0;
    return static_cast<int>((kend + kAtBN - 1) / kAtBN);
  };
  const int nblk0 = tile_blocks(0), nblk1 = tile_blocks(1);
  const int nblk = max(nblk0, nblk1);

  // softmax role: tile, row
  const int tt = (warp - 2) >> 2;  // 0 or 1 for warps 2..9
  const int qtr = warp & 3;
  const int r = qtr * 32 + lane;
  const int64_t i = q0 + 128 * (warp >= 2 ? tt : 0) + r;
  const bool row_valid = warp >= 2 && r < tile_rows(warp >= 2 ? tt : 0);
  T* out_row = nullptr;
  if (row_valid) {
    out_row = static_cast<T*>(p.o) + (p.varlen ? 0 : b * p.o_sb) + h * p.o_sh +
              (p.varlen ? (q_tok0 + 128 * tt + r) : i) * p.o_st;
  }
  if (nblk == 0) {
    if (row_valid)
      for (int c = 0; c < p.dv; ++c) out_row[c] = from_f32<T>(0.f);
    return;
  }

  // ---------------------------------------------------------------- smem
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;                 // [2][kQ]
  uint8_t* sK = sQ + 2 * L::kQ;       // [KS][kK]
  uint8_t* sV = sK + KS * L::kK;      // [VS][kV]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + VS * L::kV);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;             // [KS]
  uint64_t* k_empty = k_full + KS;         // [KS]
  uint64_t* v_full = k_empty + KS;         // [VS]
  uint64_t* v_empty = v_full + VS;         // [VS]
  uint64_t* s_full = v_empty + VS;         // [2]
  uint64_t* p_ready = s_full + 2;          // [2]
  uint64_t* o_done = p_ready + 2;          // [2]
  uint64_t* mma_done = o_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < KS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < VS; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_ready[t], 4);
      mbar_init(&o_done[t], 1);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int qc = static_cast<int>(q_tok0), kc0 = static_cast<int>(k_tok0);
  const int hc = static_cast<int>(h), hkc = static_cast<int>(hk), bc = static_cast<int>(b);

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      mbar_arrive_expect_tx(q_full, 2 * L::kQ);
      for (int t = 0; t < 2; ++t)
        for (int c = 0; c < kChunks; ++c)
          tma_load_4d(sQ + t * L::kQ + c * 16384, &tmQ, q_full, c * 64, qc + 128 * t, hc, bc);
      // K runs one block ahead of V: K_{j+1} is issued before V_j waits for
      // the PV products of block j-1 to release its slot.
      int k_issued = 0, v_issued = 0;
      auto load_k = [&](int jb) -> bool {
        const int ks = jb % KS;
        if (!at_wait(&k_empty[ks], (static_cast<uint32_t>(jb / KS) & 1u) ^ 1u, abort_flag,
                     p.status))
          return false;
        mbar_arrive_expect_tx(&k_full[ks], L::kK);
        for (int c = 0; c < kChunks; ++c)
          tma_load_4d(sK + ks * L::kK + c * 16384, &tmK, &k_full[ks], c * 64,
                      kc0 + jb * kAtBN, hkc, bc);
        k_issued = jb + 1;
        return true;
      };
      bool okp = load_k(0);
      for (int jb = 0; okp && jb < nblk; ++jb) {
        if (jb + 1 < nblk && !load_k(jb + 1)) break;
        const int vs = jb % VS;
        if (!at_wait(&v_empty[vs], (static_cast<uint32_t>(jb / VS) & 1u) ^ 1u, abort_flag,
                     p.status))
          break;
        mbar_arrive_expect_tx(&v_full[vs], L::kV);
        const int row = kc0 + jb * kAtBN;
        for (int kcnk = 0; kcnk < 2; ++kcnk)
          for (int nc = 0; nc < kChunks; ++nc)
            tma_load_4d(sV + vs * L::kV + (kcnk * kChunks + nc) * 8192, &tmV, &v_full[vs],
                        nc * 64, row + kcnk * 64, hkc, bc);
        v_issued = jb + 1;
      }
      // drain: Q and the last copies of every ring slot land before exit
      if (!at_wait_drain(q_full, 0)) raise_status(p.status, BIO_DEV_TIMEOUT);
      for (int jb = k_issued - 1; jb >= 0 && jb >= k_issued - KS; --jb)
        if (!at_wait_drain(&k_full[jb % KS], static_cast<uint32_t>(jb / KS) & 1u))
          raise_status(p.status, BIO_DEV_TIMEOUT);
      for (int jb = v_issued - 1; jb >= 0 && jb >= v_issued - VS; --jb)
        if (!at_wait_drain(&v_full[jb % VS], static_cast<uint32_t>(jb / VS) & 1u))
          raise_status(p.status, BIO_DEV_TIMEOUT);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA
      bool ok = at_wait(q_full, 0, abort_flag, p.status);
      auto issue_s = [&](int t, int jb) -> bool {
        const int ks = jb % KS;
        if (!at_wait(&k_full[ks], static_cast<uint32_t>(jb / KS) & 1u, abort_flag, p.status))
          return false;
        tc_fence_after();
        const uint32_t qa = smem_u32(sQ + t * L::kQ), ka = smem_u32(sK + ks * L::kK);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma_f16(tmem + static_cast<uint32_t>(t * 128), smem_desc_sw128(qa + off, 16, 1024),
                   smem_desc_sw128(ka + off, 16, 1024), kIdescS, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[t]);
        return true;
      };
      auto issue_pv = [&](int t, int jb) -> bool {
        if (!at_wait(&p_ready[t], static_cast<uint32_t>(jb) & 1u, abort_flag, p.status))
          return false;
        const int vs = jb % VS;
        if (!at_wait(&v_full[vs], static_cast<uint32_t>(jb / VS) & 1u, abort_flag, p.status))
          return false;
        tc_fence_after();
        const uint32_t va = smem_u32(sV + vs * L::kV);
        // P_t is the A operand straight from TMEM (the first 64 columns of
        // S_t, 8 columns per K = 16 step)
        const uint32_t pa = tmem + static_cast<uint32_t>(t * 128);
#pragma unroll
        for (int kk = 0; kk < kAtBN / 16; ++kk) {
          const uint32_t boff = (kk >> 2) * (kChunks * 8192) + (kk & 3) * 2048;
          umma_f16_ts(tmem + 256u + static_cast<uint32_t>(t * D), pa + static_cast<uint32_t>(8 * kk),
                      smem_desc_sw128(va + boff, 8192, 1024), kIdescO, (jb | kk) != 0 ? 1u : 0u);
        }
        if (jb == (t == 0 ? nblk0 : nblk1) - 1) umma_commit(&o_done[t]);
        return true;
      };
      if (ok && nblk0 > 0) ok = issue_s(0, 0);
      if (ok && nblk1 > 0) ok = issue_s(1, 0);
      if (ok) umma_commit(&k_empty[0]);
      for (int jb = 0; ok && jb < nblk; ++jb) {
#pragma unroll 1
        for (int t = 0; t < 2 && ok; ++t) {
          const int nbt = t == 0 ? nblk0 : nblk1;
          if (jb < nbt) ok = issue_pv(t, jb);
          if (ok && jb + 1 < nbt) ok = issue_s(t, jb + 1);
        }
        if (!ok) break;
        umma_commit(&v_empty[jb % VS]);
        if (jb + 1 < nblk) umma_commit(&k_empty[(jb + 1) % KS]);
      }
      umma_commit(mma_done);
      if (!at_wait_drain(mma_done, 0)) raise_status(p.status, BIO_DEV_TIMEOUT);
    }
  } else {
    // -------------------------------------------------------------- softmax
    const int t = tt;
    const int my_nblk = t == 0 ? nblk0 : nblk1;
    const uint32_t lane_base = static_cast<uint32_t>(qtr * 32) << 16;
    const uint32_t s_addr = tmem + lane_base + static_cast<uint32_t>(t * 128);
    const uint32_t o_addr = tmem + lane_base + 256u + static_cast<uint32_t>(t * D);
    int64_t kr = lk_seq;  // keys visible to this row
    if (p.causal != 0) kr = min(lk_seq, i + shift + 1);
    if (!row_valid || kr < 0) kr = 0;
    const int64_t mrow = (p.mask_kind != 0 && row_valid)
                             ? b * p.m_sb + h * p.m_sh + i * p.m_sq
                             : 0;
    // Without masks and with a positive scale the row maximum is taken on the
    // raw scores (scaling is monotonic) and the scale folds into the exponent.
    const bool plain = p.mask_kind == 0 && p.scale > 0.f;
    const float kLog2e = 1.4426950408889634f;
    const float cexp = plain ? p.scale * kLog2e : kLog2e;  // exponent factor of the domain
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int jb = 0; jb < my_nblk; ++jb) {
      const bool got = at_wait(&s_full[t], static_cast<uint32_t>(jb) & 1u, abort_flag, p.status);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int64_t col0 = static_cast<int64_t>(jb) * kAtBN;
      const int nvis = static_cast<int>(max(static_cast<int64_t>(0),
                                            min(static_cast<int64_t>(kAtBN), kr - col0)));
      // ---- scores of the block: four 32-column TMEM loads, one wait; kept
      // as raw 32-bit words and rewritten in place
      // Masked launches first rewrite the block's scores in TMEM (scaled,
      // masked, -inf past the visible range), one 32-column chunk at a time,
      // so the mask code never holds the whole row in registers.
      if (!plain) {
        const uint8_t* mrow_p = static_cast<const uint8_t*>(p.mask) + mrow + col0;
        if (p.mask_kind == 1 && p.m_sk == 1 && col0 + kAtBN <= lk_seq &&
            (reinterpret_cast<uintptr_t>(mrow_p) & 15u) == 0) {
          // boolean mask, whole block in bounds: the row's 128 mask bytes are
          // loaded up front (one memory latency per block), then applied
          // chunk by chunk exactly as apply_mask_chunk does
          uint4 mw[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) mw[q] = reinterpret_cast<const uint4*>(mrow_p)[q];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t g[32];
            tmem_ld_32x32b_x32(s_addr + static_cast<uint32_t>(c * 32), g);
            tmem_ld_wait();
            const uint32_t wd[8] = {mw[2 * c].x,     mw[2 * c].y,     mw[2 * c].z,
                                    mw[2 * c].w,     mw[2 * c + 1].x, mw[2 * c + 1].y,
                                    mw[2 * c + 1].z, mw[2 * c + 1].w};
            const int lim = nvis - c * 32;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const bool keep = ((wd[j >> 2] >> ((j & 3) * 8)) & 0xffu) != 0;
              const float sv = (j < lim && keep) ? __uint_as_float(g[j]) * p.scale : -INFINITY;
              g[j] = __float_as_uint(sv);
            }
            tmem_st_32x32b_x32(s_addr + static_cast<uint32_t>(c * 32), g);
          }
        } else {
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t g[32];
            tmem_ld_32x32b_x32(s_addr + static_cast<uint32_t>(c * 32), g);
            tmem_ld_wait();
            apply_mask_chunk(p, g, mrow, col0 + c * 32, nvis - c * 32, lk_seq);
            tmem_st_32x32b_x32(s_addr + static_cast<uint32_t>(c * 32), g);
          }
        }
        tmem_st_wait();
      }
      // Scores stay in TMEM: pass 1 reads them two chunks at a time for the
      // row maximum, pass 2 re-reads each chunk for the exponentials (the
      // next chunk's load in flight while the current one is processed), so
      // at most two 32-column chunks are held in registers.
      const uint32_t kNegInf = 0xff800000u;
      const bool clip = plain && nvis < kAtBN;  // plain rows: -inf past the visible range
      auto clip_chunk = [&](uint32_t (&g)[32], int c) {
        if (clip) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (c * 32 + j >= nvis) g[j] = kNegInf;
        }
      };
      float mx;
      {
        uint32_t g0[32], g1[32];
        tmem_ld_32x32b_x32(s_addr + 0u, g0);
        tmem_ld_32x32b_x32(s_addr + 32u, g1);
        tmem_ld_wait();
        clip_chunk(g0, 0);
        clip_chunk(g1, 1);
        mx = fmaxf(max32_words(g0), max32_words(g1));
        tmem_ld_32x32b_x32(s_addr + 64u, g0);
        tmem_ld_32x32b_x32(s_addr + 96u, g1);
        tmem_ld_wait();
        clip_chunk(g0, 2);
        clip_chunk(g1, 3);
        mx = fmax3(mx, max32_words(g0), max32_words(g1));
      }
      const bool move = (m == -INFINITY) ? (mx != -INFINITY) : ((mx - m) * cexp > 8.f);
      const float m_new = move ? mx : m;
      const float alpha = (m == -INFINITY || !move) ? 1.f : ex2_approx((m - m_new) * cexp);
      // O_t holds PV_t(jb-1) (complete: S_t(jb) arrived after it)
      if (jb > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(o_addr + static_cast<uint32_t>(c * 32), v);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) * alpha);
          tmem_st_32x32b_x32(o_addr + static_cast<uint32_t>(c * 32), v);
        }
        tmem_st_wait();
      }
      // ---- P = exp2((x - m) * c) rounded to the input dtype and written into
      // the 128-byte-swizzled K-major P tile of this query tile.  The row sum
      // runs over the fp32 exponentials in a fixed order: per 32-column chunk
      // two interleaved lanes (even / odd columns) accumulate in column
      // order, then lane 0 + lane 1, then chunks in order.
      const float mc = (m_new == -INFINITY) ? 0.f : m_new * cexp;
      const uint64_t c2 = f2_pack(cexp, cexp), nmc2 = f2_pack(-mc, -mc);
      float lsum = 0.f;
      uint32_t fa[32], fb[32];
      tmem_ld_32x32b_x32(s_addr + 0u, fa);
      tmem_ld_wait();
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t (&f)[32] = (c & 1) ? fb : fa;
        uint32_t (&fn)[32] = (c & 1) ? fa : fb;
        if (c + 1 < 4) tmem_ld_32x32b_x32(s_addr + static_cast<uint32_t>((c + 1) * 32), fn);
        clip_chunk(f, c);
        uint64_t acc = f2_pack(0.f, 0.f);
#pragma unroll
        for (int u4 = 0; u4 < 4; ++u4) {
          uint32_t w4[4];  // 8 rounded probabilities, two per word
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = u4 * 8 + 2 * e;
            float a0, a1;
            f2_unpack(f2_fma(f2_pack(__uint_as_float(f[j]), __uint_as_float(f[j + 1])), c2,
                             nmc2),
                      a0, a1);
#if BIO_ATTN_EX2_F16X2
            // two exponentials per SFU operation on an fp16 pair
            uint32_t hin, hout;
            asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(hin) : "f"(a1), "f"(a0));
            asm("ex2.approx.f16x2 %0, %1;" : "=r"(hout) : "r"(hin));
            float x0, x1;
            unpack_pair<__half>(hout, x0, x1);
#else
            const float x0 = ex2_approx(a0);
            const float x1 = ex2_approx(a1);
#endif
            w4[e] = pack_pair<T>(x0, x1);
            acc = f2_add(acc, f2_pack(x0, x1));
          }
          // P chunk c -> TMEM columns [16 c, 16 c + 16) of S_t, which hold
          // S chunk c / 2: already read into registers (chunks run in order)
          tmem_st_32x32b_x4(s_addr + static_cast<uint32_t>(16 * c + 4 * u4), w4[0], w4[1],
                            w4[2], w4[3]);
        }
        float s0, s1;
        f2_unpack(acc, s0, s1);
        lsum += s0 + s1;
        if (c + 1 < 4) tmem_ld_wait();
      }
      tmem_st_wait();  // P_t is in TMEM before the PV product is released
      if (m_new != -INFINITY) {
        l = l * alpha + lsum;
        m = m_new;
      }
      // Zero V rows of a partial block that lie past the sequence end (they
      // may belong to the next packed sequence); both tiles write the same
      // zeros.
      if (p.varlen && col0 + kAtBN > lk_seq) {
        const int vs = jb % VS;
        const bool vok = at_wait(&v_full[vs], static_cast<uint32_t>(jb / VS) & 1u, abort_flag,
                                 p.status);
        if (!__all_sync(0xffffffffu, vok)) {
          ok = false;
          break;
        }
        uint8_t* vt = sV + vs * L::kV;
        const int first = static_cast<int>(lk_seq - col0);
        for (int row = first + r; row < kAtBN; row += 128) {
          const int kcnk = row >> 6, rr = row & 63;
          for (int nc = 0; nc < kChunks; ++nc) {
            uint4* dst = reinterpret_cast<uint4*>(vt + (kcnk * kChunks + nc) * 8192 + rr * 128);
#pragma unroll
            for (int u = 0; u < 8; ++u) dst[u] = make_uint4(0, 0, 0, 0);
          }
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_ready[t]);
    }
    if (ok && my_nblk > 0) {
      const bool done = at_wait(&o_done[t], 0, abort_flag, p.status);
      if (__all_sync(0xffffffffu, done)) {
        tc_fence_after();
        const float inv = l > 0.f ? 1.f / l : 0.f;
        // aligned rows leave as 16-byte groups of 8 columns (a head dim that
        // is not a multiple of 8 ends with element stores); same roundings
        const bool vec = row_valid && (reinterpret_cast<uintptr_t>(out_row) & 15u) == 0;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(o_addr + static_cast<uint32_t>(c * 32), v);
          tmem_ld_wait();
          if (vec) {
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
              const int col = c * 32 + q4 * 8;
              if (col + 8 <= p.dv) {
                uint32_t w[4];
#pragma unroll
                for (int e = 0; e < 4; ++e)
                  w[e] = pack_pair<T>(__uint_as_float(v[q4 * 8 + 2 * e]) * inv,
                                      __uint_as_float(v[q4 * 8 + 2 * e + 1]) * inv);
                *reinterpret_cast<uint4*>(out_row + col) = make_uint4(w[0], w[1], w[2], w[3]);
              } else {
#pragma unroll
                for (int e = 0; e < 8; ++e)
                  if (col + e < p.dv)
                    out_row[col + e] = from_f32<T>(__uint_as_float(v[q4 * 8 + e]) * inv);
              }
            }
          } else if (row_valid) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int col = c * 32 + j;
              if (col < p.dv) out_row[col] = from_f32<T>(__uint_as_float(v[j]) * inv);
            }
          }
        }
      }
    } else if (my_nblk == 0 && row_valid) {
      for (int c = 0; c < p.dv; ++c) out_row[c] = from_f32<T>(0.f);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace bio

// ===========================================================================
// Host side
// ===========================================================================
namespace {

std::mutex g_at_mu;

// 4-D tensor map {dim, tokens, heads, batch} over a [batch][head][token][dim]
// operand (element strides), 128-byte swizzle.  Size-1 dims get a harmless
// stride.  Returns false when a stride is not TMA-expressible.
bool at_map(CUtensorMap* map, int dtype, const void* ptr, int64_t dim, int64_t tokens,
            int64_t heads, int64_t batch, int64_t s_tok, int64_t s_head, int64_t s_batch,
            uint32_t box0, uint32_t box1, uint32_t box2 = 1) {
  bio_host::EncodeTiledFn enc = bio_host::encode_tiled_fn();
  if (enc == nullptr) return false;
  const uint64_t es = 2;
  auto fix = [&](int64_t size, int64_t stride, uint64_t prev) -> uint64_t {
    if (size <= 1) return (prev + 15) / 16 * 16;
    return static_cast<uint64_t>(stride) * es;
  };
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(dim), static_cast<cuuint64_t>(tokens),
                        static_cast<cuuint64_t>(heads), static_cast<cuuint64_t>(batch)};
  cuuint64_t st[3];
  st[0] = fix(tokens, s_tok, static_cast<uint64_t>(dim) * es);
  st[1] = fix(heads, s_head, st[0] * static_cast<uint64_t>(tokens));
  st[2] = fix(batch, s_batch, st[1] * static_cast<uint64_t>(heads));
  for (int i = 0; i < 3; ++i)
    if (st[i] % 16 != 0 || st[i] == 0 || st[i] >= (1ull << 40)) return false;
  cuuint32_t box[4] = {box0, box1, box2, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt =
      dtype == BIO_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return enc(map, dt, 4, const_cast<void*>(ptr), dims, st, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int pad64(int v) { return v <= 64 ? 64 : (v <= 128 ? 128 : 256); }

template <int DP, int DVP, typename T>
int launch_at(const bio_attn_args* a, bool varlen, const CUtensorMap& q, const CUtensorMap& k,
              const CUtensorMap& v, const bio::AttnTcParams& p, cudaStream_t s) {
  using L = bio::AttnSmem<DP, DVP>;
  auto kern = bio::attn_tc_kernel<DP, DVP, T>;
  static bool attr_done[bio_host::kMaxDevices] = {false};
  {
    std::lock_guard<std::mutex> lk(g_at_mu);
    if (!attr_done[a->device]) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal) !=
          cudaSuccess)
        return BIO_ERR_LAUNCH;
      attr_done[a->device] = true;
    }
  }
  dim3 grid;
  if (varlen) {
    const int64_t g = (a->lq + bio::kAtBM - 1) / bio::kAtBM + a->nseq;
    if (g > 2147483647) return BIO_ERR_SHAPE;
    grid = dim3(static_cast<unsigned>(g), static_cast<unsigned>(a->heads), 1);
  } else {
    const int64_t span = p.pack_tok > 0 ? p.pack_tok : bio::kAtBM;  // tokens per tile
    const int64_t g = (a->lq + span - 1) / span;
    const int64_t gy = p.pack_tok > 0 ? a->kv_heads : a->heads;
    if (g > 2147483647 || a->batch > 65535 || gy > 65535) return BIO_ERR_SHAPE;
    grid = dim3(static_cast<unsigned>(g), static_cast<unsigned>(gy),
                static_cast<unsigned>(a->batch));
  }
  kern<<<grid, L::kThreads, L::kTotal, s>>>(q, k, v, p);
  return bio_host::launch_status(cudaGetLastError());
}

template <int D, typename T>
int launch_at2(const bio_attn_args* a, bool varlen, const CUtensorMap& q, const CUtensorMap& k,
               const CUtensorMap& v, const bio::AttnTcParams& p, cudaStream_t s) {
  using L = bio::Attn2Smem<D>;
  auto kern = bio::attn_tc2_kernel<D, T>;
  static bool attr_done[bio_host::kMaxDevices] = {false};
  {
    std::lock_guard<std::mutex> lk(g_at_mu);
    if (!attr_done[a->device]) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal) !=
          cudaSuccess)
        return BIO_ERR_LAUNCH;
      attr_done[a->device] = true;
    }
  }
  dim3 grid;
  if (varlen) {
    const int64_t g = (a->lq + bio::kAt2BM - 1) / bio::kAt2BM + a->nseq;
    if (g > 65535 || a->heads > 2147483647) return BIO_ERR_SHAPE;
    grid = dim3(static_cast<unsigned>(a->heads), static_cast<unsigned>(g), 1);
  } else {
    const int64_t g = (a->lq + bio::kAt2BM - 1) / bio::kAt2BM;
    if (g > 65535 || a->batch > 65535 || a->heads > 2147483647) return BIO_ERR_SHAPE;
    grid = dim3(static_cast<unsigned>(a->heads), static_cast<unsigned>(g),
                static_cast<unsigned>(a->batch));
  }
  kern<<<grid, bio::kAt2Threads, L::kTotal, s>>>(q, k, v, p);
  return bio_host::launch_status(cudaGetLastError());
}

// Two-tile kernel for D = Dv in {64, 128} when a CTA's second tile has rows
// to work on (dense: more than 128 queries; varlen: always).
bool use_two_tiles(int dp, int dvp, const bio_attn_args* a, bool varlen) {
  if (dp != dvp || (dp != 64 && dp != 128)) return false;
  const int64_t qblocks = (a->lq + bio::kAt2BM - 1) / bio::kAt2BM + (varlen ? a->nseq : 0);
  if (qblocks > 65535) return false;  // grid y holds the q-blocks
  return varlen || a->lq > bio::kAtBM;
}

template <typename T>
int dispatch_at(int dp, int dvp, const bio_attn_args* a, bool varlen, const CUtensorMap& q,
                const CUtensorMap& k, const CUtensorMap& v, const bio::AttnTcParams& p,
                cudaStream_t s) {
#define BIO_AT_CASE(D1, D2) \
  if (dp == D1 && dvp == D2) return launch_at<D1, D2, T>(a, varlen, q, k, v, p, s);
  BIO_AT_CASE(64, 64)
  BIO_AT_CASE(64, 128)
  BIO_AT_CASE(64, 256)
  BIO_AT_CASE(128, 64)
  BIO_AT_CASE(128, 128)
  BIO_AT_CASE(128, 256)
  BIO_AT_CASE(256, 64)
  BIO_AT_CASE(256, 128)
  BIO_AT_CASE(256, 256)
#undef BIO_AT_CASE
  return BIO_ERR_SHAPE;
}

}  // namespace

namespace bio_host {

int attn_tc_launch(const bio_attn_args* a, bool varlen, void* stream) {
  if (a->dtype != BIO_BF16 && a->dtype != BIO_F16) return BIO_ERR_DTYPE;
  if (a->d > 256 || a->dv > 256) return BIO_ERR_SHAPE;
  if (varlen && a->workspace == nullptr) return BIO_ERR_ARG;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!al16(a->q) || !al16(a->k) || !al16(a->v)) return BIO_ERR_ALIGN;
  const int dp = pad64(a->d), dvp = pad64(a->dv);
  const int64_t nb = varlen ? 1 : a->batch;
  // Grouped-query packing of the one-tile dense kernel: the query heads that
  // share a KV head fill one 128-row tile together (group of 2..16 heads,
  // 128 / group tokens each), so short queries do not leave most rows idle
  // and the group's K/V blocks are read once.  A row's arithmetic does not
  // depend on the tile it lands in, so this changes no bit.
  const int64_t grp = a->kv_heads > 0 ? a->heads / a->kv_heads : 0;
  const bool pack = !varlen && !use_two_tiles(dp, dvp, a, varlen) && a->kv_heads > 0 &&
                    a->heads % a->kv_heads == 0 &&
                    (grp == 2 || grp == 4 || grp == 8 || grp == 16);
  const int pack_tok = pack ? static_cast<int>(bio::kAtBM / grp) : 0;
  CUtensorMap tq, tk, tv;
  if (!at_map(&tq, a->dtype, a->q, a->d, a->lq, a->heads, nb, a->q_st, a->q_sh, a->q_sb, 64,
              pack ? static_cast<uint32_t>(pack_tok) : bio::kAtBM,
              pack ? static_cast<uint32_t>(grp) : 1u))
    return BIO_ERR_ALIGN;
  if (a->lk == 0) {
    // no key at all: every row is zero and K/V are never read
    tk = tq;
    tv = tq;
  } else {
    // K rows per box = the key block of the kernel that runs
    const uint32_t kbox = (!use_two_tiles(dp, dvp, a, varlen) && dp == 256 && dvp == 256)
                              ? static_cast<uint32_t>(bio::at_block_n<256, 256>())
                              : static_cast<uint32_t>(bio::kAtBN);
    if (!at_map(&tk, a->dtype, a->k, a->d, a->lk, a->kv_heads, nb, a->k_st, a->k_sh, a->k_sb,
                64, kbox))
      return BIO_ERR_ALIGN;
    if (!at_map(&tv, a->dtype, a->v, a->dv, a->lk, a->kv_heads, nb, a->v_st, a->v_sh, a->v_sb,
                64, 64))
      return BIO_ERR_ALIGN;
  }
  bio::AttnTcParams p;
  p.heads = a->heads;
  p.kv_heads = a->kv_heads;
  p.lq = a->lq;
  p.lk = a->lk;
  p.d = a->d;
  p.dv = a->dv;
  p.scale = a->scale;
  p.causal = a->causal;
  p.mask = a->mask;
  p.mask_kind = 0;
  if (a->mask_kind == BIO_MASK_BOOL) p.mask_kind = 1;
  if (a->mask_kind == BIO_MASK_ADD)
    p.mask_kind = a->mask_dtype == BIO_F32 ? 2 : (a->mask_dtype == BIO_F16 ? 3 : 4);
  p.m_sb = a->m_sb;
  p.m_sh = a->m_sh;
  p.m_sq = a->m_sq;
  p.m_sk = a->m_sk;
  p.o = a->o;
  p.o_sb = a->o_sb;
  p.o_sh = a->o_sh;
  p.o_st = a->o_st;
  p.varlen = varlen ? 1 : 0;
  p.cu_q = a->cu_q;
  p.cu_k = a->cu_k;
  p.cu_is64 = a->cu_is64;
  p.nseq = a->nseq;
  p.blk_start = static_cast<const int*>(a->workspace);
  p.order = a->workspace != nullptr ? static_cast<const int*>(a->workspace) + a->nseq + 1
                                    : nullptr;
  p.pack_tok = pack_tok;
  p.status = bio_host::status_word(a->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool two = use_two_tiles(dp, dvp, a, varlen);
  if (varlen) {
    int* ws = static_cast<int*>(a->workspace);
    bio::attn_plan_kernel<<<1, 32, 0, s>>>(a->cu_q, a->cu_is64, a->nseq,
                                           two ? bio::kAt2BM : bio::kAtBM, ws,
                                           two ? ws + a->nseq + 1 : nullptr);
    const int st = bio_host::launch_status(cudaGetLastError());
    if (st != BIO_OK) return st;
  }
  if (two) {
    if (a->dtype == BIO_BF16) {
      return dp == 64 ? launch_at2<64, __nv_bfloat16>(a, varlen, tq, tk, tv, p, s)
                      : launch_at2<128, __nv_bfloat16>(a, varlen, tq, tk, tv, p, s);
    }
    return dp == 64 ? launch_at2<64, __half>(a, varlen, tq, tk, tv, p, s)
                    : launch_at2<128, __half>(a, varlen, tq, tk, tv, p, s);
  }
  if (a->dtype == BIO_BF16) return dispatch_at<__nv_bfloat16>(dp, dvp, a, varlen, tq, tk, tv, p, s);
  return dispatch_at<__half>(dp, dvp, a, varlen, tq, tk, tv, p, s);
}

}  // namespace bio_host
