// fp32 GEMM on the int8 tensor cores with exact integer slices.
//
// Every row of A (and every column of B) is scaled by a power of two so that
// its largest magnitude lies in [0.25, 0.5), then cut into four signed
// digits in [-64, 64] by repeated round-to-nearest:
//     A[m][k] = 2^ea[m] * sum_{s=0..3} a_s[m][k] * 2^{-7(s+1)}   (+ a tail of
//     at most 2^{ea[m]-29}, unbiased),
// and the same for B with exponents eb[n].  Products of digits are summed by
// tcgen05.mma kind::i8 into int32 TMEM accumulators, which is exact; digit
// pairs with the same weight 2^{-7(s+t+2)} share an accumulator (levels
// s+t = 0..3; pairs with s+t > 3 weigh below 2^{-35} and are dropped).  The
// epilogue combines the four levels in fp64, applies 2^{ea[m]+eb[n]}, alpha
// and the bias, and rounds to fp32 once.
//
// Accuracy: each operand is represented to 2^-27 of its row/column maximum
// with rounding errors of either sign, and the integer sums are exact, so an
// output element is within K * 2^-26 * max|A[m,:]| * max|B[:,n]| of the exact
// product sum (typically far less) -- ~1e-7 normwise on the BASELINE fp32
// shapes, including the cancelling linspace case where every fp32
// accumulation order loses 2e-4.
//
// Batch invariance: ea[m] depends on row m of A only, eb and the B digits on
// B only, the integer sums are exact (independent of tile, order and
// schedule) and the epilogue is elementwise, so every output row depends on
// its own A row and on B, never on the other rows.
//
// Limits: K <= 65536 (level 3 sums four digit products: 4 * K * 64^2 must
// stay below 2^31).  Rows or columns holding Inf/NaN produce NaN outputs.
//
// Reference: matmul_persistent / bmm_persistent fp32 configuration
// (batch_invariant_ops.py:271-431, INPUT_PRECISION "ieee").
#include <mutex>

#include "bio_common.cuh"

namespace bio {

constexpr int kXS = 4;           // digits per operand
constexpr int kXBK = 64;         // k-block: 64 int8 = one 64-byte swizzle row
constexpr int kXBM = 128;
constexpr int kXBN = 128;
constexpr int kXStages = 3;
constexpr int kXPairs = 10;      // digit pairs with s + t <= 3
constexpr int kXThreads = 320;   // warp 0 TMA, warp 1 MMA, warps 2..9 epilogue
constexpr int kXMaxK = 65536;

// digit pair p -> (s, t); pairs are grouped by level s + t
__device__ __forceinline__ int x_s_of(int p) {
  constexpr int kS[kXPairs] = {0, 0, 1, 0, 1, 2, 0, 1, 2, 3};
  return kS[p];
}
__device__ __forceinline__ int x_t_of(int p) {
  constexpr int kT[kXPairs] = {0, 1, 0, 2, 1, 0, 3, 2, 1, 0};
  return kT[p];
}
__device__ __forceinline__ bool x_first_of_level(int p) {
  return p == 0 || p == 1 || p == 3 || p == 6;
}

// Strided view of one operand as (batch element, row, k):
// address = base + b1 * s1 + b2 * s2 + row * s_row + k * s_k (elements); the
// slicer works on distinct batch elements only (nb1 x nb2 of them).
struct XView {
  const float* base;
  int64_t rows, k;
  int64_t nb1, nb2;
  int64_t s1, s2, s_row, s_k;
};

// Exponent e with max |x| * 2^-e in [0.25, 0.5) (0 for an all-zero row; a
// sentinel for rows holding Inf/NaN).
constexpr int kXNonFinite = -100000;

__device__ __forceinline__ int x_exponent(float mx) {
  if (!(mx <= 3.4e38f)) return kXNonFinite;  // Inf or NaN
  if (mx == 0.f) return 0;
  int e;
  frexpf(mx, &e);  // mx = f * 2^e, f in [0.5, 1)
  return e + 1;
}

// One warp per row, k contiguous (s_k == 1) or any stride.
__global__ void __launch_bounds__(256) x_exponent_rows_kernel(XView v, int* __restrict__ e) {
  const int lane = threadIdx.x & 31;
  const int64_t nrows = v.nb1 * v.nb2 * v.rows;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t w = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       w < nrows; w += warps) {
    const int64_t row = w % v.rows, bb = w / v.rows;
    const float* x = v.base + (bb / v.nb2) * v.s1 + (bb % v.nb2) * v.s2 + row * v.s_row;
    float mx = 0.f;
    bool bad = false;
    for (int64_t k = lane; k < v.k; k += 32) {
      const float a = fabsf(x[k * v.s_k]);
      if (!(a <= 3.4e38f)) bad = true;
      mx = fmaxf(mx, a);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    bad = __any_sync(0xffffffffu, bad);
    if (lane == 0) e[w] = bad ? kXNonFinite : x_exponent(mx);
  }
}

// Rows contiguous (s_row == 1): block (x, z) covers 32 rows x one k range of
// kc, 8 k-lanes per row (loads coalesce across rows); the block maximum is
// merged into maxbits[row] with an integer atomicMax on the fp32 bit pattern
// (exact and order independent for non-negative values; Inf/NaN patterns
// compare above every finite one).
__global__ void __launch_bounds__(256) x_colmax_kernel(XView v, unsigned* __restrict__ maxbits,
                                                       int64_t kc) {
  __shared__ float pmax[8][33];
  const int rl = threadIdx.x & 31, j = threadIdx.x >> 5;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 32 + rl;
  const int64_t bb = blockIdx.y;
  const int64_t k0 = static_cast<int64_t>(blockIdx.z) * kc;
  const int64_t k1 = min(v.k, k0 + kc);
  float mx = 0.f;
  if (row < v.rows) {
    const float* x = v.base + (bb / v.nb2) * v.s1 + (bb % v.nb2) * v.s2 + row * v.s_row;
#pragma unroll 4
    for (int64_t k = k0 + j; k < k1; k += 8) {
      const float a = fabsf(x[k * v.s_k]);
      mx = (a != a) ? __int_as_float(0x7fffffff) : fmaxf(mx, a);
    }
  }
  pmax[j][rl] = mx;
  __syncthreads();
  if (j == 0 && row < v.rows) {
#pragma unroll
    for (int q = 1; q < 8; ++q) {
      const float o = pmax[q][rl];
      mx = (o != o || mx != mx) ? __int_as_float(0x7fffffff) : fmaxf(mx, o);
    }
    atomicMax(&maxbits[bb * v.rows + row], __float_as_uint(mx));
  }
}

__global__ void x_exponent_from_bits_kernel(const unsigned* __restrict__ maxbits,
                                            int* __restrict__ e, int64_t n) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    e[i] = x_exponent(__uint_as_float(maxbits[i]));
}

// Four digits of x * 2^-e (|x * 2^-e| < 0.5): d = rint(r * 128) in [-64, 64],
// r = r * 128 - d in [-0.5, 0.5]; all steps exact in fp32.
__device__ __forceinline__ uint32_t x_digits(float x, int e) {
  if (e == kXNonFinite) return 0u;
  float r = ldexpf(x, -e);
  uint32_t out = 0;
#pragma unroll
  for (int s = 0; s < kXS; ++s) {
    r *= 128.f;
    const float d = rintf(r);
    r -= d;
    out |= (static_cast<uint32_t>(static_cast<int>(d)) & 0xffu) << (8 * s);
  }
  return out;
}

// Digits of rows with k contiguous (any stride works, coalesced for s_k == 1):
// out[bb][s][row][kpad], one thread per 4 consecutive k of a row.
__global__ void __launch_bounds__(256) x_digits_rows_kernel(XView v, const int* __restrict__ e,
                                                             int8_t* __restrict__ out,
                                                             int64_t kpad) {
  const int64_t groups = kpad / 4;
  const int64_t total = v.nb1 * v.nb2 * v.rows * groups;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t g = idx % groups;
    const int64_t w = idx / groups;  // (bb, row)
    const int64_t row = w % v.rows, bb = w / v.rows;
    const float* x = v.base + (bb / v.nb2) * v.s1 + (bb % v.nb2) * v.s2 + row * v.s_row;
    const int ex = e[w];
    uint32_t d[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t k = g * 4 + j;
      d[j] = k < v.k ? x_digits(x[k * v.s_k], ex) : 0u;
    }
#pragma unroll
    for (int s = 0; s < kXS; ++s) {
      uint32_t packed = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) packed |= ((d[j] >> (8 * s)) & 0xffu) << (8 * j);
      reinterpret_cast<uint32_t*>(out + ((bb * kXS + s) * v.rows + row) * kpad)[g] = packed;
    }
  }
}

// Digits of rows that are contiguous across rows (s_row == 1, e.g. the
// columns of a row-major B): a 64-row x 64-k tile is read along rows, turned
// into digits and written along k through shared memory.
__global__ void __launch_bounds__(256) x_digits_cols_kernel(XView v, const int* __restrict__ e,
                                                             int8_t* __restrict__ out,
                                                             int64_t kpad) {
  __shared__ uint32_t tile[64][65];  // [k][row] digit words
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * 64;
  const int64_t k0 = static_cast<int64_t>(blockIdx.y) * 64;
  const int64_t bb = blockIdx.z;
  const float* x = v.base + (bb / v.nb2) * v.s1 + (bb % v.nb2) * v.s2;
  const int tr = threadIdx.x & 63, tk = threadIdx.x >> 6;  // 64 rows x 4 k per pass
  const int64_t row = row0 + tr;
  const int ex = row < v.rows ? e[bb * v.rows + row] : 0;
  for (int kk = tk; kk < 64; kk += 4) {
    const int64_t k = k0 + kk;
    tile[kk][tr] = (row < v.rows && k < v.k) ? x_digits(x[row * v.s_row + k * v.s_k], ex) : 0u;
  }
  __syncthreads();
  // write: each thread stores 4 consecutive k (one word per digit) of one row
  const int wr = threadIdx.x >> 4, wk = (threadIdx.x & 15) * 4;  // 16 rows x 64 k per pass
  for (int r0 = 0; r0 < 64; r0 += 16) {
    const int rr = r0 + wr;
    const int64_t orow = row0 + rr;
    if (orow >= v.rows || k0 + wk >= kpad) continue;
#pragma unroll
    for (int s = 0; s < kXS; ++s) {
      uint32_t packed = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) packed |= ((tile[wk + j][rr] >> (8 * s)) & 0xffu) << (8 * j);
      *reinterpret_cast<uint32_t*>(out + ((bb * kXS + s) * v.rows + orow) * kpad + k0 + wk) =
          packed;
    }
  }
}

struct XGemmParams {
  int m, n, k_blocks;
  int tiles_m, tiles_n;
  int64_t batch2, total_tiles;
  // distinct digit images: A index = (b1 % a_n1) * a_n2 + (b2 / a_div2) % a_n2
  int64_t a_n1, a_n2, a_div2, b_n1, b_n2, b_div2;
  const int* ea;  // [a images][m]
  const int* eb;  // [b images][n]
  float* c;
  int64_t c_sm, c_sn, c_s1, c_s2;
  const float* bias;
  int64_t bias_s2;
  int bias_per_row;
  float alpha;
  int* status;
};

__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Shared-memory descriptor of a K-major operand in the 64-byte swizzle layout
// (8-row atoms of 64-byte rows, atoms 512 bytes apart).
__device__ __forceinline__ uint64_t smem_desc_sw64(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;                    // leading offset (unused)
  d |= static_cast<uint64_t>((512u >> 4) & 0x3FFFu) << 32;  // stride offset
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(4u) << 61;                    // SWIZZLE_64B
  return d;
}

// Instruction descriptor, kind::i8: signed int8 A and B (K-major), int32 D.
__host__ __device__ constexpr uint32_t idesc_i8(uint32_t m, uint32_t n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

// One stage holds all four digit slices of A and of B for one k-block, so the
// ten digit-pair products of that k-block reuse them (8 copies per 20 MMAs).
struct XSmem {
  static constexpr uint32_t kSlice = 128 * kXBK;  // 8 KB
  static constexpr uint32_t kA = kXS * kXBM * kXBK;
  static constexpr uint32_t kB = kXS * kXBN * kXBK;
  static constexpr uint32_t kStage = kA + kB;
  static constexpr uint32_t kBar = 256;
  static constexpr uint32_t kTotal = 1024 + kXStages * kStage + kBar;
};

__global__ void __launch_bounds__(kXThreads, 1)
    gemm_i8x_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const XGemmParams p) {
  using L = XSmem;
  constexpr uint32_t kIdesc = idesc_i8(kXBM, kXBN);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kXStages * L::kA;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + kXStages * L::kStage);
  uint64_t* empty_bar = full_bar + kXStages;
  uint64_t* tfull = empty_bar + kXStages;
  uint64_t* tempty = tfull + 1;
  uint64_t* mma_done = tempty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kXStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(tempty, 8);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto decode = [&](int64_t t, int64_t& b1, int64_t& b2, int& mb, int& nb) {
    nb = static_cast<int>(t % p.tiles_n);
    int64_t rest = t / p.tiles_n;
    mb = static_cast<int>(rest % p.tiles_m);
    rest /= p.tiles_m;
    b2 = rest % p.batch2;
    b1 = rest / p.batch2;
  };

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      int stage = 0;
      uint32_t phase = 0;
      int64_t issued = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; ok && t < p.total_tiles; t += gridDim.x) {
        int64_t b1, b2;
        int mb, nb;
        decode(t, b1, b2, mb, nb);
        const int64_t ai = (b1 % p.a_n1) * p.a_n2 + (b2 / p.a_div2) % p.a_n2;
        const int64_t bi = (b1 % p.b_n1) * p.b_n2 + (b2 / p.b_div2) % p.b_n2;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, p.status)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[stage], L::kStage);
          // one box = the four digit slices of this k-block
          tma_load_4d(sA + stage * L::kA, &tmA, &full_bar[stage], kb * kXBK, mb * kXBM,
                      static_cast<int>(ai * kXS), 0);
          tma_load_4d(sB + stage * L::kB, &tmB, &full_bar[stage], kb * kXBK, nb * kXBN,
                      static_cast<int>(bi * kXS), 0);
          ++issued;
          if (++stage == kXStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      const int64_t pending = issued < kXStages ? issued : kXStages;
      int s = stage;
      uint32_t ph = phase;
      for (int64_t i = 0; i < pending; ++i) {
        if (--s < 0) {
          s = kXStages - 1;
          ph ^= 1u;
        }
        if (!mbar_wait_drain(&full_bar[s], ph)) raise_status(p.status, BIO_DEV_TIMEOUT);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------- MMA
      int stage = 0;
      uint32_t phase = 0;
      uint32_t tphase = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; ok && t < p.total_tiles; t += gridDim.x) {
        if (!mbar_wait(tempty, tphase ^ 1u, abort_flag, p.status)) break;
        tphase ^= 1u;
        tc_fence_after();
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * L::kA);
          const uint32_t b_addr = smem_u32(sB + stage * L::kB);
#pragma unroll
          for (int pr = 0; pr < kXPairs; ++pr) {
            const uint32_t d = tmem + static_cast<uint32_t>((x_s_of(pr) + x_t_of(pr)) * kXBN);
            const uint32_t aa = a_addr + static_cast<uint32_t>(x_s_of(pr)) * L::kSlice;
            const uint32_t ba = b_addr + static_cast<uint32_t>(x_t_of(pr)) * L::kSlice;
            const bool first = x_first_of_level(pr) && kb == 0;
#pragma unroll
            for (int kk = 0; kk < kXBK / 32; ++kk) {
              umma_i8(d, smem_desc_sw64(aa + kk * 32), smem_desc_sw64(ba + kk * 32), kIdesc,
                      (first && kk == 0) ? 0u : 1u);
            }
          }
          umma_commit(&empty_bar[stage]);
          if (++stage == kXStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(tfull);
      }
      umma_commit(mma_done);
      if (!mbar_wait_drain(mma_done, 0)) raise_status(p.status, BIO_DEV_TIMEOUT);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // warps 2..9: TMEM lane quarter (warp & 3), column half (warp - 2) >> 2
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    uint32_t tphase = 0;
    for (int64_t t = blockIdx.x; t < p.total_tiles; t += gridDim.x) {
      int64_t b1, b2;
      int mb, nb;
      decode(t, b1, b2, mb, nb);
      const int64_t ai = (b1 % p.a_n1) * p.a_n2 + (b2 / p.a_div2) % p.a_n2;
      const int64_t bi = (b1 % p.b_n1) * p.b_n2 + (b2 / p.b_div2) % p.b_n2;
      const bool got = mbar_wait(tfull, tphase, abort_flag, p.status);
      tphase ^= 1u;
      if (!__all_sync(0xffffffffu, got)) break;
      tc_fence_after();
      const int m = mb * kXBM + q * 32 + lane;
      const bool mvalid = m < p.m;
      const int ea = mvalid ? p.ea[ai * p.m + m] : 0;
      float* crow = p.c + b1 * p.c_s1 + b2 * p.c_s2 + static_cast<int64_t>(m) * p.c_sm;
      const float* bias = p.bias != nullptr ? p.bias + b2 * p.bias_s2 : nullptr;
      const float brow = (bias != nullptr && p.bias_per_row && mvalid) ? bias[m] : 0.f;
#pragma unroll 1
      for (int c0 = half * (kXBN / 2); c0 < (half + 1) * (kXBN / 2); c0 += 32) {
        uint32_t g0[32], g1[32], g2[32], g3[32];
        const uint32_t base = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(c0);
        tmem_ld_32x32b_x32(base + 0 * kXBN, g0);
        tmem_ld_32x32b_x32(base + 1 * kXBN, g1);
        tmem_ld_32x32b_x32(base + 2 * kXBN, g2);
        tmem_ld_32x32b_x32(base + 3 * kXBN, g3);
        const int n0 = nb * kXBN + c0;
        // column data of this chunk: lane j holds column n0 + j
        const bool nlane = n0 + lane < p.n;
        const int eb_l = nlane ? p.eb[bi * p.n + n0 + lane] : 0;
        const float bcol_l = (bias != nullptr && !p.bias_per_row && nlane) ? bias[n0 + lane] : 0.f;
        tmem_ld_wait();
        if (n0 >= p.n) continue;
        float out[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int eb = __shfl_sync(0xffffffffu, eb_l, j);
          const float bj = p.bias_per_row ? brow : __shfl_sync(0xffffffffu, bcol_l, j);
          double v = fma(static_cast<double>(static_cast<int>(g1[j])), 0x1p-21,
                         static_cast<double>(static_cast<int>(g0[j])) * 0x1p-14);
          v = fma(static_cast<double>(static_cast<int>(g2[j])), 0x1p-28, v);
          v = fma(static_cast<double>(static_cast<int>(g3[j])), 0x1p-35, v);
          // 2^(ea + eb) built from its exponent bits (ldexp when out of range)
          const int ex = ea + eb;
          const double sc = (ex > -1000 && ex < 1000)
                                ? __hiloint2double((ex + 1023) << 20, 0)
                                : ldexp(1.0, ex > 0 ? 1100 : -1100);
          v = fma(v * sc, static_cast<double>(p.alpha), static_cast<double>(bj));
          out[j] = (ea == kXNonFinite || eb == kXNonFinite) ? __int_as_float(0x7fc00000)
                                                            : __double2float_rn(v);
        }
        if (mvalid) {
          const bool vec = p.c_sn == 1 && n0 + 32 <= p.n &&
                           (reinterpret_cast<uintptr_t>(crow + n0) & 15u) == 0;
          if (vec) {
            float4* dst = reinterpret_cast<float4*>(crow + n0);
#pragma unroll
            for (int j = 0; j < 8; ++j)
              dst[j] = make_float4(out[4 * j], out[4 * j + 1], out[4 * j + 2], out[4 * j + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (n0 + j < p.n) crow[static_cast<int64_t>(n0 + j) * p.c_sn] = out[j];
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty);
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

namespace {

std::mutex g_x_mu;

unsigned grid_for(int64_t work, int64_t per_block) {
  int64_t b = (work + per_block - 1) / per_block;
  if (b > 65536 * 4) b = 65536 * 4;
  if (b < 1) b = 1;
  return static_cast<unsigned>(b);
}

int64_t align256(int64_t v) { return (v + 255) / 256 * 256; }

// Distinct images of one operand along the two batch levels.
void images(int64_t batch1, int64_t batch2, int64_t s1, int64_t s2, int64_t div2, int64_t* n1,
            int64_t* n2) {
  *n1 = (s1 == 0 || batch1 <= 1) ? 1 : batch1;
  *n2 = (s2 == 0 || batch2 <= 1) ? 1 : (batch2 + div2 - 1) / div2;
}

struct XPlan {
  int64_t kpad, a_n1, a_n2, b_n1, b_n2;
  int64_t off_ad, off_bd, off_ea, off_eb, total;
};

XPlan plan(const bio_gemm_args* a) {
  XPlan pl;
  pl.kpad = (a->k + bio::kXBK - 1) / bio::kXBK * bio::kXBK;
  images(a->batch1, a->batch2, a->a_s1, a->a_s2, a->a_div2, &pl.a_n1, &pl.a_n2);
  images(a->batch1, a->batch2, a->b_s1, a->b_s2, a->b_div2, &pl.b_n1, &pl.b_n2);
  const int64_t na = pl.a_n1 * pl.a_n2, nb = pl.b_n1 * pl.b_n2;
  pl.off_ad = 0;
  pl.off_bd = align256(na * bio::kXS * a->m * pl.kpad);
  pl.off_ea = pl.off_bd + align256(nb * bio::kXS * a->n * pl.kpad);
  pl.off_eb = pl.off_ea + align256(na * a->m * 4);
  pl.total = pl.off_eb + align256(nb * a->n * 4);
  return pl;
}

bool x_map(CUtensorMap* map, const void* ptr, int64_t kpad, int64_t rows, int64_t images_s) {
  bio_host::EncodeTiledFn enc = bio_host::encode_tiled_fn();
  if (enc == nullptr) return false;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(kpad), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(images_s), 1};
  cuuint64_t st[3] = {static_cast<cuuint64_t>(kpad), static_cast<cuuint64_t>(kpad * rows),
                      static_cast<cuuint64_t>(kpad * rows * images_s)};
  cuuint32_t box[4] = {static_cast<cuuint32_t>(bio::kXBK), 128, bio::kXS, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(ptr), dims, st, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Exponents and digits of one operand view.
int digitise(const bio::XView& v, int* e, int8_t* out, int64_t kpad, cudaStream_t s) {
  const int64_t rows_total = v.nb1 * v.nb2 * v.rows;
  if (v.s_k == 1 || v.s_row != 1) {
    bio::x_exponent_rows_kernel<<<grid_for(rows_total, 8), 256, 0, s>>>(v, e);
  } else {
    // the digits buffer doubles as the maxima scratch until it is written
    unsigned* maxbits = reinterpret_cast<unsigned*>(out);
    if (cudaMemsetAsync(maxbits, 0, static_cast<size_t>(rows_total) * 4, s) != cudaSuccess)
      return BIO_ERR_LAUNCH;
    const int64_t nbb = v.nb1 * v.nb2;
    const int64_t row_blocks = (v.rows + 31) / 32;
    int64_t ksplit = (4 * 148 + row_blocks * nbb - 1) / (row_blocks * nbb);
    if (ksplit > (v.k + 255) / 256) ksplit = (v.k + 255) / 256;
    if (ksplit < 1) ksplit = 1;
    if (ksplit > 65535) ksplit = 65535;
    const int64_t kc = (v.k + ksplit - 1) / ksplit;
    if (nbb > 65535) return BIO_ERR_SHAPE;
    dim3 grid(static_cast<unsigned>(row_blocks), static_cast<unsigned>(nbb),
              static_cast<unsigned>(ksplit));
    bio::x_colmax_kernel<<<grid, 256, 0, s>>>(v, maxbits, kc);
    bio::x_exponent_from_bits_kernel<<<grid_for(rows_total, 256), 256, 0, s>>>(maxbits, e,
                                                                             rows_total);
  }
  int st = bio_host::launch_status(cudaGetLastError());
  if (st != BIO_OK) return st;
  if (v.s_row == 1 && v.s_k != 1) {
    const int64_t nbb = v.nb1 * v.nb2;
    if (nbb > 65535 || (kpad + 63) / 64 > 65535) return BIO_ERR_SHAPE;
    dim3 grid(static_cast<unsigned>((v.rows + 63) / 64), static_cast<unsigned>((kpad + 63) / 64),
              static_cast<unsigned>(nbb));
    bio::x_digits_cols_kernel<<<grid, 256, 0, s>>>(v, e, out, kpad);
  } else {
    bio::x_digits_rows_kernel<<<grid_for(rows_total * (kpad / 4), 256), 256, 0, s>>>(v, e, out,
                                                                                    kpad);
  }
  return bio_host::launch_status(cudaGetLastError());
}

}  // namespace

extern "C" {

int64_t bio_gemm_f32_exact_workspace(const bio_gemm_args* a) {
  if (a == nullptr || a->dtype != BIO_F32 || a->m <= 0 || a->n <= 0 || a->k <= 0 ||
      a->k > bio::kXMaxK || a->batch1 < 1 || a->batch2 < 1 || a->a_div2 < 1 || a->b_div2 < 1)
    return 0;
  return plan(a).total;
}

int bio_gemm_f32_exact(const bio_gemm_args* a, void* workspace, int64_t workspace_bytes,
                       void* stream_v) {
  if (a == nullptr) return BIO_ERR_ARG;
  if (a->dtype != BIO_F32) return BIO_ERR_DTYPE;
  if ((a->flags & ~BIO_GEMM_BIAS_PER_ROW) != 0) return BIO_ERR_ARG;
  if (a->m < 0 || a->n < 0 || a->k < 0 || a->batch1 < 0 || a->batch2 < 1) return BIO_ERR_SHAPE;
  if (a->a_div2 < 1 || a->b_div2 < 1) return BIO_ERR_ARG;
  const int64_t batch = a->batch1 * a->batch2;
  if (batch == 0 || a->m == 0 || a->n == 0) return BIO_OK;
  if (a->k == 0 || a->k > bio::kXMaxK) return BIO_ERR_SHAPE;  // use bio_gemm
  if (a->m > 2147483647 || a->n > 2147483647) return BIO_ERR_SHAPE;
  if (a->a == nullptr || a->b == nullptr || a->c == nullptr || workspace == nullptr)
    return BIO_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return BIO_ERR_ALIGN;
  const XPlan pl = plan(a);
  if (workspace_bytes < pl.total) return BIO_ERR_SCRATCH;
  int st = bio_host::ensure_device(a->device);
  if (st != BIO_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream_v);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int8_t* ad = reinterpret_cast<int8_t*>(ws + pl.off_ad);
  int8_t* bd = reinterpret_cast<int8_t*>(ws + pl.off_bd);
  int* ea = reinterpret_cast<int*>(ws + pl.off_ea);
  int* eb = reinterpret_cast<int*>(ws + pl.off_eb);

  // A rows: (row = m, k); B rows: (row = n, k)
  bio::XView va{static_cast<const float*>(a->a), a->m, a->k, pl.a_n1, pl.a_n2,
                pl.a_n1 > 1 ? a->a_s1 : 0, pl.a_n2 > 1 ? a->a_s2 : 0, a->a_sm, a->a_sk};
  bio::XView vb{static_cast<const float*>(a->b), a->n, a->k, pl.b_n1, pl.b_n2,
                pl.b_n1 > 1 ? a->b_s1 : 0, pl.b_n2 > 1 ? a->b_s2 : 0, a->b_sn, a->b_sk};
  st = digitise(va, ea, ad, pl.kpad, s);
  if (st != BIO_OK) return st;
  st = digitise(vb, eb, bd, pl.kpad, s);
  if (st != BIO_OK) return st;

  static bool attr_done[bio_host::kMaxDevices] = {false};
  {
    std::lock_guard<std::mutex> lk(g_x_mu);
    if (!attr_done[a->device]) {
      if (cudaFuncSetAttribute(bio::gemm_i8x_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               bio::XSmem::kTotal) != cudaSuccess)
        return BIO_ERR_LAUNCH;
      attr_done[a->device] = true;
    }
  }
  CUtensorMap tmA, tmB;
  if (!x_map(&tmA, ad, pl.kpad, a->m, pl.a_n1 * pl.a_n2 * bio::kXS) ||
      !x_map(&tmB, bd, pl.kpad, a->n, pl.b_n1 * pl.b_n2 * bio::kXS))
    return BIO_ERR_ALIGN;
  bio::XGemmParams p;
  p.m = static_cast<int>(a->m);
  p.n = static_cast<int>(a->n);
  p.k_blocks = static_cast<int>(pl.kpad / bio::kXBK);
  p.tiles_m = static_cast<int>((a->m + bio::kXBM - 1) / bio::kXBM);
  p.tiles_n = static_cast<int>((a->n + bio::kXBN - 1) / bio::kXBN);
  p.batch2 = a->batch2;
  p.total_tiles = batch * p.tiles_m * p.tiles_n;
  p.a_n1 = pl.a_n1;
  p.a_n2 = pl.a_n2;
  p.a_div2 = a->a_div2;
  p.b_n1 = pl.b_n1;
  p.b_n2 = pl.b_n2;
  p.b_div2 = a->b_div2;
  p.ea = ea;
  p.eb = eb;
  p.c = static_cast<float*>(a->c);
  p.c_sm = a->c_sm;
  p.c_sn = a->c_sn;
  p.c_s1 = a->c_s1;
  p.c_s2 = a->c_s2;
  p.bias = static_cast<const float*>(a->bias);
  p.bias_s2 = a->bias_s2;
  p.bias_per_row = (a->flags & BIO_GEMM_BIAS_PER_ROW) ? 1 : 0;
  p.alpha = a->alpha;
  p.status = bio_host::status_word(a->device);
  const int64_t sms = bio_host::sm_count(a->device);
  const int64_t grid = p.total_tiles < sms ? p.total_tiles : sms;
  bio::gemm_i8x_kernel<<<static_cast<unsigned>(grid), bio::kXThreads, bio::XSmem::kTotal, s>>>(
      tmA, tmB, p);
  return bio_host::launch_status(cudaGetLastError());
}

}  // extern "C"
