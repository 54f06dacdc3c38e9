// Self-test of the bounded-wait exit path (bio_selftest_bounded_wait).
//
// Every spin in this library's kernels is an mbarrier wait bounded by time
// and by poll count (bio_common.cuh: mbar_wait / mbar_wait_drain).  When a
// wait gives up, the kernel must set BIO_DEV_TIMEOUT in the status word,
// drain the copies it still has in flight, free its tensor memory and
// return, leaving the context usable.  This kernel runs the same producer /
// consumer shape as the GEMMs, with the same wait functions, on a pipeline in
// which the consumer never releases a stage and waits on a barrier that
// nothing arrives at, so both waits run out after `timeout_ns`.
#include "bio_common.cuh"

namespace bio {

constexpr int kSelfStages = 2;
constexpr uint32_t kSelfStageBytes = 4096;

// out[0]: producer wait gave up (1) ; out[1]: consumer wait gave up (1);
// out[2]: stage 0 landed and holds the source bytes (1); out[3]: drain ok (1)
__global__ void __launch_bounds__(64, 1)
    bounded_wait_selftest_kernel(const uint8_t* __restrict__ src, int* out, uint64_t timeout_ns,
                                 int* status) {
  __shared__ __align__(128) uint8_t stage_buf[kSelfStages][kSelfStageBytes];
  __shared__ __align__(8) uint64_t full_bar[kSelfStages];
  __shared__ __align__(8) uint64_t empty_bar[kSelfStages];
  __shared__ __align__(8) uint64_t never_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_word;
  volatile int* abort_flag = &abort_word;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kSelfStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(&never_bar, 1);
    abort_word = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;

  if (warp == 0 && lane == 0) {
    // producer: three rounds over a two-stage ring; the third needs stage 0
    // back, which the consumer never releases
    int issued = 0;
    bool gave_up = false;
    for (int r = 0; r < 3; ++r) {
      const int s = r % kSelfStages;
      const uint32_t parity = ((r / kSelfStages) & 1u) ^ 1u;
      if (!mbar_wait(&empty_bar[s], parity, abort_flag, status, timeout_ns)) {
        gave_up = true;
        break;
      }
      mbar_arrive_expect_tx(&full_bar[s], kSelfStageBytes);
      asm volatile(
          "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, "
          "[%3];" ::"r"(smem_u32(stage_buf[s])),
          "l"(reinterpret_cast<uint64_t>(src + static_cast<size_t>(s) * kSelfStageBytes)),
          "r"(kSelfStageBytes), "r"(smem_u32(&full_bar[s]))
          : "memory");
      ++issued;
    }
    // drain: every copy issued must land before shared memory is released
    bool drained = true;
    for (int i = 0; i < issued && i < kSelfStages; ++i)
      drained &= mbar_wait_drain(&full_bar[i], 0u, timeout_ns);
    if (!drained) raise_status(status, BIO_DEV_TIMEOUT);
    out[0] = gave_up ? 1 : 0;
    out[3] = drained ? 1 : 0;
  } else if (warp == 1 && lane == 0) {
    // consumer: takes stage 0, checks it, keeps it, then waits for an event
    // that never comes
    int landed = 0;
    if (mbar_wait(&full_bar[0], 0u, abort_flag, status, timeout_ns)) {
      landed = 1;
      for (uint32_t i = 0; i < kSelfStageBytes; i += 97)
        landed &= stage_buf[0][i] == src[i] ? 1 : 0;
    }
    const bool got = mbar_wait(&never_bar, 0u, abort_flag, status, timeout_ns);
    out[1] = got ? 0 : 1;
    out[2] = landed;
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 32);
  }
}

}  // namespace bio

extern "C" {

int bio_selftest_bounded_wait(const void* src, int32_t* out, int64_t timeout_ns, int32_t device,
                              void* stream) {
  if (src == nullptr || out == nullptr) return BIO_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(src) & 15u) != 0) return BIO_ERR_ALIGN;
  if (timeout_ns < 1000 || timeout_ns > 2000000000ll) return BIO_ERR_ARG;
  int st = bio_host::ensure_device(device);
  if (st != BIO_OK) return st;
  int* status = bio_host::status_word(device);
  if (status == nullptr) return BIO_ERR_LAUNCH;
  bio::bounded_wait_selftest_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(src), out, static_cast<uint64_t>(timeout_ns), status);
  return bio_host::launch_status(cudaGetLastError());
}

}  // extern "C"
