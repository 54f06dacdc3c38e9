// Library bookkeeping: ABI version, status strings, per-device SM count and
// the device status word that kernels raise instead of trapping.
#include <mutex>

#include "bio_common.cuh"

namespace {

// One status word per device context.  Kernels OR BIO_DEV_* bits into it
// (bounded-wait timeouts, out-of-range indices); the host reads it on demand.
__device__ int g_status_word;

std::mutex g_mu;
int g_sm_count[bio_host::kMaxDevices] = {0};
int* g_status_ptr[bio_host::kMaxDevices] = {nullptr};

}  // namespace

namespace bio_host {

int launch_status(cudaError_t e) { return e == cudaSuccess ? BIO_OK : BIO_ERR_LAUNCH; }

EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int ensure_device(int device) {
  if (device < 0 || device >= kMaxDevices) return BIO_ERR_ARG;
  int cur = -1;
  if (cudaGetDevice(&cur) != cudaSuccess) return BIO_ERR_LAUNCH;
  if (cur != device && cudaSetDevice(device) != cudaSuccess) return BIO_ERR_LAUNCH;
  return BIO_OK;
}

int sm_count(int device) {
  if (device < 0 || device >= kMaxDevices) return 0;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_sm_count[device] > 0) return g_sm_count[device];
  }
  int v = 0;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lk(g_mu);
  g_sm_count[device] = v;
  return v;
}

int* status_word(int device) {
  if (device < 0 || device >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_status_ptr[device] != nullptr) return g_status_ptr[device];
  if (ensure_device(device) != BIO_OK) return nullptr;
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_status_word) != cudaSuccess) return nullptr;
  g_status_ptr[device] = static_cast<int*>(p);
  return g_status_ptr[device];
}

}  // namespace bio_host

extern "C" {

int bio_abi_version(void) { return 1; }

const char* bio_status_string(int status) {
  switch (status) {
    case BIO_OK: return "ok";
    case BIO_ERR_SHAPE: return "inconsistent or unsupported shape";
    case BIO_ERR_STRIDE: return "stride layout not accepted by this path";
    case BIO_ERR_ALIGN: return "pointer or stride alignment not accepted";
    case BIO_ERR_DTYPE: return "unsupported dtype";
    case BIO_ERR_LAUNCH: return "CUDA launch or attribute error";
    case BIO_ERR_DRIVER: return "CUDA driver entry point or tensor map error";
    case BIO_ERR_ARG: return "invalid argument";
    case BIO_ERR_DEVICE: return "device-side check failed";
    case BIO_ERR_SCRATCH: return "scratch or workspace too small for this problem";
    default: return "unknown status";
  }
}

int bio_sm_count(int device, int* out) {
  if (out == nullptr) return BIO_ERR_ARG;
  int v = bio_host::sm_count(device);
  if (v <= 0) return BIO_ERR_LAUNCH;
  *out = v;
  return BIO_OK;
}

int bio_device_status(int device, int* out) {
  if (out == nullptr) return BIO_ERR_ARG;
  int st = bio_host::ensure_device(device);
  if (st != BIO_OK) return st;
  if (bio_host::status_word(device) == nullptr) return BIO_ERR_LAUNCH;
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_status_word, sizeof(int)) != cudaSuccess) return BIO_ERR_LAUNCH;
  *out = v;
  return BIO_OK;
}

int bio_clear_device_status(int device) {
  int st = bio_host::ensure_device(device);
  if (st != BIO_OK) return st;
  if (bio_host::status_word(device) == nullptr) return BIO_ERR_LAUNCH;
  const int zero = 0;
  if (cudaMemcpyToSymbol(g_status_word, &zero, sizeof(int)) != cudaSuccess) return BIO_ERR_LAUNCH;
  return BIO_OK;
}

}  // extern "C"
