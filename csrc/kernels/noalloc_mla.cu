// Allocation-free entry point for the split-K sparse MLA decode (see
// noalloc_mla.h for the contract).  It reuses the library's cta_group::2
// split-K kernel and LSE combine unchanged; only the scratch comes from a fixed
// device array instead of a caller or allocator buffer.
#include <atomic>
#include <mutex>
#include <stdexcept>

#include "launchers.h"
#include "noalloc_mla.h"

namespace {

constexpr int kHeads = 128;
constexpr int kValueDim = 512;
// Per (split, token) row: 128 heads x 512 FP32 partial outputs + 128 LSEs.
constexpr size_t kScratchFloats = size_t(CXLD_NOALLOC_MLA_MAX_ROWS) * kHeads * (kValueDim + 1);

// The scratch lives in the library image.  Host code must not pass the
// symbol itself to a kernel: on the host it only names a stand-in, so its
// device address is looked up once per device below.
static __device__ __align__(256) float g_mla_scratch[kScratchFloats];
static __device__ int g_mla_error_word;

struct DeviceScratch {
  float* scratch = nullptr;
  int* error_word = nullptr;
  // Published with release order after the two pointers are written; a
  // reader that sees true (acquire) also sees the pointers.
  std::atomic<bool> ready{false};
};

constexpr int kMaxDevices = 64;
DeviceScratch g_devices[kMaxDevices];
std::mutex g_setup_mutex;

// First call per device: resolve the device addresses with that device current.
int setup_current_device(DeviceScratch** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return CXLD_NOALLOC_SETUP_FAILED;
  DeviceScratch& d = g_devices[dev];
  if (!d.ready.load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!d.ready.load(std::memory_order_relaxed)) {
      void* scratch = nullptr;
      void* err = nullptr;
      if (cudaGetSymbolAddress(&scratch, g_mla_scratch) != cudaSuccess || scratch == nullptr)
        return CXLD_NOALLOC_SETUP_FAILED;
      if (cudaGetSymbolAddress(&err, g_mla_error_word) != cudaSuccess || err == nullptr)
        return CXLD_NOALLOC_SETUP_FAILED;
      d.scratch = static_cast<float*>(scratch);
      d.error_word = static_cast<int*>(err);
      d.ready.store(true, std::memory_order_release);
    }
  }
  *out = &d;
  return CXLD_NOALLOC_OK;
}

}  // namespace

extern "C" int cxld_sparse_mla_split_noalloc(const void* q, const void* kv, const int* ids, int T, int K,
                                             int P, float scale, int splits, void* out, float* lse,
                                             cudaStream_t stream) {
  if (q == nullptr || kv == nullptr || ids == nullptr || out == nullptr) return CXLD_NOALLOC_BAD_ARGUMENT;
  if (T < 1 || K < 1 || P < 1 || splits < 1 || splits > 32) return CXLD_NOALLOC_BAD_ARGUMENT;
  if (int64_t(splits) * T > CXLD_NOALLOC_MLA_MAX_ROWS) return CXLD_NOALLOC_TOO_LARGE;
  DeviceScratch* d = nullptr;
  const int rc = setup_current_device(&d);
  if (rc != CXLD_NOALLOC_OK) return rc;
  b200::MLAArgs a{};
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.kv = static_cast<const __nv_bfloat16*>(kv);
  a.ids = ids;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.lse = lse;
  a.T = T;
  a.H = kHeads;
  a.K = K;
  a.P = P;
  a.scale = scale;
  a.err = d->error_word;
  // Each call reports only its own device errors: the word is cleared in
  // stream order before the kernel runs (the kernel records the first error
  // of the call and never clears it).
  if (cudaMemsetAsync(d->error_word, 0, sizeof(int), stream) != cudaSuccess) return CXLD_NOALLOC_LAUNCH_FAILED;
  try {
    b200::launch_sparse_mla_2sm(a, splits, d->scratch, stream);
  } catch (const std::exception&) {
    return CXLD_NOALLOC_LAUNCH_FAILED;
  }
  return CXLD_NOALLOC_OK;
}

extern "C" int cxld_sparse_mla_noalloc_error(int* device_code, cudaStream_t stream) {
  if (device_code == nullptr) return CXLD_NOALLOC_BAD_ARGUMENT;
  DeviceScratch* d = nullptr;
  const int rc = setup_current_device(&d);
  if (rc != CXLD_NOALLOC_OK) return rc;
  // The copy is ordered after the work already on `stream`; the host value
  // is settled once the stream has been synchronised.
  if (cudaMemcpyAsync(device_code, d->error_word, sizeof(int), cudaMemcpyDeviceToHost, stream) != cudaSuccess)
    return CXLD_NOALLOC_LAUNCH_FAILED;
  if (cudaStreamSynchronize(stream) != cudaSuccess) return CXLD_NOALLOC_LAUNCH_FAILED;
  return CXLD_NOALLOC_OK;
}

extern "C" int cxld_sparse_mla_noalloc_max_rows(void) { return CXLD_NOALLOC_MLA_MAX_ROWS; }

extern "C" const char* cxld_noalloc_error_string(int code) {
  switch (code) {
    case CXLD_NOALLOC_OK:
      return "ok";
    case CXLD_NOALLOC_BAD_ARGUMENT:
      return "bad argument (null pointer or non-positive size, or splits outside [1, 32])";
    case CXLD_NOALLOC_TOO_LARGE:
      return "splits * T exceeds the fixed scratch capacity (cxld_sparse_mla_noalloc_max_rows)";
    case CXLD_NOALLOC_SETUP_FAILED:
      return "could not resolve the device address of the scratch array on the current device";
    case CXLD_NOALLOC_LAUNCH_FAILED:
      return "kernel launch failed";
    default:
      return "unknown error code";
  }
}
