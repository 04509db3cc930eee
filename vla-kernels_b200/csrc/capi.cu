// Library identity, status strings, thread-local error detail, and the
// per-device / driver-entry-point caches used by the launchers.

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>

#include <atomic>
#include <mutex>
#include <string>

#include "vlak_internal.h"

namespace vlak {
namespace {
thread_local std::string t_last_error;
}

void clear_error() { t_last_error.clear(); }

int set_error(int status, const char* msg) {
  t_last_error = msg ? msg : "";
  return status;
}

int set_errorf(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return status;
}

int set_cuda_error(const char* what, cudaError_t err) {
  return set_errorf(VLAK_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
}

EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<EncodeTiledFn>(nullptr);
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

int current_device_info(DeviceInfo* out) {
  constexpr int kMaxDev = 64;
  static DeviceInfo cache[kMaxDev];
  static std::once_flag once[kMaxDev];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_cuda_error("cudaGetDevice", e);
  if (dev < 0 || dev >= kMaxDev) return set_error(VLAK_ERR_CUDA, "device ordinal out of range");
  int status = VLAK_OK;
  std::call_once(once[dev], [&] {
    DeviceInfo d;
    d.device = dev;
    int smem = 0;
    if (cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) {
      d.device = -1;
    }
    d.max_smem_optin = static_cast<size_t>(smem);
    cache[dev] = d;
  });
  if (cache[dev].device < 0) {
    // attribute query failed (e.g. no device); retry is pointless, report it
    return set_error(VLAK_ERR_CUDA, "cudaDeviceGetAttribute failed for the current device");
  }
  *out = cache[dev];
  return status;
}

namespace {
std::mutex g_host_word_mu;
std::atomic<int*> g_host_word{nullptr};
}  // namespace

int* host_error_word(cudaStream_t stream, bool may_allocate) {
  int* w = g_host_word.load(std::memory_order_acquire);
  if (w != nullptr || !may_allocate) return w;
  // cudaHostAlloc is not allowed while the stream is being captured (it
  // would invalidate the capture): such a launch reports through the device
  // word instead
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) {
    cudaGetLastError();
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_host_word_mu);
  w = g_host_word.load(std::memory_order_acquire);
  if (w != nullptr) return w;
  void* p = nullptr;
  if (cudaHostAlloc(&p, sizeof(int), cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  // unified addressing: the device sees the word at its host address
  void* d = nullptr;
  if (cudaHostGetDevicePointer(&d, p, 0) != cudaSuccess || d != p) {
    cudaGetLastError();
    cudaFreeHost(p);
    return nullptr;
  }
  *static_cast<volatile int*>(p) = 0;
  g_host_word.store(static_cast<int*>(p), std::memory_order_release);
  return static_cast<int*>(p);
}

}  // namespace vlak

extern "C" int vlak_device_error_poll(int* code) {
  int v = 0;
  int* w = vlak::g_host_word.load(std::memory_order_acquire);
  if (w != nullptr) {
    volatile int* vw = w;
    v = *vw;
    if (v != 0) *vw = 0;
  }
  if (code) *code = v;
  return VLAK_OK;
}

extern "C" int vlak_abi_version(void) { return VLAK_ABI_VERSION; }

extern "C" const char* vlak_status_string(int status) {
  switch (status) {
    case VLAK_OK: return "ok";
    case VLAK_ERR_INVALID_ARGUMENT: return "invalid argument";
    case VLAK_ERR_ALIGNMENT: return "misaligned pointer or stride";
    case VLAK_ERR_UNSUPPORTED_DTYPE: return "unsupported dtype";
    case VLAK_ERR_CUDA: return "CUDA error";
    case VLAK_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
    case VLAK_ERR_UNSUPPORTED_DEVICE: return "unsupported device (needs sm_100)";
    default: return "unknown status";
  }
}

extern "C" const char* vlak_last_error_message(void) { return vlak::t_last_error.c_str(); }
