// Host-side internals shared by the translation units of libvlak_b200.so.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/vlak_b200.h"

namespace vlak {

// Thread-local error detail behind vlak_last_error_message().
void clear_error();
int set_error(int status, const char* msg);
int set_cuda_error(const char* what, cudaError_t err);
int set_errorf(int status, const char* fmt, ...);

// cuTensorMapEncodeTiled resolved through the runtime's driver entry point
// (no link-time dependency on libcuda). Returns nullptr if unavailable.
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled_fn();

// Per-device facts needed at launch (cached; thread-safe).
struct DeviceInfo {
  int device = -1;
  int sm_count = 0;
  int cc_major = 0, cc_minor = 0;
  size_t max_smem_optin = 0;
};
int current_device_info(DeviceInfo* out);

// The process's host-mapped error word (pinned, device-mapped, portable to
// every device), allocated on first use; nullptr when it is not set up yet
// and `stream` is capturing (no allocation happens during a capture) or when
// the allocation failed. Kernels write a failed bounded wait's status there;
// vlak_device_error_poll reads it without synchronizing the device. With
// may_allocate false it only returns a word set up earlier (or nullptr).
int* host_error_word(cudaStream_t stream, bool may_allocate = true);

}  // namespace vlak
