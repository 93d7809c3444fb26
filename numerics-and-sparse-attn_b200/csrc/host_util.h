// Host-side helpers shared by the C-ABI launchers: status/message plumbing,
// device properties, and TMA tensor-map encoding through the driver entry
// point (no link-time dependency on libcuda).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <string>
#include <utility>

#include "nsa_b200.h"

namespace nsa {

// Records a formatted message for nsa_last_error_message() and returns code.
int fail(int code, const char* fmt, ...);
// Clears the last message (call at entry of every API function).
void clear_error();
// Converts a CUDA runtime status into NSA_ERR_CUDA with a message.
int cuda_fail(cudaError_t e, const char* what);

// Device error word of the current device (a __device__ int, no allocation).
int* device_error_word();

struct DeviceInfo {
  int device = -1;
  int sm_count = 0;
  int max_smem_optin = 0;
};
// Properties of the current device (cached per device).
const DeviceInfo& current_device();

// cuTensorMapEncodeTiled via cudaGetDriverEntryPoint.
int encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t rank, const void* base,
                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                 CUtensorMapSwizzle swizzle);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Whether launches use programmatic dependent launch (default on; NSA_PDL=0
// turns it off).  Every kernel of this library waits (griddepcontrol.wait)
// before it reads or writes global memory that an earlier kernel of the
// stream may use, so the attribute only lets its prologue overlap the tail of
// the previous kernel.
bool pdl_enabled();

// Launch `kernel` on `stream` with the programmatic-stream-serialization
// attribute when pdl_enabled().
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace nsa

namespace nsa {
// Validates an nsa_kivi_stream_cache descriptor (shared by append / decode).
int kivi_check_stream_cache(const nsa_kivi_stream_cache& c);
}  // namespace nsa
