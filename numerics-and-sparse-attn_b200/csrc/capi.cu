// Status plumbing, device error word and tensor-map encoding for the C ABI.
#include <cstdarg>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "host_util.h"

namespace nsa {

namespace {
thread_local char g_msg[512] = {0};
}  // namespace

// One error word per device, written by kernels through set_error().  A
// __device__ variable: every GPU that loads the library holds it; reading its
// address needs no allocation.
__device__ int g_device_error_word;

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return code;
}

void clear_error() { g_msg[0] = 0; }

int cuda_fail(cudaError_t e, const char* what) {
  return fail(NSA_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mu;
DeviceInfo g_dev[kMaxDevices];
int* g_err_ptr[kMaxDevices] = {nullptr};
}  // namespace

const DeviceInfo& current_device() {
  static DeviceInfo invalid;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return invalid;
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceInfo& d = g_dev[dev];
  if (d.device < 0) {
    cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    d.device = dev;
  }
  return d;
}

int* device_error_word() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_err_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error_word) != cudaSuccess) return nullptr;
    g_err_ptr[dev] = static_cast<int*>(p);
  }
  return g_err_ptr[dev];
}

namespace {
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  });
  return fn;
}
}  // namespace

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("NSA_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

int encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t rank, const void* base,
                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                 CUtensorMapSwizzle swizzle) {
  EncodeFn fn = encode_fn();
  if (!fn) return fail(NSA_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5];
  cuuint32_t e[5];
  for (uint32_t i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i + 1 < rank) s[i] = strides_bytes[i];
  }
  CUresult r = fn(map, dtype, rank, const_cast<void*>(base), d, s, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(NSA_ERR_INVALID, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
  return NSA_OK;
}

}  // namespace nsa

extern "C" {

const char* nsa_error_string(int status) {
  switch (status) {
    case NSA_OK: return "NSA_OK";
    case NSA_ERR_INVALID: return "NSA_ERR_INVALID";
    case NSA_ERR_ALIGN: return "NSA_ERR_ALIGN";
    case NSA_ERR_UNSUPPORTED: return "NSA_ERR_UNSUPPORTED";
    case NSA_ERR_WORKSPACE: return "NSA_ERR_WORKSPACE";
    case NSA_ERR_CUDA: return "NSA_ERR_CUDA";
    case NSA_ERR_TIMEOUT: return "NSA_ERR_TIMEOUT";
    default: return "NSA_ERR_UNKNOWN";
  }
}

const char* nsa_last_error_message(void) { return nsa::g_msg; }

const char* nsa_version(void) { return "nsa_b200 0.1 sm_100a"; }

int nsa_device_error(int* code, nsa_stream_t stream) {
  nsa::clear_error();
  if (!code) return nsa::fail(NSA_ERR_INVALID, "code must not be NULL");
  *code = NSA_OK;
  cudaError_t e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return nsa::cuda_fail(e, "cudaStreamSynchronize");
  int* w = nsa::device_error_word();
  if (!w) return nsa::fail(NSA_ERR_CUDA, "device error word unavailable");
  int v = 0;
  e = cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return nsa::cuda_fail(e, "read device error word");
  if (v != 0) {
    const int zero = 0;
    e = cudaMemcpy(w, &zero, sizeof(int), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return nsa::cuda_fail(e, "clear device error word");
  }
  *code = v;
  return NSA_OK;
}

}  // extern "C"

// ---------------------------------------------------------------- self-test
// One CTA waits, with a limit of limit_ns, on an mbarrier phase that nothing
// completes: the bounded wait gives up, records NSA_ERR_TIMEOUT in the
// device error word and the kernel returns -- the path every kernel takes
// when a copy never lands.  The context stays usable.
namespace nsa {
namespace {
__global__ void wait_timeout_kernel(int* err, uint64_t limit_ns) {
  __shared__ uint64_t bar;
  const uint32_t b = smem_u32(&bar);
  if (threadIdx.x == 0) {
    mbar_init(b, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(b, 0, err, limit_ns);  // phase 0 never completes
}
}  // namespace
}  // namespace nsa

extern "C" int nsa_selftest_wait_timeout(int64_t limit_ns, nsa_stream_t stream) {
  nsa::clear_error();
  if (limit_ns <= 0 || limit_ns > 2000000000ll) return nsa::fail(NSA_ERR_INVALID, "limit_ns must be in (0, 2e9]");
  int* w = nsa::device_error_word();
  if (!w) return nsa::fail(NSA_ERR_CUDA, "device error word unavailable");
  nsa::wait_timeout_kernel<<<1, 32, 0, stream>>>(w, static_cast<uint64_t>(limit_ns));
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? NSA_OK : nsa::cuda_fail(e, "wait_timeout_kernel launch");
}
