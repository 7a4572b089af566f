// linear_nf4_static.cu — fb_linear_nf4_static: the NF4 Linear of fb_linear_nf4 for callers that
// cannot allocate device memory.
//
// Who needs it: fb_linear_nf4 wants a decode workspace from its caller, and the library's own
// fb_init allocates a status word. Some callers can do neither. selas's planner hands its ring arena
// every byte of HBM it can spare and budgets the rest to the byte, so one more allocation in the
// middle of a step can push the process out of memory. Code being captured into a CUDA graph may not
// call cudaMalloc at all. An engine that has already handed device memory to another allocator has
// nothing left to give. This entry point needs no allocation from anyone: its workspace and its
// status word live in one fixed array of device memory that is part of the library image itself.
//
// What it costs and how it behaves:
//   - The array is kStaticBytes (16 MiB): a 256-byte status area, then the decode workspace. Every
//     GPU that loads this part of the library holds it until the process exits.
//   - The weight is decoded into the array as bf16 in whole 256-row chunks, so the reduction dimension
//     is bounded: min(n, 256) * k * 2 bytes must fit in kWorkBytes (k <= 32767 for n >= 256). Larger
//     problems are rejected with FB_ERR_ARG and a message before anything is launched.
//   - Every call uses the same array and leaves its contents behind. The decoded weight is fully
//     rewritten before each use; the status word is cleared (an async memset on the call's stream)
//     at the start of every call. Calls whose work overlaps on the GPU (other streams, other host
//     threads on the same device) race on the array: keep them ordered on one stream.
//   - The first call on each device does the set-up (resolving the array's device address with
//     cudaGetSymbolAddress while that device is current, the driver's tensor-map encoder, the kernels'
//     shared-memory limits). Make that first call before any stream capture.
//   - A kernel that gives up on a bounded wait records its code in the first word of the array (not in
//     the word fb_device_status reads).
#include <mutex>

#include "fb_internal.h"

namespace fb {

namespace {

constexpr int64_t kStaticBytes = 16ll << 20;
constexpr int64_t kStatusBytes = 256;
constexpr int64_t kWorkBytes = kStaticBytes - kStatusBytes;

static __device__ __align__(256) uint8_t g_static_scratch[kStaticBytes];

struct StaticDevice {
  uint8_t* base = nullptr;  // device address of g_static_scratch on this device
  int sm_count = 0;
  bool ready = false;
};

constexpr int kMaxDevices = 64;
StaticDevice g_static_dev[kMaxDevices];
std::mutex g_static_mu;

// Set-up for the current device, once: no allocation anywhere on this path.
StaticDevice* static_device(std::string& err) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    err = std::string("cudaGetDevice: ") + cudaGetErrorString(e);
    return nullptr;
  }
  StaticDevice& s = g_static_dev[dev];
  if (s.ready) return &s;
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (s.ready) return &s;
  if (driver_init(err) != FB_OK) return nullptr;
  int major = 0, minor = 0, sms = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (major != 10 || minor != 0) {
    err = "libflux_b200 needs an sm_100 (B200) device";
    return nullptr;
  }
  const std::string msg = gemm_setup();
  if (!msg.empty()) {
    err = msg;
    return nullptr;
  }
  void* ptr = nullptr;
  e = cudaGetSymbolAddress(&ptr, g_static_scratch);
  if (e != cudaSuccess || ptr == nullptr) {
    err = std::string("cudaGetSymbolAddress(static scratch): ") + cudaGetErrorString(e);
    return nullptr;
  }
  s.base = static_cast<uint8_t*>(ptr);
  s.sm_count = sms;
  s.ready = true;
  return &s;
}

}  // namespace

}  // namespace fb

using namespace fb;

extern "C" int32_t fb_linear_nf4_static(const fb_linear* problem, int32_t epilogue, void* stream) {
  std::string err;
  if (!problem) {
    set_last_error("fb_linear_nf4_static: null problem");
    return FB_ERR_ARG;
  }
  const int64_t n = problem->n, k = problem->k;
  if (n > 0 && k > 0 && std::min<int64_t>(n, 256) * k * 2 > kWorkBytes) {
    set_last_error("fb_linear_nf4_static: k = " + std::to_string(k) + " is too large for the fixed " +
                     std::to_string(kWorkBytes) + "-byte decode area (needs min(n, 256) * k * 2 = " +
                     std::to_string(std::min<int64_t>(n, 256) * k * 2) + " bytes); use fb_linear_nf4 with a "
                     "caller-provided workspace");
    return FB_ERR_ARG;
  }
  StaticDevice* d = static_device(err);
  if (!d) {
    set_last_error(err);
    return FB_ERR_INIT;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int* status = reinterpret_cast<int*>(d->base);
  const cudaError_t e = cudaMemsetAsync(status, 0, sizeof(int), st);
  if (e != cudaSuccess) {
    set_last_error(std::string("fb_linear_nf4_static: clearing the status word: ") + cudaGetErrorString(e));
    return FB_ERR_CUDA;
  }
  const int rc = launch_linear_nf4(*problem, epilogue, d->base + kStatusBytes, kWorkBytes, status, d->sm_count, st, err);
  if (rc) set_last_error(err);
  return rc;
}
