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
//     rewritten before each use. Calls whose work overlaps on the GPU (other streams, other host
//     threads on the same device) race on the array: keep them ordered on one stream.
//   - The first call on each device does the set-up (resolving the array's device address with
//     cudaGetSymbolAddress while that device is current, clearing the status word, the driver's
//     tensor-map encoder, the kernels' shared-memory limits). Make that first call before any stream
//     capture.
//   - A kernel that gives up on a bounded wait records its code in the array's first word (the first
//     code sticks; later ones do not overwrite it). fb_linear_nf4_static_status reads that word,
//     without allocating, and clears it on request; calls do not clear it, so a timeout stays visible
//     until it is read.
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
  std::atomic<bool> ready{false};  // stored with release once base and sm_count are filled
};

constexpr int kMaxDevices = 64;
StaticDevice g_static_dev[kMaxDevices];
std::mutex g_static_mu;

int current_ordinal(int& dev, std::string& err) {
  const cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    err = std::string("cudaGetDevice: ") + cudaGetErrorString(e);
    return FB_ERR_INIT;
  }
  return FB_OK;
}

// Set-up for the current device, once: no allocation anywhere on this path.
StaticDevice* static_device(std::string& err) {
  int dev = 0;
  if (current_ordinal(dev, err) != FB_OK) return nullptr;
  StaticDevice& s = g_static_dev[dev];
  if (s.ready.load(std::memory_order_acquire)) return &s;
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (s.ready.load(std::memory_order_relaxed)) return &s;
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
  cudaError_t e = cudaGetSymbolAddress(&ptr, g_static_scratch);
  if (e != cudaSuccess || ptr == nullptr) {
    err = std::string("cudaGetSymbolAddress(static scratch): ") + cudaGetErrorString(e);
    return nullptr;
  }
  // The status word starts at zero; later calls only ever CAS a code into it or clear it on a read.
  const int zero = 0;
  e = cudaMemcpyToSymbol(g_static_scratch, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    err = std::string("clearing the static status word: ") + cudaGetErrorString(e);
    return nullptr;
  }
  s.base = static_cast<uint8_t*>(ptr);
  s.sm_count = sms;
  s.ready.store(true, std::memory_order_release);
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
  int* status = reinterpret_cast<int*>(d->base);
  const int rc = launch_linear_nf4(*problem, epilogue, d->base + kStatusBytes, kWorkBytes, status, d->sm_count,
                                   static_cast<cudaStream_t>(stream), err);
  if (rc) set_last_error(err);
  return rc;
}

extern "C" int32_t fb_linear_nf4_static_status(int32_t* code, int32_t clear) {
  if (!code) {
    set_last_error("fb_linear_nf4_static_status: null output");
    return FB_ERR_ARG;
  }
  std::string err;
  int dev = 0;
  if (current_ordinal(dev, err) != FB_OK) {
    set_last_error(err);
    return FB_ERR_INIT;
  }
  if (!g_static_dev[dev].ready.load(std::memory_order_acquire)) {  // nothing ran here: nothing to report
    *code = 0;
    return FB_OK;
  }
  // Every earlier call's kernels, on whichever stream, must have finished before the word is read.
  cudaError_t e = cudaDeviceSynchronize();
  int v = 0;
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&v, g_static_scratch, sizeof(v), 0, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && clear && v != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_static_scratch, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice);
  }
  if (e != cudaSuccess) {
    set_last_error(std::string("fb_linear_nf4_static_status: ") + cudaGetErrorString(e));
    return FB_ERR_CUDA;
  }
  *code = v;
  return FB_OK;
}

extern "C" int32_t fb_selftest_static_wait_timeout(int32_t budget_ms, void* stream) {
  if (budget_ms <= 0 || budget_ms > 1000) {
    set_last_error("fb_selftest_static_wait_timeout: budget_ms in 1..1000");
    return FB_ERR_ARG;
  }
  std::string err;
  StaticDevice* d = static_device(err);
  if (!d) {
    set_last_error(err);
    return FB_ERR_INIT;
  }
  const cudaError_t e = launch_selftest_wait(reinterpret_cast<int*>(d->base),
                                             static_cast<uint64_t>(budget_ms) * 1000000ull,
                                             static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    set_last_error(std::string("fb_selftest_static_wait_timeout: ") + cudaGetErrorString(e));
    return FB_ERR_CUDA;
  }
  return FB_OK;
}
