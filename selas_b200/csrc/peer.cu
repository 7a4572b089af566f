// peer.cu — what the ranks of a sequence-parallel group share over NVLink: CUDA IPC of device
// buffers, and a stream-ordered device-side barrier on flags in peer memory.
//
// The barrier follows the release/acquire pattern at system scope: each rank stores the epoch into
// every rank's flag array (st.release.sys, after a system fence), then polls its own array
// (ld.acquire.sys) until every rank's epoch is there. Kernels before the barrier on a rank's stream
// (e.g. a GEMM whose epilogue stored into a peer's buffer) have completed their stores when the barrier
// kernel starts; kernels after it on a waiting rank's stream start only after it has seen every flag.
// Every wait is bounded: on timeout the kernel records FB_DEV_TIMEOUT_PEER and returns.
#include <cstring>

#include "fb_internal.h"

namespace fb {
namespace {

typedef CUresult (*AddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

AddressRangeFn address_range_fn() {
  static const AddressRangeFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<AddressRangeFn>(nullptr);
    return reinterpret_cast<AddressRangeFn>(f);
  }();
  return fn;
}

int fail(int code, const std::string& msg) {
  set_last_error(msg);
  return code;
}

struct BarrierArgs {
  int32_t* flags[8];
  int world, rank, epoch;
  uint64_t budget_ns;
  int* status;
};

__global__ void peer_barrier_kernel(const BarrierArgs a) {
  const int p = threadIdx.x;
  if (p >= a.world) return;
  __threadfence_system();
  int32_t* theirs = a.flags[p] + a.rank;  // rank p's flag for this rank
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(theirs), "r"(a.epoch) : "memory");
  const int32_t* mine = a.flags[a.rank] + p;  // this rank's flag for rank p
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    int32_t v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
    if (v >= a.epoch) break;
    if (globaltimer_ns() - t0 > a.budget_ns) {
      atomicCAS(a.status, 0, FB_DEV_TIMEOUT_PEER);
      break;
    }
  }
}

}  // namespace
}  // namespace fb

using namespace fb;

extern "C" {

int32_t fb_ipc_export(const void* ptr, void* handle64, int64_t* offset) {
  if (!ptr || !handle64 || !offset) return fail(FB_ERR_ARG, "fb_ipc_export: null argument");
  AddressRangeFn range = address_range_fn();
  if (!range) return fail(FB_ERR_INIT, "fb_ipc_export: cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail(FB_ERR_ARG, "fb_ipc_export: not a device allocation");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return fail(FB_ERR_CUDA, std::string("fb_ipc_export: ") + cudaGetErrorString(e));
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  std::memcpy(handle64, &h, sizeof(h));
  *offset = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return FB_OK;
}

int32_t fb_ipc_open(const void* handle64, int64_t offset, void** peer_ptr, void** peer_base) {
  if (!handle64 || !peer_ptr || !peer_base || offset < 0) return fail(FB_ERR_ARG, "fb_ipc_open: bad argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle64, sizeof(h));
  void* base = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(FB_ERR_CUDA, std::string("fb_ipc_open: ") + cudaGetErrorString(e));
  *peer_base = base;
  *peer_ptr = static_cast<char*>(base) + offset;
  return FB_OK;
}

int32_t fb_ipc_close(void* peer_base) {
  const cudaError_t e = cudaIpcCloseMemHandle(peer_base);
  return e == cudaSuccess ? FB_OK : fail(FB_ERR_CUDA, std::string("fb_ipc_close: ") + cudaGetErrorString(e));
}

int32_t fb_peer_barrier(int32_t* const* flags, int32_t world, int32_t rank, int32_t epoch, int32_t timeout_ms,
                        void* stream) {
  if (!flags || world < 1 || world > 8 || rank < 0 || rank >= world || epoch < 1 || timeout_ms < 1)
    return fail(FB_ERR_ARG, "fb_peer_barrier: need 1 <= world <= 8, 0 <= rank < world, epoch >= 1, timeout_ms >= 1");
  std::string err;
  DeviceState* d = current_device(err);
  if (!d) return fail(FB_ERR_INIT, err);
  BarrierArgs a;
  std::memset(&a, 0, sizeof(a));
  for (int r = 0; r < world; ++r) {
    if (!flags[r] || (reinterpret_cast<uintptr_t>(flags[r]) & 3u))
      return fail(FB_ERR_ARG, "fb_peer_barrier: null or misaligned flag array");
    a.flags[r] = flags[r];
  }
  a.world = world;
  a.rank = rank;
  a.epoch = epoch;
  a.budget_ns = static_cast<uint64_t>(timeout_ms) * 1000000ull;
  a.status = d->status;
  peer_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(a);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? FB_OK : fail(FB_ERR_CUDA, std::string("fb_peer_barrier: ") + cudaGetErrorString(e));
}

}  // extern "C"
