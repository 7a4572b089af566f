// fb_internal.h — host-side declarations shared by the .cu files of libflux_b200.so.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <atomic>
#include <cstring>
#include <string>

#include "../../include/flux_b200.h"
#include "fb_common.cuh"

namespace fb {

constexpr int kNumSms = 148;

// Per-device state resolved once by fb_init / ensure_device.
struct DeviceState {
  int* status = nullptr;  // device status word (fb_device_code)
  int sm_count = 0;
  // split-K partial sums of the decoding GEMM: one [2][128][256] fp32 block per work item (at most one
  // item per CTA pair), and one arrival counter per (tile, CTA of the pair), zero between launches
  float* splitk_ws = nullptr;
  int* splitk_count = nullptr;
  // set (release) after every field above is filled; the unlocked fast path reads it with acquire
  std::atomic<bool> ready{false};
};

// Returns the state of the current device (initialising it on first use), or nullptr with `err` set.
DeviceState* current_device(std::string& err);

// cuTensorMapEncodeTiled, resolved through the runtime's driver entry point (no libcuda link).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn();
// Resolves the driver entry points once (cudaGetDeviceCount, cudaGetDriverEntryPoint); allocates nothing.
int driver_init(std::string& err);
// Sets the message fb_last_error() returns on this thread.
void set_last_error(const std::string& msg);
// Launches the self-test kernel whose bounded wait on an mbarrier that nothing completes gives up after
// budget_ns, records FB_DEV_TIMEOUT_EPI in *status and returns.
cudaError_t launch_selftest_wait(int* status, uint64_t budget_ns, cudaStream_t st);

cudaError_t launch_nf4_dequant(const uint8_t* packed, const float* absmax, const float* code16, int64_t n_bytes,
                               int blocksize, void* out, int out_dtype, cudaStream_t st);
cudaError_t launch_ln_mod(const float* x, int64_t rows, int dim, int rows_per_batch, const uint16_t* shift,
                          const uint16_t* scale, int64_t mod_bstride, uint16_t* out, cudaStream_t st);
cudaError_t launch_ln_mod_grouped(const fb_ln_mod_problem* probs, int count, cudaStream_t st);
cudaError_t launch_gated_add(const float* x, const uint16_t* g, const uint16_t* y, float* out, int64_t rows, int dim,
                             int rows_per_batch, int64_t g_bstride, int guard, cudaStream_t st);
cudaError_t launch_gelu(const uint16_t* h, uint16_t* out, int64_t n, cudaStream_t st);
cudaError_t launch_qk_norm_rope(const uint16_t* qkv, int64_t ld_qkv, int batch, int rows, int heads, int head_dim,
                                const float* q_scale, const float* k_scale, const float* rcos, const float* rsin,
                                uint16_t* q, uint16_t* k, uint16_t* v, int seq_total, int seq_offset,
                                cudaStream_t st);

// Returns an FB_ERR_* code (0 = launched) and fills `err` on failure.
int launch_linear_grouped(const fb_linear* probs, int count, int epilogue, cudaStream_t st, std::string& err);
// The same launch with an explicit device status word and SM count. `n_offsets` (or nullptr) gives,
// per problem, the column of the full Linear that the problem's column 0 is (QKV epilogue on a
// column chunk of a larger Linear).
int launch_linear_on(const fb_linear* probs, int count, int epilogue, const int* n_offsets, int* status,
                     int sm_count, cudaStream_t st, std::string& err, const DeviceState* splitk = nullptr);
// An NF4 Linear: the weight is decoded bit-exactly into `workspace` (bf16), as many whole 256-row
// chunks of output features at a time as fit, and each chunk runs through the tcgen05 GEMM with the
// problem's epilogue. Stream-ordered: a chunk's decode starts after the previous chunk's GEMM.
int launch_linear_nf4(const fb_linear& problem, int epilogue, void* workspace, int64_t workspace_bytes, int* status,
                      int sm_count, cudaStream_t st, std::string& err);
int launch_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out0, int64_t ld0,
                     uint16_t* out1, int64_t ld1, int split, int batch, int heads, int seq, int head_dim, float scale,
                     cudaStream_t st, std::string& err);

int launch_attention_sp(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* const* out_peers,
                        int64_t ld_out, int col0, int heads, int seq_local, int sp_world, int head_dim, float scale,
                        cudaStream_t st, std::string& err);

// One-time kernel attribute set-up (dynamic shared memory limits); returns an error string or "".
std::string gemm_setup();
std::string attention_setup();

}  // namespace fb
