// capi.cu — the extern "C" boundary of libflux_b200.so (declared in include/flux_b200.h):
// one-time initialisation, per-device state, argument validation and error reporting.
#include <cstring>
#include <mutex>

#include "fb_internal.h"

namespace fb {

namespace {

thread_local std::string t_last_error;
std::once_flag g_init_once;
int g_init_rc = FB_ERR_INIT;
std::string g_init_err;
EncodeTiledFn g_encode = nullptr;
std::mutex g_dev_mu;
constexpr int kMaxDevices = 64;
DeviceState g_dev[kMaxDevices];

int fail(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

void do_init() {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0) {
    g_init_err = std::string("no CUDA device: ") + cudaGetErrorString(e);
    return;
  }
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr) {
    g_init_err = "cuTensorMapEncodeTiled not found in the driver";
    return;
  }
  g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  g_init_rc = FB_OK;
}

}  // namespace

EncodeTiledFn encode_fn() { return g_encode; }

void set_last_error(const std::string& msg) { t_last_error = msg; }

int driver_init(std::string& err) {
  std::call_once(g_init_once, do_init);
  if (g_init_rc != FB_OK) err = g_init_err;
  return g_init_rc;
}

DeviceState* current_device(std::string& err) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    err = std::string("cudaGetDevice: ") + cudaGetErrorString(e);
    return nullptr;
  }
  DeviceState& s = g_dev[dev];
  if (s.ready.load(std::memory_order_acquire)) return &s;
  std::lock_guard<std::mutex> lock(g_dev_mu);
  if (s.ready.load(std::memory_order_relaxed)) return &s;
  int major = 0, minor = 0, sms = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (major != 10 || minor != 0) {
    err = "libflux_b200 needs an sm_100 (B200) device; device " + std::to_string(dev) + " is sm_" +
          std::to_string(major) + std::to_string(minor);
    return nullptr;
  }
  std::string msg = gemm_setup();
  if (msg.empty()) msg = attention_setup();
  if (!msg.empty()) {
    err = msg;
    return nullptr;
  }
  int* status = nullptr;
  e = cudaMalloc(&status, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(status, 0, sizeof(int));
  if (e != cudaSuccess) {
    err = std::string("status word allocation: ") + cudaGetErrorString(e);
    return nullptr;
  }
  // split-K workspace of the decoding GEMM (allocated here, outside any graph capture)
  const size_t items = static_cast<size_t>(sms / 2);
  e = cudaMalloc(&s.splitk_ws, items * 2 * 128 * 256 * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&s.splitk_count, items * 2 * sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(s.splitk_count, 0, items * 2 * sizeof(int));
  if (e != cudaSuccess) {
    err = std::string("split-K workspace allocation: ") + cudaGetErrorString(e);
    return nullptr;
  }
  s.status = status;
  s.sm_count = sms;
  s.ready.store(true, std::memory_order_release);
  return &s;
}

}  // namespace fb

using namespace fb;

extern "C" {

int32_t fb_init(void) {
  std::call_once(g_init_once, do_init);
  if (g_init_rc != FB_OK) return fail(g_init_rc, g_init_err);
  std::string err;
  if (!current_device(err)) return fail(FB_ERR_INIT, err);
  return FB_OK;
}

const char* fb_last_error(void) { return t_last_error.c_str(); }

const char* fb_version(void) { return "flux_b200 sm_100a " __DATE__; }

int32_t fb_device_status(int32_t* code, int32_t clear) {
  if (!code) return fail(FB_ERR_ARG, "fb_device_status: null output");
  std::string err;
  DeviceState* d = current_device(err);
  if (!d) return fail(FB_ERR_INIT, err);
  int v = 0;
  cudaError_t e = cudaMemcpy(&v, d->status, sizeof(int), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && clear) e = cudaMemset(d->status, 0, sizeof(int));
  if (e != cudaSuccess) return fail(FB_ERR_CUDA, std::string("fb_device_status: ") + cudaGetErrorString(e));
  *code = v;
  return FB_OK;
}

namespace fb {
// Waits, bounded by budget_ns, for a phase of a fresh mbarrier that nothing ever completes: the wait
// gives up, records FB_DEV_TIMEOUT_EPI in the status word (as every kernel's bounded waits do) and
// the kernel returns normally.
__global__ void selftest_wait_kernel(int* status, uint64_t budget_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(&bar, 0)) {
      if (globaltimer_ns() - t0 > budget_ns) {
        atomicCAS(status, 0, FB_DEV_TIMEOUT_EPI);
        break;
      }
    }
  }
}

extern "C++" cudaError_t launch_selftest_wait(int* status, uint64_t budget_ns, cudaStream_t st) {
  selftest_wait_kernel<<<1, 32, 0, st>>>(status, budget_ns);
  return cudaGetLastError();
}
}  // namespace fb

int32_t fb_selftest_wait_timeout(int32_t budget_ms, void* stream) {
  if (budget_ms <= 0 || budget_ms > 1000) return fail(FB_ERR_ARG, "fb_selftest_wait_timeout: budget_ms in 1..1000");
  std::string err;
  DeviceState* d = current_device(err);
  if (!d) return fail(FB_ERR_INIT, err);
  const cudaError_t e =
      fb::launch_selftest_wait(d->status, static_cast<uint64_t>(budget_ms) * 1000000ull, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(FB_ERR_CUDA, std::string("fb_selftest_wait_timeout: ") + cudaGetErrorString(e));
  return FB_OK;
}

static int ready_or_fail() {
  if (g_init_rc != FB_OK) {
    const int rc = fb_init();
    if (rc != FB_OK) return rc;
  }
  return FB_OK;
}

static int cuda_rc(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return FB_OK;
  return fail(FB_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int32_t fb_nf4_dequant(const uint8_t* packed, const float* absmax, const float* code16, int64_t n_bytes,
                       int32_t blocksize, void* out, int32_t out_dtype, void* stream) {
  if (int rc = ready_or_fail()) return rc;
  if (n_bytes < 0 || blocksize <= 0 || blocksize % 2 != 0 || (n_bytes * 2) % blocksize != 0)
    return fail(FB_ERR_ARG, "fb_nf4_dequant: need an even blocksize dividing 2 * n_bytes");
  if (out_dtype != FB_F32 && out_dtype != FB_F16 && out_dtype != FB_BF16)
    return fail(FB_ERR_ARG, "fb_nf4_dequant: out_dtype must be FB_F32, FB_F16 or FB_BF16");
  if (n_bytes > 0 && (!packed || !absmax || !code16 || !out)) return fail(FB_ERR_ARG, "fb_nf4_dequant: null pointer");
  const size_t esz = out_dtype == FB_F32 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(out) % esz) != 0 || (reinterpret_cast<uintptr_t>(absmax) % 4) != 0 ||
      (reinterpret_cast<uintptr_t>(code16) % 4) != 0)
    return fail(FB_ERR_ALIGN, "fb_nf4_dequant: misaligned out/absmax/code16");
  return cuda_rc(launch_nf4_dequant(packed, absmax, code16, n_bytes, blocksize, out, out_dtype,
                                    static_cast<cudaStream_t>(stream)),
                 "fb_nf4_dequant");
}

int32_t fb_ln_mod(const float* x, int64_t rows, int32_t dim, int32_t rows_per_batch, const uint16_t* shift,
                  const uint16_t* scale, int64_t mod_batch_stride, uint16_t* out, void* stream) {
  if (int rc = ready_or_fail()) return rc;
  if (rows < 0 || dim <= 0 || dim % 4 != 0 || rows_per_batch <= 0)
    return fail(FB_ERR_ARG, "fb_ln_mod: need rows >= 0, dim % 4 == 0, rows_per_batch > 0");
  const uintptr_t a = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out);
  const uintptr_t m = reinterpret_cast<uintptr_t>(shift) | reinterpret_cast<uintptr_t>(scale);
  if ((a & 15u) || (m & 7u) || (mod_batch_stride % 4) != 0)
    return fail(FB_ERR_ALIGN, "fb_ln_mod: x/out must be 16-byte aligned, shift/scale 8-byte aligned, stride % 4");
  return cuda_rc(launch_ln_mod(x, rows, dim, rows_per_batch, shift, scale, mod_batch_stride, out,
                               static_cast<cudaStream_t>(stream)),
                 "fb_ln_mod");
}

int32_t fb_ln_mod_grouped(const fb_ln_mod_problem* problems, int32_t count, void* stream) {
  if (int rc = ready_or_fail()) return rc;
  if (!problems || count < 1 || count > 2) return fail(FB_ERR_ARG, "fb_ln_mod_grouped: need 1 or 2 problems");
  for (int i = 0; i < count; ++i) {
    const fb_ln_mod_problem& p = problems[i];
    if (p.rows < 0 || p.dim <= 0 || p.dim % 4 != 0 || p.rows_per_batch <= 0)
      return fail(FB_ERR_ARG, "fb_ln_mod_grouped: need rows >= 0, dim % 4 == 0, rows_per_batch > 0");
    const uintptr_t a = reinterpret_cast<uintptr_t>(p.x) | reinterpret_cast<uintptr_t>(p.out);
    const uintptr_t m = reinterpret_cast<uintptr_t>(p.shift) | reinterpret_cast<uintptr_t>(p.scale);
    if ((a & 15u) || (m & 7u) || (p.mod_batch_stride % 4) != 0)
      return fail(FB_ERR_ALIGN, "fb_ln_mod_grouped: x/out 16-byte aligned, shift/scale 8-byte aligned, stride % 4");
  }
  return cuda_rc(launch_ln_mod_grouped(problems, count, static_cast<cudaStream_t>(stream)), "fb_ln_mod_grouped");
}

int32_t fb_linear_grouped(const fb_linear* problems, int32_t count, int32_t epilogue, void* stream) {
  if (int rc = ready_or_fail()) return rc;
  if (!problems) return fail(FB_ERR_ARG, "fb_linear_grouped: null problems");
  std::string err;
  const int rc = launch_linear_grouped(problems, count, epilogue, static_cast<cudaStream_t>(stream), err);
  return rc ? fail(rc, err) : FB_OK;
}

int32_t fb_linear_nf4(const fb_linear* problem, int32_t epilogue, void* workspace, int64_t workspace_bytes,
                      void* stream) {
  if (int rc = ready_or_fail()) return rc;
  if (!problem) return fail(FB_ERR_ARG, "fb_linear_nf4: null problem");
  std::string err;
  DeviceState* d = current_device(err);
  if (!d) return fail(FB_ERR_INIT, err);
  const int rc = launch_linear_nf4(*problem, epilogue, workspace, workspace_bytes, d->status, d->sm_count,
                                   static_cast<cudaStream_t>(stream), err);
  return rc ? fail(rc, err) : FB_OK;
}

int32_t fb_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out, int64_t ld_out,
                     int32_t batch, int32_t heads, int32_t seq, int32_t head_dim, float scale, void* stream) {
  if (int rc = ready_or_fail()) return rc;
  std::string err;
  const int rc = launch_attention(q, k, v, nullptr, 0, out, ld_out, 0, batch, heads, seq, head_dim, scale,
                                  static_cast<cudaStream_t>(stream), err);
  return rc ? fail(rc, err) : FB_OK;
}

int32_t fb_attention_split(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out0, int64_t ld0,
                           uint16_t* out1, int64_t ld1, int32_t split, int32_t batch, int32_t heads, int32_t seq,
                           int32_t head_dim, float scale, void* stream) {
  if (int rc = ready_or_fail()) return rc;
  std::string err;
  const int rc = launch_attention(q, k, v, out0, ld0, out1, ld1, split, batch, heads, seq, head_dim, scale,
                                  static_cast<cudaStream_t>(stream), err);
  return rc ? fail(rc, err) : FB_OK;
}

int32_t fb_attention_sp(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* const* out_peers,
                        int64_t ld_out, int32_t col0, int32_t heads, int32_t seq_local, int32_t sp_world,
                        int32_t head_dim, float scale, void* stream) {
  if (int rc = ready_or_fail()) return rc;
  std::string err;
  const int rc = launch_attention_sp(q, k, v, out_peers, ld_out, col0, heads, seq_local, sp_world, head_dim, scale,
                                     static_cast<cudaStream_t>(stream), err);
  return rc ? fail(rc, err) : FB_OK;
}

int32_t fb_gated_add(const float* x, const uint16_t* g, const uint16_t* y, float* out, int64_t rows, int32_t dim,
                     int32_t rows_per_batch, int64_t g_batch_stride, int32_t guard, void* stream) {
  if (int rc = ready_or_fail()) return rc;
  if (rows < 0 || dim <= 0 || dim % 4 != 0 || rows_per_batch <= 0)
    return fail(FB_ERR_ARG, "fb_gated_add: need dim % 4 == 0 and rows_per_batch > 0");
  const uintptr_t a = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out);
  const uintptr_t b = reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(y);
  if ((a & 15u) || (b & 7u) || (g_batch_stride % 4) != 0)
    return fail(FB_ERR_ALIGN, "fb_gated_add: x/out 16-byte aligned, g/y 8-byte aligned, g stride % 4");
  return cuda_rc(launch_gated_add(x, g, y, out, rows, dim, rows_per_batch, g_batch_stride, guard,
                                  static_cast<cudaStream_t>(stream)),
                 "fb_gated_add");
}

int32_t fb_gelu_tanh(const uint16_t* h, uint16_t* out, int64_t n, void* stream) {
  if (int rc = ready_or_fail()) return rc;
  if (n < 0 || n % 8 != 0) return fail(FB_ERR_ARG, "fb_gelu_tanh: n must be a multiple of 8");
  if ((reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(out)) & 15u)
    return fail(FB_ERR_ALIGN, "fb_gelu_tanh: h/out must be 16-byte aligned");
  return cuda_rc(launch_gelu(h, out, n, static_cast<cudaStream_t>(stream)), "fb_gelu_tanh");
}

int32_t fb_qk_norm_rope(const uint16_t* qkv, int64_t ld_qkv, int32_t batch, int32_t rows, int32_t heads,
                        int32_t head_dim, const float* q_scale, const float* k_scale, const float* rope_cos,
                        const float* rope_sin, uint16_t* q, uint16_t* k, uint16_t* v, int32_t seq_total,
                        int32_t seq_offset, void* stream) {
  if (int rc = ready_or_fail()) return rc;
  if (head_dim != 128 && head_dim != 64) return fail(FB_ERR_UNSUPPORTED, "fb_qk_norm_rope: head_dim must be 64 or 128");
  if (batch < 0 || rows < 0 || heads <= 0 || seq_offset < 0 || seq_offset + rows > seq_total ||
      ld_qkv < 3LL * heads * head_dim)
    return fail(FB_ERR_ARG, "fb_qk_norm_rope: bad shape");
  if ((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
       reinterpret_cast<uintptr_t>(v)) & 3u || (ld_qkv & 1))
    return fail(FB_ERR_ALIGN, "fb_qk_norm_rope: 4-byte alignment needed");
  return cuda_rc(launch_qk_norm_rope(qkv, ld_qkv, batch, rows, heads, head_dim, q_scale, k_scale, rope_cos, rope_sin,
                                     q, k, v, seq_total, seq_offset, static_cast<cudaStream_t>(stream)),
                 "fb_qk_norm_rope");
}

}  // extern "C"
