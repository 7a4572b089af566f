// stepcache.cu — the device side of selas's step cache (selas/stepcache.py): the probe distance
// reduction, the residual prediction and the residual capture. All three are HBM-bound streams over
// the fp32 hidden state ([B, L, 3072] fp32: 50 MB per image at 1024^2), so each reads every input
// once with 16-byte loads, on a grid of a few blocks per SM that loops over the vector.
//
// * fb_probe_distance — selas/stepcache.py:127-129 with the residual of selas/models/flux.py:548:
//   r = x - x_in (written out when asked: the next reference if the step is computed in full), and
//   sum|r - ref|, sum|ref| in fp64. The elementwise values are the reference's own fp32 ops
//   (r, r - ref and |.| each rounded once); the sums are fp64 (more exact than an fp32 mean), block
//   partials reduced by a second one-block kernel in a fixed order (deterministic).
// * fb_residual_predict — _Hist.predict (selas/stepcache.py:84-94) plus the add of
//   selas/models/flux.py:553 / :571: p = r1 + a * (r1 - r0) (or p = r1), out = x + p, every op an
//   fp32 op rounded once, as torch's separate elementwise kernels do (bit-exact).
// * fb_residual_diff — the residual capture of selas/models/flux.py:566 / :576 / :580:
//   r = (x - x0) cast to fp32 or bf16 (round to nearest even).
#include "fb_internal.h"

namespace fb {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxBlocks = 8 * kNumSms;  // partial sums per launch: 2 * kMaxBlocks doubles
static_assert(2 + 2 * kMaxBlocks <= FB_PROBE_WORK_DOUBLES, "probe workspace too small");

int blocks_for(int64_t n4) {
  const int64_t b = (n4 + kThreads - 1) / kThreads;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(b, kMaxBlocks)));
}

__device__ __forceinline__ double block_sum(double v, double* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  double t = 0.0;
  if (threadIdx.x < 32) {
    t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  }
  return t;  // valid in thread 0
}

__global__ void __launch_bounds__(kThreads) probe_kernel(const float4* __restrict__ x, const float4* __restrict__ x_in,
                                                         const float4* __restrict__ ref, float4* __restrict__ resid,
                                                         int64_t n4, double* __restrict__ work) {
  __shared__ double red[kThreads / 32];
  double s_diff = 0.0, s_ref = 0.0;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < n4; i += stride) {
    float4 r = __ldg(x + i);
    if (x_in) {
      const float4 b = __ldg(x_in + i);
      r = make_float4(__fsub_rn(r.x, b.x), __fsub_rn(r.y, b.y), __fsub_rn(r.z, b.z), __fsub_rn(r.w, b.w));
    }
    if (resid) resid[i] = r;
    if (ref) {
      const float4 q = __ldg(ref + i);
      // |r - ref| per element in fp32, summed in fp64; fp32 partials of four would round again
      s_diff += static_cast<double>(fabsf(__fsub_rn(r.x, q.x))) + static_cast<double>(fabsf(__fsub_rn(r.y, q.y))) +
                static_cast<double>(fabsf(__fsub_rn(r.z, q.z))) + static_cast<double>(fabsf(__fsub_rn(r.w, q.w)));
      s_ref += static_cast<double>(fabsf(q.x)) + static_cast<double>(fabsf(q.y)) + static_cast<double>(fabsf(q.z)) +
               static_cast<double>(fabsf(q.w));
    }
  }
  if (!ref) return;
  const double a = block_sum(s_diff, red);
  const double b = block_sum(s_ref, red);
  if (threadIdx.x == 0) {
    work[2 + 2 * blockIdx.x] = a;
    work[3 + 2 * blockIdx.x] = b;
  }
}

__global__ void __launch_bounds__(kThreads) probe_finish_kernel(double* __restrict__ work, int parts) {
  __shared__ double red[kThreads / 32];
  double a = 0.0, b = 0.0;
  for (int i = threadIdx.x; i < parts; i += kThreads) {
    a += work[2 + 2 * i];
    b += work[3 + 2 * i];
  }
  const double sa = block_sum(a, red);
  const double sb = block_sum(b, red);
  if (threadIdx.x == 0) {
    work[0] = sa;
    work[1] = sb;
  }
}

template <bool kBf16>
__device__ __forceinline__ float4 load4(const void* p, int64_t i) {
  if constexpr (kBf16) {
    const uint2 u = __ldg(reinterpret_cast<const uint2*>(p) + i);
    return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u), __uint_as_float(u.y << 16),
                       __uint_as_float(u.y & 0xffff0000u));
  } else {
    return __ldg(reinterpret_cast<const float4*>(p) + i);
  }
}

__device__ __forceinline__ float predict1(float r1, float r0, float a) {
  return __fadd_rn(r1, __fmul_rn(a, __fsub_rn(r1, r0)));
}

template <bool kBf16>
__global__ void __launch_bounds__(kThreads) predict_kernel(const float4* __restrict__ x, const void* __restrict__ r1,
                                                           const void* __restrict__ r0, float a,
                                                           float4* __restrict__ out, int64_t n4) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < n4; i += stride) {
    float4 p = load4<kBf16>(r1, i);
    if (r0) {
      const float4 q = load4<kBf16>(r0, i);
      p = make_float4(predict1(p.x, q.x, a), predict1(p.y, q.y, a), predict1(p.z, q.z, a), predict1(p.w, q.w, a));
    }
    if (x) {
      const float4 b = __ldg(x + i);
      p = make_float4(__fadd_rn(b.x, p.x), __fadd_rn(b.y, p.y), __fadd_rn(b.z, p.z), __fadd_rn(b.w, p.w));
    }
    out[i] = p;
  }
}

__global__ void __launch_bounds__(kThreads) diff_kernel(const float4* __restrict__ x, const float4* __restrict__ x0,
                                                        void* __restrict__ r, int bf16, int64_t n4) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < n4; i += stride) {
    const float4 a = __ldg(x + i), b = __ldg(x0 + i);
    const float4 d = make_float4(__fsub_rn(a.x, b.x), __fsub_rn(a.y, b.y), __fsub_rn(a.z, b.z), __fsub_rn(a.w, b.w));
    if (bf16) {
      reinterpret_cast<uint2*>(r)[i] = make_uint2(pack_bf16x2(d.x, d.y), pack_bf16x2(d.z, d.w));
    } else {
      reinterpret_cast<float4*>(r)[i] = d;
    }
  }
}

int fail(int code, const std::string& msg) {
  set_last_error(msg);
  return code;
}

int launched(const char* what) {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? FB_OK : fail(FB_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

bool misaligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) != 0; }

int ready(const char* what) {
  std::string err;
  if (!current_device(err)) return fail(FB_ERR_INIT, std::string(what) + ": " + err);
  return FB_OK;
}

}  // namespace
}  // namespace fb

using namespace fb;

extern "C" {

int32_t fb_probe_distance(const float* x, const float* x_in, const float* ref, float* resid, int64_t n, double* work,
                          void* stream) {
  if (int rc = ready("fb_probe_distance")) return rc;
  if (n < 0 || n % 4 != 0 || !x || (ref && !work))
    return fail(FB_ERR_ARG, "fb_probe_distance: need n % 4 == 0, x, and a workspace when ref is given");
  if (misaligned(x, 16) || misaligned(x_in, 16) || misaligned(ref, 16) || misaligned(resid, 16) || misaligned(work, 8))
    return fail(FB_ERR_ALIGN, "fb_probe_distance: x, x_in, ref and resid must be 16-byte aligned");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t n4 = n / 4;
  const int grid = blocks_for(n4);
  probe_kernel<<<grid, kThreads, 0, st>>>(reinterpret_cast<const float4*>(x), reinterpret_cast<const float4*>(x_in),
                                          reinterpret_cast<const float4*>(ref), reinterpret_cast<float4*>(resid), n4,
                                          work);
  if (ref) probe_finish_kernel<<<1, kThreads, 0, st>>>(work, grid);
  return launched("fb_probe_distance");
}

int32_t fb_residual_predict(const float* x, const void* r1, const void* r0, int32_t r_dtype, float a, float* out,
                            int64_t n, void* stream) {
  if (int rc = ready("fb_residual_predict")) return rc;
  if (n < 0 || n % 4 != 0 || !r1 || !out || (r_dtype != FB_F32 && r_dtype != FB_BF16))
    return fail(FB_ERR_ARG, "fb_residual_predict: need n % 4 == 0, r1, out, and r_dtype FB_F32 or FB_BF16");
  const uintptr_t ra = r_dtype == FB_F32 ? 16 : 8;
  if (misaligned(x, 16) || misaligned(out, 16) || misaligned(r1, ra) || misaligned(r0, ra))
    return fail(FB_ERR_ALIGN, "fb_residual_predict: x/out 16-byte aligned, residuals 16 (f32) or 8 (bf16) bytes");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t n4 = n / 4;
  const int grid = blocks_for(n4);
  if (r_dtype == FB_BF16)
    predict_kernel<true><<<grid, kThreads, 0, st>>>(reinterpret_cast<const float4*>(x), r1, r0, a,
                                                    reinterpret_cast<float4*>(out), n4);
  else
    predict_kernel<false><<<grid, kThreads, 0, st>>>(reinterpret_cast<const float4*>(x), r1, r0, a,
                                                     reinterpret_cast<float4*>(out), n4);
  return launched("fb_residual_predict");
}

int32_t fb_residual_diff(const float* x, const float* x0, void* r, int32_t r_dtype, int64_t n, void* stream) {
  if (int rc = ready("fb_residual_diff")) return rc;
  if (n < 0 || n % 4 != 0 || !x || !x0 || !r || (r_dtype != FB_F32 && r_dtype != FB_BF16))
    return fail(FB_ERR_ARG, "fb_residual_diff: need n % 4 == 0, x, x0, r, and r_dtype FB_F32 or FB_BF16");
  if (misaligned(x, 16) || misaligned(x0, 16) || misaligned(r, r_dtype == FB_F32 ? 16 : 8))
    return fail(FB_ERR_ALIGN, "fb_residual_diff: x/x0 16-byte aligned, r 16 (f32) or 8 (bf16) bytes");
  const int64_t n4 = n / 4;
  diff_kernel<<<blocks_for(n4), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const float4*>(x), reinterpret_cast<const float4*>(x0), r, r_dtype == FB_BF16, n4);
  return launched("fb_residual_diff");
}

}  // extern "C"
