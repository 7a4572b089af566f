// encode.cu — weight encoders on the device (conversion time): NF4 (selas/codecs.py:99-119) and int8_row
// (selas/codecs.py:87-97), bit-exact with selas's torch code on the same input values.
//
// Both are HBM-bound streams: each input element is read once (fp32, bf16 or fp16), the packed codes and
// the per-block / per-row scales written once.
//
// NF4: one warp per block of `blocksize` values. Lane l owns packed byte l (+32, +64, ...), i.e. the
// values 2l and 2l + 1: absmax is a warp max of |v|; each value is divided by it (IEEE fp32 division,
// 1 for an all-zero block) and bucketized against the 15 midpoints (c[i] + c[i+1]) / 2 of the code
// table: the code index is the number of midpoints strictly below the value, which puts a value that
// equals a midpoint in the lower code (torch.bucketize(right=False), the bitsandbytes tie rule). The
// first value of a pair goes to the high nibble.
//
// int8_row: one CTA per row: absmax by a block reduction, scale = absmax / 127 (1 for an all-zero row),
// q = clamp(round_half_even(w / scale), -127, 127).
#include <cuda_fp16.h>

#include "fb_internal.h"

namespace fb {
namespace {

template <int DT>
__device__ __forceinline__ float2 load2(const void* p, int64_t i) {  // values 2i, 2i + 1
  if constexpr (DT == FB_F32) {
    return __ldg(reinterpret_cast<const float2*>(p) + i);
  } else {
    const uint32_t u = __ldg(reinterpret_cast<const uint32_t*>(p) + i);
    if constexpr (DT == FB_BF16) {
      return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xFFFF0000u));
    } else {
      const __half2 h = *reinterpret_cast<const __half2*>(&u);
      return __half22float2(h);
    }
  }
}

template <int DT>
__device__ __forceinline__ float load1(const void* p, int64_t i) {
  if constexpr (DT == FB_F32) {
    return __ldg(reinterpret_cast<const float*>(p) + i);
  } else if constexpr (DT == FB_BF16) {
    return __uint_as_float(static_cast<uint32_t>(__ldg(reinterpret_cast<const unsigned short*>(p) + i)) << 16);
  } else {
    return __half2float(__ldg(reinterpret_cast<const __half*>(p) + i));
  }
}

__device__ __forceinline__ uint32_t bucket(float x, const float (&mids)[15]) {
  uint32_t n = 0;
#pragma unroll
  for (int i = 0; i < 15; ++i) n += mids[i] < x ? 1u : 0u;
  return n;
}

template <int DT>
__global__ void __launch_bounds__(256) nf4_encode_kernel(const void* __restrict__ w, int64_t nblocks, int blocksize,
                                                         const float* __restrict__ code16, uint8_t* __restrict__ packed,
                                                         float* __restrict__ absmax_out) {
  float mids[15];
#pragma unroll
  for (int i = 0; i < 15; ++i) mids[i] = __fmul_rn(__fadd_rn(__ldg(code16 + i + 1), __ldg(code16 + i)), 0.5f);
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int half = blocksize >> 1;  // packed bytes per block
  for (int64_t blk = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); blk < nblocks;
       blk += warps) {
    const int64_t p0 = blk * half;  // first value pair of the block
    float m = 0.f;
    for (int j = lane; j < half; j += 32) {
      const float2 v = load2<DT>(w, p0 + j);
      m = fmaxf(m, fmaxf(fabsf(v.x), fabsf(v.y)));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float safe = m > 0.f ? m : 1.f;
    for (int j = lane; j < half; j += 32) {
      const float2 v = load2<DT>(w, p0 + j);
      const uint32_t hi = bucket(__fdiv_rn(v.x, safe), mids), lo = bucket(__fdiv_rn(v.y, safe), mids);
      packed[p0 + j] = static_cast<uint8_t>((hi << 4) | lo);
    }
    if (lane == 0) absmax_out[blk] = m;
  }
}

// 8 consecutive values (16-byte loads; fp32 takes two).
template <int DT>
__device__ __forceinline__ void load8(const void* p, int64_t i8, float (&v)[8]) {
  if constexpr (DT == FB_F32) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p) + 2 * i8);
    const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 2 * i8 + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p) + i8);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if constexpr (DT == FB_BF16) {
        v[2 * k] = __uint_as_float(w[k] << 16);
        v[2 * k + 1] = __uint_as_float(w[k] & 0xFFFF0000u);
      } else {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[k]));
        v[2 * k] = f.x;
        v[2 * k + 1] = f.y;
      }
    }
  }
}

// NF4 for blocksize = 8 * L (L a power of two <= 32): L lanes per block, 8 values and 4 packed bytes per
// lane, 32 / L blocks per warp step; the block's absmax by an L-lane butterfly. Same arithmetic as
// nf4_encode_kernel, 4x fewer memory instructions.
template <int DT, int L>
__global__ void __launch_bounds__(256) nf4_encode8_kernel(const void* __restrict__ w, int64_t nblocks,
                                                          const float* __restrict__ code16, uint8_t* __restrict__ packed,
                                                          float* __restrict__ absmax_out) {
  float mids[15];
#pragma unroll
  for (int i = 0; i < 15; ++i) mids[i] = __fmul_rn(__fadd_rn(__ldg(code16 + i + 1), __ldg(code16 + i)), 0.5f);
  const int lane = threadIdx.x & 31;
  const int sub = lane % L;  // this lane's 8 values within its block
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t units = (nblocks + (32 / L) - 1) / (32 / L);  // warp steps
  for (int64_t u = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); u < units; u += warps) {
    const int64_t blk = u * (32 / L) + lane / L;
    const bool ok = blk < nblocks;
    float v[8];
    float m = 0.f;
    if (ok) {
      load8<DT>(w, blk * L + sub, v);
#pragma unroll
      for (int k = 0; k < 8; ++k) m = fmaxf(m, fabsf(v[k]));
    }
#pragma unroll
    for (int o = L / 2; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (!ok) continue;
    const float safe = m > 0.f ? m : 1.f;
    uint32_t word = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t hi = bucket(__fdiv_rn(v[2 * k], safe), mids), lo = bucket(__fdiv_rn(v[2 * k + 1], safe), mids);
      word |= ((hi << 4) | lo) << (8 * k);
    }
    reinterpret_cast<uint32_t*>(packed)[blk * L + sub] = word;
    if (sub == 0) absmax_out[blk] = m;
  }
}

template <int DT>
__global__ void __launch_bounds__(256) int8_row_encode_kernel(const void* __restrict__ w, int64_t cols,
                                                              int8_t* __restrict__ q, float* __restrict__ scale_out) {
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  const int64_t base = row * cols;
  const bool vec = cols % 8 == 0;  // rows of whole 8-value groups: 16-byte loads, 8-byte stores
  float m = 0.f;
  if (vec) {
    for (int64_t c8 = threadIdx.x; c8 < cols / 8; c8 += blockDim.x) {
      float v[8];
      load8<DT>(w, base / 8 + c8, v);
#pragma unroll
      for (int k = 0; k < 8; ++k) m = fmaxf(m, fabsf(v[k]));
    }
  } else {
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) m = fmaxf(m, fabsf(load1<DT>(w, base + c)));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  m = red[0];
  for (int i = 1; i < static_cast<int>(blockDim.x >> 5); ++i) m = fmaxf(m, red[i]);
  const float scale = m > 0.f ? __fdiv_rn(m, 127.0f) : 1.0f;
  if (vec) {
    for (int64_t c8 = threadIdx.x; c8 < cols / 8; c8 += blockDim.x) {
      float v[8];
      load8<DT>(w, base / 8 + c8, v);
      uint32_t lo = 0, hi = 0;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int32_t r = static_cast<int32_t>(fminf(fmaxf(rintf(__fdiv_rn(v[k], scale)), -127.f), 127.f));
        const uint32_t b = static_cast<uint32_t>(r) & 0xFFu;
        if (k < 4) lo |= b << (8 * k); else hi |= b << (8 * (k - 4));
      }
      reinterpret_cast<uint2*>(q + base)[c8] = make_uint2(lo, hi);
    }
  } else {
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
      const float r = rintf(__fdiv_rn(load1<DT>(w, base + c), scale));
      q[base + c] = static_cast<int8_t>(fminf(fmaxf(r, -127.f), 127.f));
    }
  }
  if (threadIdx.x == 0) scale_out[row] = scale;
}

int fail(int code, const std::string& msg) {
  set_last_error(msg);
  return code;
}

int launched(const char* what) {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? FB_OK : fail(FB_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

}  // namespace
}  // namespace fb

using namespace fb;

extern "C" {

int32_t fb_nf4_encode(const void* w, int32_t w_dtype, int64_t n, int32_t blocksize, const float* code16,
                      uint8_t* packed, float* absmax, void* stream) {
  std::string err;
  if (!current_device(err)) return fail(FB_ERR_INIT, "fb_nf4_encode: " + err);
  if (n < 0 || blocksize <= 0 || blocksize % 2 || n % blocksize || (w_dtype != FB_F32 && w_dtype != FB_BF16 &&
                                                                    w_dtype != FB_F16))
    return fail(FB_ERR_ARG, "fb_nf4_encode: need an even blocksize dividing n and w_dtype FB_F32/FB_BF16/FB_F16");
  if (n == 0) return FB_OK;
  if (!w || !code16 || !packed || !absmax) return fail(FB_ERR_ARG, "fb_nf4_encode: null pointer");
  const uintptr_t wa = reinterpret_cast<uintptr_t>(w);
  if ((w_dtype == FB_F32 ? wa & 7u : wa & 3u) || (reinterpret_cast<uintptr_t>(absmax) & 3u) ||
      (reinterpret_cast<uintptr_t>(code16) & 3u))
    return fail(FB_ERR_ALIGN, "fb_nf4_encode: w must be aligned to a value pair, absmax/code16 to 4 bytes");
  const int64_t nblocks = n / blocksize;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int esz = w_dtype == FB_F32 ? 4 : 2;
  const bool vec = (blocksize == 64 || blocksize == 128) && (wa % 16u) == 0 && (reinterpret_cast<uintptr_t>(packed) & 3u) == 0;
  if (vec) {
    // 8 values per lane: blocksize 64 -> 8 lanes, 128 -> 16 lanes per block
    const int64_t per_warp = 32 / (blocksize / 8);
    const int64_t warps = (nblocks + per_warp - 1) / per_warp;
    const int grid = static_cast<int>(std::min<int64_t>((warps + 7) / 8, 16 * kNumSms));
    (void)esz;
    if (blocksize == 64) {
      switch (w_dtype) {
        case FB_F32: nf4_encode8_kernel<FB_F32, 8><<<grid, 256, 0, st>>>(w, nblocks, code16, packed, absmax); break;
        case FB_BF16: nf4_encode8_kernel<FB_BF16, 8><<<grid, 256, 0, st>>>(w, nblocks, code16, packed, absmax); break;
        default: nf4_encode8_kernel<FB_F16, 8><<<grid, 256, 0, st>>>(w, nblocks, code16, packed, absmax); break;
      }
    } else {
      switch (w_dtype) {
        case FB_F32: nf4_encode8_kernel<FB_F32, 16><<<grid, 256, 0, st>>>(w, nblocks, code16, packed, absmax); break;
        case FB_BF16: nf4_encode8_kernel<FB_BF16, 16><<<grid, 256, 0, st>>>(w, nblocks, code16, packed, absmax); break;
        default: nf4_encode8_kernel<FB_F16, 16><<<grid, 256, 0, st>>>(w, nblocks, code16, packed, absmax); break;
      }
    }
    return launched("fb_nf4_encode");
  }
  const int grid = static_cast<int>(std::min<int64_t>((nblocks + 7) / 8, 16 * kNumSms));
  switch (w_dtype) {
    case FB_F32: nf4_encode_kernel<FB_F32><<<grid, 256, 0, st>>>(w, nblocks, blocksize, code16, packed, absmax); break;
    case FB_BF16: nf4_encode_kernel<FB_BF16><<<grid, 256, 0, st>>>(w, nblocks, blocksize, code16, packed, absmax); break;
    default: nf4_encode_kernel<FB_F16><<<grid, 256, 0, st>>>(w, nblocks, blocksize, code16, packed, absmax); break;
  }
  return launched("fb_nf4_encode");
}

int32_t fb_int8_row_encode(const void* w, int32_t w_dtype, int64_t rows, int64_t cols, int8_t* q, float* scale,
                           void* stream) {
  std::string err;
  if (!current_device(err)) return fail(FB_ERR_INIT, "fb_int8_row_encode: " + err);
  if (rows < 0 || cols <= 0 || rows > 0x7fffffff || (w_dtype != FB_F32 && w_dtype != FB_BF16 && w_dtype != FB_F16))
    return fail(FB_ERR_ARG, "fb_int8_row_encode: need rows >= 0, cols > 0 and w_dtype FB_F32/FB_BF16/FB_F16");
  if (rows == 0) return FB_OK;
  if (!w || !q || !scale) return fail(FB_ERR_ARG, "fb_int8_row_encode: null pointer");
  if ((reinterpret_cast<uintptr_t>(w) & 15u) || (reinterpret_cast<uintptr_t>(q) & 7u) ||
      (reinterpret_cast<uintptr_t>(scale) & 3u))
    return fail(FB_ERR_ALIGN, "fb_int8_row_encode: w must be 16-byte aligned, q 8-byte, scale 4-byte");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (w_dtype) {
    case FB_F32: int8_row_encode_kernel<FB_F32><<<static_cast<unsigned>(rows), 256, 0, st>>>(w, cols, q, scale); break;
    case FB_BF16: int8_row_encode_kernel<FB_BF16><<<static_cast<unsigned>(rows), 256, 0, st>>>(w, cols, q, scale); break;
    default: int8_row_encode_kernel<FB_F16><<<static_cast<unsigned>(rows), 256, 0, st>>>(w, cols, q, scale); break;
  }
  return launched("fb_int8_row_encode");
}

}  // extern "C"
