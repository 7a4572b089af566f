// glue.cu — the memory-bound kernels of the FLUX step: NF4 decode, LayerNorm + adaLN modulation,
// and the elementwise segments (gated residual add, GELU-tanh, QK-RMSNorm + RoPE + head split).
//
// All of them are HBM-bound: 16-byte vector loads/stores where alignment allows, one warp per row
// for the row reductions (warp-shuffle sums, no shared memory), grids sized to the 148 SMs.
#include "fb_internal.h"

namespace fb {

// ============================================================================================ NF4

// Bit-exact NF4 decode (selas/codecs.py:178-199, :211-221): value = fp32(code[nibble]) *
// fp32(absmax[block]) with one IEEE multiply, then a round-to-nearest-even cast. The high nibble of
// byte i is element 2i.
template <typename OutT>
__device__ __forceinline__ OutT cvt_out(float v);
template <>
__device__ __forceinline__ float cvt_out<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half cvt_out<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 cvt_out<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// Vector path: 16 packed bytes (32 outputs) per thread step; packed and out 16-B aligned.
// bytes_per_block % 16 == 0, so one chunk shares one absmax.
template <typename OutT>
__global__ void __launch_bounds__(256) nf4_dequant_vec_kernel(const uint8_t* __restrict__ packed,
                                                              const float* __restrict__ absmax,
                                                              const float* __restrict__ code16, int64_t n_chunks,
                                                              int chunks_per_block, OutT* __restrict__ out) {
  __shared__ float code[16];
  if (threadIdx.x < 16) code[threadIdx.x] = code16[threadIdx.x];
  __syncthreads();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < n_chunks; c += stride) {
    const uint4 p = __ldg(reinterpret_cast<const uint4*>(packed) + c);
    const float s = __ldg(absmax + c / chunks_per_block);
    const uint32_t words[4] = {p.x, p.y, p.z, p.w};
    alignas(16) OutT vals[32];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const uint32_t byte = (words[w] >> (8 * b)) & 0xFFu;
        vals[8 * w + 2 * b] = cvt_out<OutT>(__fmul_rn(code[byte >> 4], s));
        vals[8 * w + 2 * b + 1] = cvt_out<OutT>(__fmul_rn(code[byte & 15u], s));
      }
    }
    uint4* dst = reinterpret_cast<uint4*>(out + 32 * c);
    const uint4* src = reinterpret_cast<const uint4*>(vals);
#pragma unroll
    for (int i = 0; i < static_cast<int>(32 * sizeof(OutT) / 16); ++i) dst[i] = src[i];
  }
}

// Scalar path for any alignment / block size: one packed byte per thread step.
template <typename OutT>
__global__ void __launch_bounds__(256) nf4_dequant_scalar_kernel(const uint8_t* __restrict__ packed,
                                                                 const float* __restrict__ absmax,
                                                                 const float* __restrict__ code16, int64_t n_bytes,
                                                                 int bytes_per_block, OutT* __restrict__ out) {
  __shared__ float code[16];
  if (threadIdx.x < 16) code[threadIdx.x] = code16[threadIdx.x];
  __syncthreads();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n_bytes; i += stride) {
    const uint32_t byte = packed[i];
    const float s = absmax[i / bytes_per_block];
    out[2 * i] = cvt_out<OutT>(__fmul_rn(code[byte >> 4], s));
    out[2 * i + 1] = cvt_out<OutT>(__fmul_rn(code[byte & 15u], s));
  }
}

template <typename OutT>
static cudaError_t nf4_launch_t(const uint8_t* packed, const float* absmax, const float* code16, int64_t n_bytes,
                                int blocksize, void* out, cudaStream_t st) {
  const int bpb = blocksize / 2;
  const bool aligned = (reinterpret_cast<uintptr_t>(packed) % 16 == 0) && (reinterpret_cast<uintptr_t>(out) % 16 == 0);
  if (aligned && bpb % 16 == 0 && n_bytes % 16 == 0) {
    const int64_t chunks = n_bytes / 16;
    const int grid = static_cast<int>(std::min<int64_t>((chunks + 255) / 256, kNumSms * 8));
    nf4_dequant_vec_kernel<OutT><<<grid, 256, 0, st>>>(packed, absmax, code16, chunks, bpb / 16,
                                                       static_cast<OutT*>(out));
  } else {
    const int grid = static_cast<int>(std::min<int64_t>((n_bytes + 255) / 256, kNumSms * 8));
    nf4_dequant_scalar_kernel<OutT><<<grid, 256, 0, st>>>(packed, absmax, code16, n_bytes, bpb,
                                                          static_cast<OutT*>(out));
  }
  return cudaGetLastError();
}

cudaError_t launch_nf4_dequant(const uint8_t* packed, const float* absmax, const float* code16, int64_t n_bytes,
                               int blocksize, void* out, int out_dtype, cudaStream_t st) {
  if (n_bytes == 0) return cudaSuccess;
  switch (out_dtype) {
    case FB_F32: return nf4_launch_t<float>(packed, absmax, code16, n_bytes, blocksize, out, st);
    case FB_F16: return nf4_launch_t<__half>(packed, absmax, code16, n_bytes, blocksize, out, st);
    default: return nf4_launch_t<__nv_bfloat16>(packed, absmax, code16, n_bytes, blocksize, out, st);
  }
}

// ============================================================================================ LN + mod

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void ld_bf16x4(const uint16_t* p, float (&f)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  f[0] = __uint_as_float(u.x << 16);
  f[1] = __uint_as_float(u.x & 0xFFFF0000u);
  f[2] = __uint_as_float(u.y << 16);
  f[3] = __uint_as_float(u.y & 0xFFFF0000u);
}

// y = bf16(((x - mean) * rstd) * (1 + scale) + shift): the `_mod_in` segment (flux.py:164-166) with
// F.layer_norm(eps=1e-6, no affine) (flux.py:146-147). Each op rounds to fp32 separately, as the
// eager segment does (no fused multiply-add).
__device__ __forceinline__ float mod_apply(float x, float mean, float rstd, float sc, float sh) {
  const float y = __fmul_rn(__fsub_rn(x, mean), rstd);
  return __fadd_rn(__fmul_rn(y, __fadd_rn(1.0f, sc)), sh);
}

// One warp per row; the row (dim = 128 * VPL floats) stays in registers between the passes.
template <int VPL>
__global__ void __launch_bounds__(256) ln_mod_reg_kernel(const float* __restrict__ x, int64_t rows, int rows_per_batch,
                                                         const uint16_t* __restrict__ shift,
                                                         const uint16_t* __restrict__ scale, int64_t mod_bstride,
                                                         uint16_t* __restrict__ out) {
  constexpr int D = 128 * VPL;
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float4* xr = reinterpret_cast<const float4*>(x + row * D);
  float4 v[VPL];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    v[i] = __ldg(xr + lane + 32 * i);
    s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  }
  const float mean = warp_sum(s) / static_cast<float>(D);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
    q += (a * a + b * b) + (c * c + d * d);
  }
  const float rstd = rsqrtf(warp_sum(q) / static_cast<float>(D) + 1e-6f);
  const int64_t b = row / rows_per_batch;
  const uint16_t* shb = shift + b * mod_bstride;
  const uint16_t* scb = scale + b * mod_bstride;
  uint16_t* o = out + row * D;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int col = 4 * (lane + 32 * i);
    float sh[4], sc[4];
    ld_bf16x4(shb + col, sh);
    ld_bf16x4(scb + col, sc);
    uint2 packed;
    packed.x = pack_bf16x2(mod_apply(v[i].x, mean, rstd, sc[0], sh[0]), mod_apply(v[i].y, mean, rstd, sc[1], sh[1]));
    packed.y = pack_bf16x2(mod_apply(v[i].z, mean, rstd, sc[2], sh[2]), mod_apply(v[i].w, mean, rstd, sc[3], sh[3]));
    *reinterpret_cast<uint2*>(o + col) = packed;
  }
}

// One CTA of THREADS threads per row, VPT float4 per thread (dim = THREADS * 4 * VPT), row held in
// registers: few registers per thread, so many rows are in flight per SM (the one-warp-per-row
// kernel needs ~170 registers at dim 3072 and leaves the memory system under-occupied).
template <int THREADS, int VPT>
__device__ __forceinline__ void ln_mod_cta_row(const float* __restrict__ x, int64_t row, int rows_per_batch,
                                               const uint16_t* __restrict__ shift, const uint16_t* __restrict__ scale,
                                               int64_t mod_bstride, uint16_t* __restrict__ out) {
  constexpr int D = THREADS * 4 * VPT;
  constexpr int W = THREADS / 32;
  __shared__ float red[2][W];
  const int t = threadIdx.x;
  const float4* xr = reinterpret_cast<const float4*>(x + row * D);
  float4 v[VPT];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    v[i] = __ldg(xr + t + THREADS * i);
    s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  }
  s = warp_sum(s);
  if ((t & 31) == 0) red[0][t >> 5] = s;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < W; ++w) tot += red[0][w];
  const float mean = tot / static_cast<float>(D);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
    q += (a * a + b * b) + (c * c + d * d);
  }
  q = warp_sum(q);
  if ((t & 31) == 0) red[1][t >> 5] = q;
  __syncthreads();
  float qt = 0.f;
#pragma unroll
  for (int w = 0; w < W; ++w) qt += red[1][w];
  const float rstd = rsqrtf(qt / static_cast<float>(D) + 1e-6f);
  const int64_t b = row / rows_per_batch;
  const uint16_t* shb = shift + b * mod_bstride;
  const uint16_t* scb = scale + b * mod_bstride;
  uint16_t* o = out + row * D;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int col = 4 * (t + THREADS * i);
    float sh[4], sc[4];
    ld_bf16x4(shb + col, sh);
    ld_bf16x4(scb + col, sc);
    uint2 packed;
    packed.x = pack_bf16x2(mod_apply(v[i].x, mean, rstd, sc[0], sh[0]), mod_apply(v[i].y, mean, rstd, sc[1], sh[1]));
    packed.y = pack_bf16x2(mod_apply(v[i].z, mean, rstd, sc[2], sh[2]), mod_apply(v[i].w, mean, rstd, sc[3], sh[3]));
    *reinterpret_cast<uint2*>(o + col) = packed;
  }
}

template <int THREADS, int VPT>
__global__ void __launch_bounds__(THREADS) ln_mod_cta_kernel(const float* __restrict__ x, int rows_per_batch,
                                                             const uint16_t* __restrict__ shift,
                                                             const uint16_t* __restrict__ scale, int64_t mod_bstride,
                                                             uint16_t* __restrict__ out) {
  ln_mod_cta_row<THREADS, VPT>(x, blockIdx.x, rows_per_batch, shift, scale, mod_bstride, out);
}

// Two LN-mod problems of the same dim in one launch (a double block's txt and img streams): CTAs
// [0, rows of problem 0) take problem 0's rows, the rest problem 1's.
struct LnModPair {
  const float* x[2];
  const uint16_t* shift[2];
  const uint16_t* scale[2];
  uint16_t* out[2];
  int64_t mod_bstride[2];
  int rows_per_batch[2];
  int64_t rows0;
};

template <int THREADS, int VPT>
__global__ void __launch_bounds__(THREADS) ln_mod_pair_kernel(const __grid_constant__ LnModPair g) {
  const int p = static_cast<int64_t>(blockIdx.x) < g.rows0 ? 0 : 1;
  const int64_t row = p ? static_cast<int64_t>(blockIdx.x) - g.rows0 : static_cast<int64_t>(blockIdx.x);
  ln_mod_cta_row<THREADS, VPT>(g.x[p], row, g.rows_per_batch[p], g.shift[p], g.scale[p], g.mod_bstride[p], g.out[p]);
}

// Any dim that is a multiple of 4: three passes over the row (L1/L2 serve the re-reads).
__global__ void __launch_bounds__(256) ln_mod_any_kernel(const float* __restrict__ x, int64_t rows, int D,
                                                         int rows_per_batch, const uint16_t* __restrict__ shift,
                                                         const uint16_t* __restrict__ scale, int64_t mod_bstride,
                                                         uint16_t* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float* xr = x + row * D;
  float s = 0.f;
  for (int c = 4 * lane; c < D; c += 128) {
    const float4 t = *reinterpret_cast<const float4*>(xr + c);
    s += (t.x + t.y) + (t.z + t.w);
  }
  const float mean = warp_sum(s) / static_cast<float>(D);
  float q = 0.f;
  for (int c = 4 * lane; c < D; c += 128) {
    const float4 t = *reinterpret_cast<const float4*>(xr + c);
    const float a = t.x - mean, b = t.y - mean, cc = t.z - mean, d = t.w - mean;
    q += (a * a + b * b) + (cc * cc + d * d);
  }
  const float rstd = rsqrtf(warp_sum(q) / static_cast<float>(D) + 1e-6f);
  const int64_t b = row / rows_per_batch;
  for (int c = 4 * lane; c < D; c += 128) {
    const float4 t = *reinterpret_cast<const float4*>(xr + c);
    float sh[4], sc[4];
    ld_bf16x4(shift + b * mod_bstride + c, sh);
    ld_bf16x4(scale + b * mod_bstride + c, sc);
    uint2 packed;
    packed.x = pack_bf16x2(mod_apply(t.x, mean, rstd, sc[0], sh[0]), mod_apply(t.y, mean, rstd, sc[1], sh[1]));
    packed.y = pack_bf16x2(mod_apply(t.z, mean, rstd, sc[2], sh[2]), mod_apply(t.w, mean, rstd, sc[3], sh[3]));
    *reinterpret_cast<uint2*>(out + row * D + c) = packed;
  }
}

cudaError_t launch_ln_mod(const float* x, int64_t rows, int dim, int rows_per_batch, const uint16_t* shift,
                          const uint16_t* scale, int64_t mod_bstride, uint16_t* out, cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  const int warps = 8;
  const unsigned grid = static_cast<unsigned>((rows + warps - 1) / warps);
  switch (dim) {
    case 256: ln_mod_reg_kernel<2><<<grid, 32 * warps, 0, st>>>(x, rows, rows_per_batch, shift, scale, mod_bstride, out); break;
    case 512: ln_mod_reg_kernel<4><<<grid, 32 * warps, 0, st>>>(x, rows, rows_per_batch, shift, scale, mod_bstride, out); break;
    case 1024: ln_mod_reg_kernel<8><<<grid, 32 * warps, 0, st>>>(x, rows, rows_per_batch, shift, scale, mod_bstride, out); break;
    case 3072:
      ln_mod_cta_kernel<128, 6><<<static_cast<unsigned>(rows), 128, 0, st>>>(x, rows_per_batch, shift, scale,
                                                                             mod_bstride, out);
      break;
    default:
      ln_mod_any_kernel<<<grid, 32 * warps, 0, st>>>(x, rows, dim, rows_per_batch, shift, scale, mod_bstride, out);
  }
  return cudaGetLastError();
}

cudaError_t launch_ln_mod_grouped(const fb_ln_mod_problem* probs, int count, cudaStream_t st) {
  if (count == 2 && probs[0].dim == 3072 && probs[1].dim == 3072 && probs[0].rows > 0 && probs[1].rows > 0 &&
      probs[0].rows + probs[1].rows <= 0x7FFFFFFFll) {
    LnModPair g;
    for (int i = 0; i < 2; ++i) {
      g.x[i] = probs[i].x;
      g.shift[i] = probs[i].shift;
      g.scale[i] = probs[i].scale;
      g.out[i] = probs[i].out;
      g.mod_bstride[i] = probs[i].mod_batch_stride;
      g.rows_per_batch[i] = probs[i].rows_per_batch;
    }
    g.rows0 = probs[0].rows;
    ln_mod_pair_kernel<128, 6><<<static_cast<unsigned>(probs[0].rows + probs[1].rows), 128, 0, st>>>(g);
    return cudaGetLastError();
  }
  for (int i = 0; i < count; ++i) {
    const fb_ln_mod_problem& p = probs[i];
    const cudaError_t e = launch_ln_mod(p.x, p.rows, p.dim, p.rows_per_batch, p.shift, p.scale, p.mod_batch_stride,
                                        p.out, st);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// ============================================================================================ gated add

// out = x + g[b, col] * y  (flux.py:169-171), y clamped to the fp16 range first when guarding
// (flux.py:141-143). Four columns per thread step; dim % 4 == 0.
__global__ void __launch_bounds__(256) gated_add_kernel(const float* __restrict__ x, const uint16_t* __restrict__ g,
                                                        const uint16_t* __restrict__ y, float* __restrict__ out,
                                                        int64_t n4, int dim4, int rows_per_batch, int64_t g_bstride,
                                                        int guard) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
    const int64_t row = i / dim4;
    const int col = static_cast<int>(i - row * dim4) * 4;
    const int64_t b = row / rows_per_batch;
    const float4 xv = reinterpret_cast<const float4*>(x)[i];
    float gv[4], yv[4];
    ld_bf16x4(g + b * g_bstride + col, gv);
    ld_bf16x4(y + 4 * i, yv);
    if (guard) {
#pragma unroll
      for (int j = 0; j < 4; ++j) yv[j] = fminf(fmaxf(yv[j], -65504.0f), 65504.0f);
    }
    float4 o;
    o.x = __fadd_rn(xv.x, __fmul_rn(gv[0], yv[0]));
    o.y = __fadd_rn(xv.y, __fmul_rn(gv[1], yv[1]));
    o.z = __fadd_rn(xv.z, __fmul_rn(gv[2], yv[2]));
    o.w = __fadd_rn(xv.w, __fmul_rn(gv[3], yv[3]));
    reinterpret_cast<float4*>(out)[i] = o;
  }
}

cudaError_t launch_gated_add(const float* x, const uint16_t* g, const uint16_t* y, float* out, int64_t rows, int dim,
                             int rows_per_batch, int64_t g_bstride, int guard, cudaStream_t st) {
  const int64_t n4 = rows * dim / 4;
  if (n4 == 0) return cudaSuccess;
  const int grid = static_cast<int>(std::min<int64_t>((n4 + 255) / 256, kNumSms * 8));
  gated_add_kernel<<<grid, 256, 0, st>>>(x, g, y, out, n4, dim / 4, rows_per_batch, g_bstride, guard);
  return cudaGetLastError();
}

// ============================================================================================ GELU

// out = bf16(gelu_tanh(f32(h))) (flux.py:194-195); eight bf16 per thread step.
__global__ void __launch_bounds__(256) gelu_kernel(const uint16_t* __restrict__ h, uint16_t* __restrict__ out,
                                                   int64_t n8) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8; i += stride) {
    const uint4 u = reinterpret_cast<const uint4*>(h)[i];
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float lo = __uint_as_float(w[j] << 16), hi = __uint_as_float(w[j] & 0xFFFF0000u);
      o[j] = pack_bf16x2(gelu_tanh_f32(lo), gelu_tanh_f32(hi));
    }
    reinterpret_cast<uint4*>(out)[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

cudaError_t launch_gelu(const uint16_t* h, uint16_t* out, int64_t n, cudaStream_t st) {
  const int64_t n8 = n / 8;
  if (n8 == 0) return cudaSuccess;
  const int grid = static_cast<int>(std::min<int64_t>((n8 + 255) / 256, kNumSms * 8));
  gelu_kernel<<<grid, 256, 0, st>>>(h, out, n8);
  return cudaGetLastError();
}

// ============================================================================================ QK norm + RoPE

// One warp per (image, row, head): lane holds EPL = head_dim / 32 consecutive dims (an even count,
// so RoPE pairs (2i, 2i+1) stay inside a lane). q/k: RMSNorm over head_dim (eps 1e-6, fp32 scale),
// then the interleaved rotation by cos/sin of the row's global position, then bf16 (flux.py:117-126,
// :179-191). v is copied. Output layout [batch, heads, seq_total, head_dim].
template <int EPL>
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(const uint16_t* __restrict__ qkv, int64_t ld_qkv, int batch,
                                                           int rows, int heads, const float* __restrict__ q_scale,
                                                           const float* __restrict__ k_scale,
                                                           const float* __restrict__ rcos,
                                                           const float* __restrict__ rsin, uint16_t* __restrict__ q,
                                                           uint16_t* __restrict__ k, uint16_t* __restrict__ v,
                                                           int seq_total, int seq_offset) {
  constexpr int HD = 32 * EPL;
  const int lane = threadIdx.x & 31;
  const int64_t item = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int64_t total = static_cast<int64_t>(batch) * rows * heads;
  if (item >= total) return;
  const int h = static_cast<int>(item % heads);
  const int64_t br = item / heads;  // b * rows + r
  const int r = static_cast<int>(br % rows);
  const int b = static_cast<int>(br / rows);
  const int pos = seq_offset + r;
  const int d0 = lane * EPL;
  const uint16_t* src = qkv + br * ld_qkv + h * HD + d0;
  const int64_t dst = ((static_cast<int64_t>(b) * heads + h) * seq_total + pos) * HD + d0;
  for (int part = 0; part < 3; ++part) {
    const uint16_t* s = src + static_cast<int64_t>(part) * heads * HD;
    float f[EPL];
#pragma unroll
    for (int j = 0; j < EPL; ++j) f[j] = bf16_bits_to_f32(s[j]);
    uint16_t* o = (part == 0 ? q : part == 1 ? k : v) + dst;
    if (part < 2) {
      const float* sc = (part == 0 ? q_scale : k_scale) + d0;
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < EPL; ++j) ss += f[j] * f[j];
      const float rr = rsqrtf(warp_sum(ss) / static_cast<float>(HD) + 1e-6f);
#pragma unroll
      for (int j = 0; j < EPL; ++j) f[j] = __fmul_rn(__fmul_rn(f[j], rr), sc[j]);
#pragma unroll
      for (int j = 0; j < EPL; j += 2) {
        const float c = rcos[static_cast<int64_t>(pos) * (HD / 2) + (d0 + j) / 2];
        const float sn = rsin[static_cast<int64_t>(pos) * (HD / 2) + (d0 + j) / 2];
        const float e = f[j], od = f[j + 1];
        f[j] = __fsub_rn(__fmul_rn(e, c), __fmul_rn(od, sn));
        f[j + 1] = __fadd_rn(__fmul_rn(e, sn), __fmul_rn(od, c));
      }
    }
#pragma unroll
    for (int j = 0; j < EPL; j += 2) *reinterpret_cast<uint32_t*>(o + j) = pack_bf16x2(f[j], f[j + 1]);
  }
}

cudaError_t launch_qk_norm_rope(const uint16_t* qkv, int64_t ld_qkv, int batch, int rows, int heads, int head_dim,
                                const float* q_scale, const float* k_scale, const float* rcos, const float* rsin,
                                uint16_t* q, uint16_t* k, uint16_t* v, int seq_total, int seq_offset,
                                cudaStream_t st) {
  const int64_t items = static_cast<int64_t>(batch) * rows * heads;
  if (items == 0) return cudaSuccess;
  const unsigned grid = static_cast<unsigned>((items + 7) / 8);
  if (head_dim == 128) {
    qk_norm_rope_kernel<4><<<grid, 256, 0, st>>>(qkv, ld_qkv, batch, rows, heads, q_scale, k_scale, rcos, rsin, q, k, v,
                                                 seq_total, seq_offset);
  } else {
    qk_norm_rope_kernel<2><<<grid, 256, 0, st>>>(qkv, ld_qkv, batch, rows, heads, q_scale, k_scale, rcos, rsin, q, k, v,
                                                 seq_total, seq_offset);
  }
  return cudaGetLastError();
}

}  // namespace fb
