// gemm_nf4.cu — tcgen05 GEMM whose weight operand is NF4: the packed 4-bit weight and its fp32 absmax
// stream from HBM and are decoded inside the mainloop, tile by tile, into the UMMA shared-memory layout.
// The bf16 weight never exists in global memory.
//
//   y[m, n] = sum_k A[m, k] * W[n, k] (+ bias[n]),   W[n, 2i] = bf16(code[p >> 4] * absmax),
//                                                    W[n, 2i+1] = bf16(code[p & 15] * absmax)
//   (p = packed byte (n * K + 2i) / 2, absmax = absmax[(n * K + 2i) / 64]; one fp32 multiply, then a
//   round-to-nearest-even cast: the decoded tile is bit-identical to fb_nf4_dequant's output and to
//   selas/codecs.py:178-199.)
//
// CTA tile 256 x 128: two M=128 MMAs per K step share one decoded W tile, so decoding costs half as
// much per FLOP as it would with a 128-row tile. 320 threads:
//   warp 0      TMA: two 128x64 bf16 A boxes and one 128-row x 32-byte packed W box per stage
//   warp 1      TMEM allocator + MMA issuer (M=128, N=128, K=16, twice per K step)
//   warps 2..5  epilogue (the fused FLUX epilogues of gemm_common.cuh), one output row per thread
//   warps 6..9  NF4 converters, one per SM sub-partition: each thread decodes one W row per stage
//               through the 16-entry fp32 code table in shared memory (one bank per entry, so the
//               lookups of a warp never conflict), multiplies pairs by absmax with packed FP32x2
//               multiplies and writes the row in the 128-byte swizzled K-major layout; the fp32 absmax
//               of the next stage is prefetched
// Accumulators: 2 (double buffer) x 2 (M halves) x 128 columns = all 512 TMEM columns.
// Requirements (checked on the host): K % 256 == 0 (whole float4 groups of absmax per row), blocksize
// 64, 16-byte aligned absmax.
#include "gemm_common.cuh"

namespace fb {
namespace gemm_nf4 {

using namespace gemm;

constexpr int BM = 256;
constexpr int BN = 128;
constexpr int kThreads = 320;
constexpr int kConvThreads = 128;
constexpr int kStages = 4;
constexpr int kABytes = 2 * 128 * BK * 2;   // 32 KB
constexpr int kBBytes = BN * BK * 2;        // 16 KB, decoded
constexpr int kPBytes = BN * BK / 2;        // 4 KB, packed
constexpr int kLutBytes = 2 * 16 * 4;       // one 16-entry fp32 code table per problem
constexpr int kSmemBytes = kStages * (kABytes + kBBytes + kPBytes) + kLutBytes + 256 + 1024;
constexpr uint32_t kIdesc = idesc_bf16_f32(128, BN, false);
constexpr uint32_t kTmemCols = 512;

__device__ __forceinline__ uint64_t mul_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1) gemm_nf4_kernel(const __grid_constant__ Args args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;                                   // kStages x 32 KB
  uint8_t* sB = sA + kStages * kABytes;                 // kStages x 16 KB
  uint8_t* sPk = sB + kStages * kBBytes;                // kStages x 4 KB
  float* code_s = reinterpret_cast<float*>(sPk + kStages * kPBytes);  // [2][16]
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(code_s) + kLutBytes);
  uint64_t* b_ready = full + kStages;
  uint64_t* empty = b_ready + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&b_ready[s], kConvThreads / 32);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp >= 6) {
    // each problem's runtime code table (problem 0 in banks 0-15, problem 1 in banks 16-31)
    const int ct = threadIdx.x - 192;
    if (ct < 16 * args.nprob) code_s[ct] = __ldg(args.prob[ct >> 4].code16 + (ct & 15));
  }
  if (warp == 0 && lane == 0) {
    for (int p = 0; p < args.nprob; ++p) {
      tma_prefetch_desc(&args.prob[p].tma_a);
      tma_prefetch_desc(&args.prob[p].tma_b);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_parity[kStages];
      for (int s = 0; s < kStages; ++s) issued_parity[s] = 0xFFFFFFFFu;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < args.total_tiles; tile += gridDim.x) {
        int p, mb, nb;
        decode_tile(args, tile, p, mb, nb);
        const Problem& P = args.prob[p];
        for (int kb = 0; kb < P.num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, args.status, FB_DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], kABytes + kPBytes);
          uint8_t* a = sA + stage * kABytes;
          tma_load_2d(&P.tma_a, &full[stage], a, kb * BK, mb * BM);
          tma_load_2d(&P.tma_a, &full[stage], a + kABytes / 2, kb * BK, mb * BM + 128);
          tma_load_2d(&P.tma_b, &full[stage], sPk + stage * kPBytes, kb * (BK / 2), nb * BN);
          issued_parity[stage] = phase;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        for (int s = 0; s < kStages; ++s)
          if (issued_parity[s] != 0xFFFFFFFFu) mbar_wait_quiet(&full[s], issued_parity[s], kWaitBudgetNs);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < args.total_tiles; tile += gridDim.x) {
        int p, mb, nb;
        decode_tile(args, tile, p, mb, nb);
        const Problem& P = args.prob[p];
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, abort_flag, args.status, FB_DEV_TIMEOUT_EPI)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        const uint32_t d0 = tmem_base + static_cast<uint32_t>(acc * 2 * BN);
        const uint32_t d1 = d0 + BN;
        for (int kb = 0; kb < P.num_kb; ++kb) {
          ok = mbar_wait(&full[stage], phase, abort_flag, args.status, FB_DEV_TIMEOUT_TMA) &&
               mbar_wait(&b_ready[stage], phase, abort_flag, args.status, FB_DEV_TIMEOUT_EPI);
          if (!ok) break;
          tc_fence_after_sync();
          const uint32_t a0 = smem_u32(sA + stage * kABytes);
          const uint32_t a1 = a0 + kABytes / 2;
          const uint32_t b0 = smem_u32(sB + stage * kBBytes);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t bd = sdesc_kmajor_sw128(b0 + 32 * k);
            const uint32_t accum = (kb > 0 || k > 0) ? 1u : 0u;
            umma_bf16_ss(d0, sdesc_kmajor_sw128(a0 + 32 * k), bd, kIdesc, accum);
            umma_bf16_ss(d1, sdesc_kmajor_sw128(a1 + 32 * k), bd, kIdesc, accum);
          }
          umma_commit(&empty[stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&acc_full[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      umma_commit(drain);
      mbar_wait_quiet(drain, 0, kWaitBudgetNs);
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------------ epilogue (warps 2..5)
    const int quarter = warp & 3;
    const int row_in_half = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < args.total_tiles; tile += gridDim.x) {
      int p, mb, nb;
      decode_tile(args, tile, p, mb, nb);
      const Problem& P = args.prob[p];
      if (!mbar_wait(&acc_full[acc], acc_phase, abort_flag, args.status, FB_DEV_TIMEOUT_MMA)) break;
      tc_fence_after_sync();
#pragma unroll 1
      for (int hf = 0; hf < 2; ++hf) {
        const uint32_t trow = tmem_base + lane_base + static_cast<uint32_t>(acc * 2 * BN + hf * BN);
        const int m = mb * BM + hf * 128 + row_in_half;
        epilogue_row<BN, EPI, true>(P, m, m < P.m, nb, trow);
      }
      tc_fence_before_sync();
      mbar_arrive(&acc_empty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  } else {
    // ------------------------------------------------------------------ NF4 converters (warps 6..9)
    const int r = threadIdx.x - 192;  // 0..127: the W row of the tile this thread decodes
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < args.total_tiles; tile += gridDim.x) {
      int p, mb, nb;
      decode_tile(args, tile, p, mb, nb);
      const Problem& P = args.prob[p];
      const float* cs = code_s + p * 16;
      const int n = nb * BN + r;
      const bool valid = n < P.n;
      // absmax arrives four K steps at a time (one float4 per row), with the next group in flight
      const float4* am4 = reinterpret_cast<const float4*>(P.absmax + static_cast<int64_t>(n) * P.absmax_per_row);
      const float4 zero4 = make_float4(0.f, 0.f, 0.f, 0.f);
      float4 cur = valid ? __ldg(am4) : zero4;
      float4 nxt = (valid && P.num_kb > 4) ? __ldg(am4 + 1) : zero4;
      for (int kb = 0; kb < P.num_kb; ++kb) {
        if (kb > 0 && (kb & 3) == 0) {
          cur = nxt;
          nxt = (valid && kb + 4 < P.num_kb) ? __ldg(am4 + (kb >> 2) + 1) : zero4;
        }
        const int q = kb & 3;
        const float s_cur = q == 0 ? cur.x : q == 1 ? cur.y : q == 2 ? cur.z : cur.w;
        if (!mbar_wait(&full[stage], phase, abort_flag, args.status, FB_DEV_TIMEOUT_TMA)) {
          ok = false;
          break;
        }
        const uint8_t* pk = sPk + stage * kPBytes + r * 32;
        uint8_t* rowp = sB + stage * kBBytes + r * 128;
        const uint4 w0 = *reinterpret_cast<const uint4*>(pk);
        const uint4 w1 = *reinterpret_cast<const uint4*>(pk + 16);
        const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        const uint64_t a2 = (static_cast<uint64_t>(__float_as_uint(s_cur)) << 32) | __float_as_uint(s_cur);
#pragma unroll
        for (int g = 0; g < 8; ++g) {  // 16-byte chunk g = elements 8g .. 8g+7 = packed bytes 4g .. 4g+3
          uint32_t o[4];
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            const float hi = cs[(words[g] >> (8 * b + 4)) & 15u];  // even element: high nibble
            const float lo = cs[(words[g] >> (8 * b)) & 15u];
            const uint64_t v = mul_f32x2((static_cast<uint64_t>(__float_as_uint(lo)) << 32) | __float_as_uint(hi), a2);
            o[b] = pack_bf16x2(__uint_as_float(static_cast<uint32_t>(v)), __uint_as_float(static_cast<uint32_t>(v >> 32)));
          }
          *reinterpret_cast<uint4*>(rowp + ((g ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&b_ready[stage]);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace gemm_nf4

std::string gemm_nf4_setup() {
  using namespace gemm_nf4;
  cudaError_t e = cudaSuccess;
  e = e ? e : cudaFuncSetAttribute(gemm_nf4_kernel<FB_EPI_STORE_BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  e = e ? e : cudaFuncSetAttribute(gemm_nf4_kernel<FB_EPI_STORE_F32>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  e = e ? e : cudaFuncSetAttribute(gemm_nf4_kernel<FB_EPI_GELU>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  e = e ? e : cudaFuncSetAttribute(gemm_nf4_kernel<FB_EPI_GATED_RESIDUAL>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  e = e ? e : cudaFuncSetAttribute(gemm_nf4_kernel<FB_EPI_QKV>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  return e == cudaSuccess ? std::string() : std::string("cudaFuncSetAttribute(gemm_nf4): ") + cudaGetErrorString(e);
}

cudaError_t launch_gemm_nf4(int epi, const gemm::Args& args, int grid, cudaStream_t st) {
  using namespace gemm_nf4;
  switch (epi) {
    case FB_EPI_STORE_BF16: gemm_nf4_kernel<FB_EPI_STORE_BF16><<<grid, kThreads, kSmemBytes, st>>>(args); break;
    case FB_EPI_STORE_F32: gemm_nf4_kernel<FB_EPI_STORE_F32><<<grid, kThreads, kSmemBytes, st>>>(args); break;
    case FB_EPI_GELU: gemm_nf4_kernel<FB_EPI_GELU><<<grid, kThreads, kSmemBytes, st>>>(args); break;
    case FB_EPI_GATED_RESIDUAL: gemm_nf4_kernel<FB_EPI_GATED_RESIDUAL><<<grid, kThreads, kSmemBytes, st>>>(args); break;
    default: gemm_nf4_kernel<FB_EPI_QKV><<<grid, kThreads, kSmemBytes, st>>>(args); break;
  }
  return cudaGetLastError();
}

}  // namespace fb
