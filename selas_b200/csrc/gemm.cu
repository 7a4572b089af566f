// gemm.cu — persistent, warp-specialised tcgen05 GEMM for the FLUX block Linears, with the
// memory-bound glue fused into the epilogue.
//
//   y[m, n] = sum_k A[m, k] * W[n, k]  (+ bias[n])      A bf16 [M, K], W bf16 [N, K] (nn.Linear)
//
// Layout of one CTA (192 threads, one CTA per SM):
//   warp 0      TMA producer: A tile 128x64 and W tile BNx64 per stage (128-byte swizzle), STAGES deep
//   warp 1      TMEM allocator + MMA issuer: one thread issues tcgen05.mma M=128 N=BN K=16
//   warps 2..5  epilogue: tcgen05.ld of the accumulator (thread = one row), fused epilogue, stores
// The accumulator is double-buffered in TMEM (2 x BN fp32 columns), so the epilogue of tile i
// overlaps the mainloop of tile i+1. Tiles are scheduled persistently (tile += gridDim.x) over up to
// two problems (the txt and img streams of a double block share one launch). Every output element
// is produced by exactly one CTA with a fixed K order, so results are run-to-run deterministic.
//
// Epilogues (the rounding mirrors the eager reference: F.linear rounds acc + bias to bf16 first):
//   STORE_BF16      out = bf16(acc + b)
//   STORE_F32       out = f32(bf16(acc + b))
//   GELU            out = bf16(gelu_tanh(bf16(acc + b)))
//   GATED_RESIDUAL  out = resid + gate[img] * f32(bf16(acc + b))            (fp32 residual stream)
//   QKV             per 128-column head group: q/k -> RMSNorm * scale -> RoPE -> bf16 into
//                   [B, H, L, 128]; v -> bf16 copy; columns >= qkv_cols -> GELU into `out`.
#include "gemm_common.cuh"

namespace fb {

namespace gemm {

constexpr int BM = 128;
constexpr int kThreads = 192;
constexpr int kEpiThreads = 128;

template <int BN>
struct Cfg {
  static constexpr int kStages = BN == 256 ? 4 : (BN == 128 ? 6 : 8);
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = BN * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN;  // two accumulators
  static constexpr int kBarrierBytes = 256;
  static constexpr int kSmemBytes = kStages * kStageBytes + kBarrierBytes + 1024;  // +1024: alignment slack
  static constexpr uint32_t kIdesc = idesc_bf16_f32(BM, BN, false);
};

template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ Args args) {
  using C = Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::kStages * C::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + C::kStages * C::kBBytes);
  uint64_t* empty = full + C::kStages;
  uint64_t* acc_full = empty + C::kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], kEpiThreads);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    for (int p = 0; p < args.nprob; ++p) {
      tma_prefetch_desc(&args.prob[p].tma_a);
      tma_prefetch_desc(&args.prob[p].tma_b);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
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
      int issued_stage = -1;
      uint32_t issued_parity[C::kStages];
      for (int s = 0; s < C::kStages; ++s) issued_parity[s] = 0xFFFFFFFFu;
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
          mbar_arrive_expect_tx(&full[stage], C::kStageBytes);
          tma_load_2d(&P.tma_a, &full[stage], sA + stage * C::kABytes, kb * BK, mb * BM);
          tma_load_2d(&P.tma_b, &full[stage], sB + stage * C::kBBytes, kb * BK, nb * BN);
          issued_parity[stage] = phase;
          issued_stage = stage;
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && issued_stage >= 0) {
        // Let the copies already in flight land before the CTA exits (bounded).
        for (int s = 0; s < C::kStages; ++s)
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
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < P.num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, args.status, FB_DEV_TIMEOUT_TMA)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t a0 = smem_u32(sA + stage * C::kABytes);
          const uint32_t b0 = smem_u32(sB + stage * C::kBBytes);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            umma_bf16_ss(d_tmem, sdesc_kmajor_sw128(a0 + 32 * k), sdesc_kmajor_sw128(b0 + 32 * k), C::kIdesc,
                         (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&acc_full[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      // Wait (bounded) for every MMA issued by this thread before TMEM is released.
      umma_commit(drain);
      mbar_wait_quiet(drain, 0, kWaitBudgetNs);
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..5)
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_tile = quarter * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < args.total_tiles; tile += gridDim.x) {
      int p, mb, nb;
      decode_tile(args, tile, p, mb, nb);
      const Problem& P = args.prob[p];
      if (!mbar_wait(&acc_full[acc], acc_phase, abort_flag, args.status, FB_DEV_TIMEOUT_MMA)) break;
      tc_fence_after_sync();
      const uint32_t trow = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
      const int m = mb * BM + row_in_tile;
      const bool row_ok = m < P.m;
      epilogue_row<BN, EPI>(P, m, row_ok, nb, trow);
      tc_fence_before_sync();
      mbar_arrive(&acc_empty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

}  // namespace gemm

// ============================================================================================ host

static int encode_kmajor_bf16(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld,
                              int box_rows, std::string& err) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) {
    err = "cuTensorMapEncodeTiled unavailable (fb_init not run?)";
    return FB_ERR_INIT;
  }
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(gemm::BK), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    err = "cuTensorMapEncodeTiled failed (" + std::to_string(static_cast<int>(r)) + ")";
    return FB_ERR_CUDA;
  }
  return FB_OK;
}

// fp32 rows [rows, cols] with row stride ld elements, read in 32-column x 32-row boxes (128-byte rows,
// 128-byte swizzle); rows and columns past the end read as zeros.
static int encode_f32_rows(CUtensorMap* map, const float* base, int64_t rows, int64_t cols, int64_t ld,
                           std::string& err) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) {
    err = "cuTensorMapEncodeTiled unavailable (fb_init not run?)";
    return FB_ERR_INIT;
  }
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 4};
  const cuuint32_t box[2] = {32, 32};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    err = "cuTensorMapEncodeTiled(resid) failed (" + std::to_string(static_cast<int>(r)) + ")";
    return FB_ERR_CUDA;
  }
  return FB_OK;
}

// A RoPE table, fp32 [seq, 64], read in 16-column x 32-row boxes (64-byte rows, 64-byte swizzle); rows
// past the end read as zeros.
static int encode_rope_table(CUtensorMap* map, const float* base, int64_t seq, std::string& err) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) {
    err = "cuTensorMapEncodeTiled unavailable (fb_init not run?)";
    return FB_ERR_INIT;
  }
  const cuuint64_t dims[2] = {64, static_cast<cuuint64_t>(seq)};
  const cuuint64_t strides[1] = {64 * 4};
  const cuuint32_t box[2] = {16, 32};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    err = "cuTensorMapEncodeTiled(rope) failed (" + std::to_string(static_cast<int>(r)) + ")";
    return FB_ERR_CUDA;
  }
  return FB_OK;
}

template <int BN, int EPI>
static cudaError_t launch_cfg(const gemm::Args& args, int grid, cudaStream_t st) {
  gemm::gemm_kernel<BN, EPI><<<grid, gemm::kThreads, gemm::Cfg<BN>::kSmemBytes, st>>>(args);
  return cudaGetLastError();
}

template <int BN>
static cudaError_t dispatch_epi(int epi, const gemm::Args& args, int grid, cudaStream_t st) {
  switch (epi) {
    case FB_EPI_STORE_BF16: return launch_cfg<BN, FB_EPI_STORE_BF16>(args, grid, st);
    case FB_EPI_STORE_F32: return launch_cfg<BN, FB_EPI_STORE_F32>(args, grid, st);
    case FB_EPI_GELU: return launch_cfg<BN, FB_EPI_GELU>(args, grid, st);
    case FB_EPI_GATED_RESIDUAL: return launch_cfg<BN, FB_EPI_GATED_RESIDUAL>(args, grid, st);
    default: return launch_cfg<BN, FB_EPI_QKV>(args, grid, st);
  }
}

template <int BN>
static std::string setup_bn() {
  const int smem = gemm::Cfg<BN>::kSmemBytes;
  cudaError_t e = cudaSuccess;
  e = e ? e : cudaFuncSetAttribute(gemm::gemm_kernel<BN, FB_EPI_STORE_BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  e = e ? e : cudaFuncSetAttribute(gemm::gemm_kernel<BN, FB_EPI_STORE_F32>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  e = e ? e : cudaFuncSetAttribute(gemm::gemm_kernel<BN, FB_EPI_GELU>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  e = e ? e : cudaFuncSetAttribute(gemm::gemm_kernel<BN, FB_EPI_GATED_RESIDUAL>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  e = e ? e : cudaFuncSetAttribute(gemm::gemm_kernel<BN, FB_EPI_QKV>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  return e == cudaSuccess ? std::string() : std::string("cudaFuncSetAttribute(gemm): ") + cudaGetErrorString(e);
}

std::string gemm_setup() {
  std::string s = setup_bn<256>();
  if (s.empty()) s = gemm_nf4_setup();
  if (s.empty()) s = gemm_pair_setup();
  if (s.empty()) s = setup_bn<64>();
  return s;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Packed NF4 weight [n rows, k/2 bytes] as a 2-D uint8 map, 128-row x 32-byte boxes (one K step of 64).
static int encode_packed_nf4(CUtensorMap* map, const uint8_t* base, int64_t rows, int64_t k, std::string& err) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) {
    err = "cuTensorMapEncodeTiled unavailable (fb_init not run?)";
    return FB_ERR_INIT;
  }
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(k / 2), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(k / 2)};
  const cuuint32_t box[2] = {32, 128};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    err = "cuTensorMapEncodeTiled(nf4) failed (" + std::to_string(static_cast<int>(r)) + ")";
    return FB_ERR_CUDA;
  }
  return FB_OK;
}

// One-byte-per-weight rows (int8_row q, fp8) [rows, k] as a UINT8 map with the 64-byte swizzle: box =
// one K step (64 bytes) of 128 rows; 16-byte chunk c of row r lands at position c ^ ((r >> 1) & 3)
// (bank-conflict-free reads by the converters).
static int encode_byte_rows(CUtensorMap* map, const void* base, int64_t rows, int64_t k, std::string& err) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) {
    err = "cuTensorMapEncodeTiled unavailable (fb_init not run?)";
    return FB_ERR_INIT;
  }
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(k)};
  const cuuint32_t box[2] = {64, 128};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    err = "cuTensorMapEncodeTiled(byte rows) failed (" + std::to_string(static_cast<int>(r)) + ")";
    return FB_ERR_CUDA;
  }
  return FB_OK;
}

int launch_linear_grouped(const fb_linear* probs, int count, int epi, cudaStream_t st, std::string& err) {
  std::string derr;
  DeviceState* dev = current_device(derr);
  if (!dev) {
    err = derr;
    return FB_ERR_INIT;
  }
  return launch_linear_on(probs, count, epi, nullptr, dev->status, dev->sm_count, st, err, dev);
}

int launch_linear_on(const fb_linear* probs, int count, int epi, const int* n_offsets, int* status, int sm_count,
                     cudaStream_t st, std::string& err, const DeviceState* splitk) {
  if (count < 1 || count > 2) {
    err = "fb_linear_grouped: count must be 1 or 2";
    return FB_ERR_ARG;
  }
  if (epi < FB_EPI_STORE_BF16 || epi > FB_EPI_QKV) {
    err = "fb_linear_grouped: unknown epilogue";
    return FB_ERR_ARG;
  }
  // bf16 weights: 128 x BN tiles, BN = 64 for narrow outputs (final layer N=64), else 256.
  // NF4, int8_row or fp8 weights (all problems of the call alike): the fused decode kernel's pair tiles
  // of 256 tokens x 256 W rows (gemm_nf4.cu), each CTA loading 128 tokens of activations.
  auto wfmt_of = [](const fb_linear& L) { return L.w_nf4 ? 1 : L.w_i8 ? 2 : L.w_f8 ? 3 : 0; };
  const int wfmt = wfmt_of(probs[0]);
  const bool nf4 = wfmt == 1, decode = wfmt != 0;
  int max_n = 0;
  for (int i = 0; i < count; ++i) max_n = std::max(max_n, probs[i].n);
  const int BN = decode ? 256 : ((max_n <= 64 && epi != FB_EPI_QKV) ? 64 : 256);
  // bf16 with 256-wide tiles runs on CTA pairs (256 x 256 per pair) unless FLUX_B200_GEMM=single.
  const bool pair = !decode && BN == 256 && gemm_pair_enabled();
  const int BM = (decode || pair) ? 256 : gemm::BM;
  const int a_box_rows = gemm::BM;          // activation rows one CTA loads per tile (128)
  const int b_box_rows = pair ? 128 : BN;      // W rows one CTA loads per tile (bf16)

  gemm::Args args;
  memset(&args, 0, sizeof(args));
  args.nprob = 0;
  int tiles = 0;
  for (int i = 0; i < count; ++i) {
    const fb_linear& L = probs[i];
    const int n_off = n_offsets ? n_offsets[i] : 0;
    if (L.m < 0 || L.n <= 0 || L.k <= 0 || n_off < 0) {
      err = "fb_linear_grouped: bad shape";
      return FB_ERR_ARG;
    }
    if ((L.w != nullptr) + (L.w_nf4 != nullptr) + (L.w_i8 != nullptr) + (L.w_f8 != nullptr) != 1 ||
        wfmt_of(L) != wfmt) {
      err = "fb_linear_grouped: each problem sets exactly one of w / w_nf4 / w_i8 / w_f8, the same kind for every "
            "problem of the call";
      return FB_ERR_ARG;
    }
    if (wfmt == 3 && (L.k % 64 != 0 || (L.w_f8_e5m2 != 0 && L.w_f8_e5m2 != 1))) {
      err = "fb_linear_grouped: fp8 weights need k % 64 == 0 and w_f8_e5m2 0 (e4m3fn) or 1 (e5m2)";
      return FB_ERR_UNSUPPORTED;
    }
    if (wfmt == 2 && (L.k % 64 != 0 || !L.w_scale || (reinterpret_cast<uintptr_t>(L.w_scale) & 3u))) {
      err = "fb_linear_grouped: int8_row weights need k % 64 == 0 and a 4-byte aligned w_scale";
      return FB_ERR_UNSUPPORTED;
    }
    if (nf4 && (L.k % 256 != 0 || L.blocksize != 64 || !L.absmax || !L.code16 || !aligned16(L.absmax) ||
                (reinterpret_cast<uintptr_t>(L.code16) & 3u))) {
      err = "fb_linear_grouped: NF4 weights need k % 256 == 0, blocksize 64, 16-byte aligned absmax and a "
            "4-byte aligned code16 (fb_linear_nf4 decodes other layouts through a workspace)";
      return FB_ERR_UNSUPPORTED;
    }
    if (L.n % 32 != 0 || L.k % 8 != 0 || L.lda % 8 != 0 || (!decode && (L.ldw % 8 != 0 || L.ldw < L.k)) || L.lda < L.k) {
      err = "fb_linear_grouped: need n % 32 == 0, k % 8 == 0, lda/ldw multiples of 8 and >= k";
      return FB_ERR_ALIGN;
    }
    const void* wptr = nf4         ? static_cast<const void*>(L.w_nf4)
                       : wfmt == 2 ? static_cast<const void*>(L.w_i8)
                       : wfmt == 3 ? static_cast<const void*>(L.w_f8)
                                   : static_cast<const void*>(L.w);
    if (!aligned16(L.a) || !aligned16(wptr) ||
        (L.bias && !aligned16(L.bias))) {
      err = "fb_linear_grouped: a, the weight and bias must be 16-byte aligned";
      return FB_ERR_ALIGN;
    }
    if (L.rows_per_batch <= 0) {
      err = "fb_linear_grouped: rows_per_batch must be > 0";
      return FB_ERR_ARG;
    }
    if (epi != FB_EPI_QKV || n_off + L.n > L.qkv_cols) {
      if (!L.out || !aligned16(L.out) || L.ld_out % 8 != 0) {
        err = "fb_linear_grouped: out must be 16-byte aligned with ld_out % 8 == 0";
        return FB_ERR_ALIGN;
      }
    }
    if (epi == FB_EPI_GATED_RESIDUAL) {
      if (!L.resid || !L.gate || !aligned16(L.resid) || !aligned16(L.gate) || L.ld_resid % 4 != 0 ||
          L.gate_batch_stride % 8 != 0) {
        err = "fb_linear_grouped: gated residual needs 16-byte aligned resid/gate, ld_resid % 4, gate stride % 8";
        return FB_ERR_ALIGN;
      }
    }
    if (epi == FB_EPI_QKV && L.sp_world != 0) {
      bool bad = L.sp_world < 1 || L.sp_world > 8 || L.sp_rank < 0 || L.sp_rank >= L.sp_world ||
                 L.heads % L.sp_world != 0 || L.rows_per_batch < L.m;
      for (int g = 0; !bad && g < L.sp_world; ++g) bad = !L.sp_qkv_dst[g] || !aligned16(L.sp_qkv_dst[g]);
      if (bad) {
        err = "fb_linear_grouped: sequence-parallel QKV needs 1 <= sp_world <= 8 dividing heads, 0 <= sp_rank < "
              "sp_world, one image (rows_per_batch >= m) and sp_world 16-byte aligned destinations";
        return FB_ERR_ARG;
      }
    }
    if (epi == FB_EPI_QKV) {
      const bool sp = L.sp_world != 0;
      if (L.head_dim != 128 || L.heads <= 0 || L.qkv_cols != 3 * L.heads * 128 || L.qkv_cols % 128 != 0 ||
          (!sp && (!L.q || !L.k_out || !L.v)) || !L.q_scale || !L.k_scale || !L.rope_cos || !L.rope_sin ||
          L.seq_offset < 0 || L.seq_offset + L.rows_per_batch > L.seq_total ||
          (n_offsets == nullptr && ((L.n - L.qkv_cols) % 128 != 0 || L.n < L.qkv_cols)) ||
          (n_offsets != nullptr && (L.n % 128 != 0 || n_off % 128 != 0))) {
        err = "fb_linear_grouped: QKV epilogue needs head_dim 128, qkv_cols = 3*heads*128, all q/k/v/scale/rope "
              "pointers, and seq_offset + rows_per_batch <= seq_total";
        return FB_ERR_UNSUPPORTED;
      }
      if ((!sp && (!aligned16(L.q) || !aligned16(L.k_out) || !aligned16(L.v))) || !aligned16(L.q_scale) ||
          !aligned16(L.k_scale) || !aligned16(L.rope_cos) || !aligned16(L.rope_sin)) {
        err = "fb_linear_grouped: q/k/v, the norm scales and the RoPE tables must be 16-byte aligned";
        return FB_ERR_ALIGN;
      }
      if (n_off + L.n > L.qkv_cols && (L.gelu_col0 < 0 || L.gelu_col0 % 8 != 0)) {
        err = "fb_linear_grouped: gelu_col0 must be >= 0 and a multiple of 8 (16-byte aligned GELU columns)";
        return FB_ERR_ALIGN;
      }
    }
    gemm::Problem& P = args.prob[i];
    int rc = encode_kmajor_bf16(&P.tma_a, L.a, std::max(L.m, 1), L.k, L.lda, a_box_rows, err);
    if (rc) return rc;
    rc = nf4 ? encode_packed_nf4(&P.tma_b, L.w_nf4, L.n, L.k, err)
             : wfmt >= 2 ? encode_byte_rows(&P.tma_b, wptr, L.n, L.k, err)
                         : encode_kmajor_bf16(&P.tma_b, L.w, L.n, L.k, L.ldw, b_box_rows, err);
    if (rc) return rc;
    if ((pair || (decode && nf4)) && epi == FB_EPI_GATED_RESIDUAL && L.m > 0) {
      rc = encode_f32_rows(&P.tma_resid, L.resid, L.m, L.n, L.ld_resid, err);
      if (rc) return rc;
    }
    if (pair && epi == FB_EPI_QKV && L.m > 0 && L.seq_total > 0) {
      rc = encode_rope_table(&P.tma_cos, L.rope_cos, L.seq_total, err);
      if (!rc) rc = encode_rope_table(&P.tma_sin, L.rope_sin, L.seq_total, err);
      if (rc) return rc;
    }
    P.absmax = wfmt == 2 ? L.w_scale : L.absmax;
    P.fp8_e5m2 = wfmt == 3 ? L.w_f8_e5m2 : 0;
    P.code16 = L.code16;
    P.absmax_per_row = L.k / 64;
    P.bias = L.bias;
    P.out = L.out;
    P.resid = L.resid;
    P.gate = L.gate;
    P.q_scale = L.q_scale;
    P.k_scale = L.k_scale;
    P.rope_cos = L.rope_cos;
    P.rope_sin = L.rope_sin;
    P.q = L.q;
    P.k = L.k_out;
    P.v = L.v;
    P.ld_out = L.ld_out;
    P.ld_resid = L.ld_resid;
    P.gate_bstride = L.gate_batch_stride;
    P.m = L.m;
    P.n = L.n;
    P.num_kb = (L.k + gemm::BK - 1) / gemm::BK;
    P.tiles_m = (L.m + BM - 1) / BM;
    P.tiles_n = (L.n + BN - 1) / BN;
    P.tile_begin = tiles;
    tiles += P.tiles_m * P.tiles_n;
    P.tile_end = tiles;
    P.rows_per_batch = L.rows_per_batch;
    P.guard = L.guard;
    P.heads = L.heads;
    P.seq_total = L.seq_total;
    P.seq_offset = L.seq_offset;
    P.qkv_cols = epi == FB_EPI_QKV ? L.qkv_cols : 0;
    P.gelu_col0 = L.gelu_col0;
    P.n_offset = n_off;
    P.sp_world = epi == FB_EPI_QKV ? L.sp_world : 0;
    P.sp_rank = L.sp_rank;
    for (int g = 0; g < 8; ++g) P.sp_dst[g] = g < P.sp_world ? L.sp_qkv_dst[g] : nullptr;
    args.nprob = i + 1;
  }
  args.total_tiles = tiles;
  args.status = status;
  args.splits = 1;
  if (tiles == 0) return FB_OK;
  // Split-K for the decoding GEMM when its tiles leave more than half of the CTA pairs idle (e.g. the
  // N = 3072 Linears of a few hundred tokens: sequence-parallel ranks): S splits of whole 4-step NF4
  // groups, at least 8 K steps each, S * tiles <= pairs (one work item per pair, so the workspace of
  // one [2][128][256] fp32 block per item always suffices).
  const int npairs = sm_count / 2;
  if (decode && splitk && splitk->splitk_ws && 2 * tiles <= npairs) {
    for (int cand = 4; cand >= 2; --cand) {
      bool fits = cand * tiles <= npairs;
      for (int i = 0; fits && i < args.nprob; ++i)
        fits = args.prob[i].num_kb % (4 * cand) == 0 && args.prob[i].num_kb / cand >= 8;
      if (fits) {
        args.splits = cand;
        break;
      }
    }
  }
  if (args.splits > 1) {
    args.splitk_ws = splitk->splitk_ws;
    args.splitk_count = splitk->splitk_count;
  }
  cudaError_t e;
  if (pair || decode) {
    const int grid = 2 * std::min(tiles * args.splits, npairs);  // whole CTA pairs
    e = decode ? launch_gemm_decode(wfmt, epi, args, grid, st) : launch_gemm_pair(epi, args, grid, st);
  } else {
    const int grid = std::min(tiles, sm_count);
    e = BN == 256 ? dispatch_epi<256>(epi, args, grid, st) : dispatch_epi<64>(epi, args, grid, st);
  }
  if (e != cudaSuccess) {
    err = std::string("gemm launch: ") + cudaGetErrorString(e);
    return FB_ERR_CUDA;
  }
  return FB_OK;
}

}  // namespace fb
