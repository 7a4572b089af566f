// gemm_pair.cu — the bf16 GEMM of gemm.cu on CTA pairs: one tcgen05.mma.cta_group::2 computes a
// 256 x 256 tile on two SMs.
//
// Each CTA of a pair (a cluster of 2) loads its own 128 rows of A and its own half of the W tile
// (128 of the 256 output features) with TMA; the pair leader issues M=256, N=256, K=16 MMAs that
// read A from each CTA's shared memory and B from both. Each CTA's TMEM holds its 128 rows of the
// accumulator (256 fp32 columns, double-buffered). Per SM and 64-wide K block that is 32 KB of
// operands for a 128 x 256 x 64 share of the MMA, against 48 KB in the one-CTA kernel.
//
// An operand stage holds two 64-wide K blocks (A and B as two 128-byte-swizzled boxes each, 64 KB per
// CTA), 3 stages: every stage costs a full-barrier wait and a commit on the MMA side and a wait plus
// TMA issues on the producer side, and with 1024 instead of 512 tensor cycles per stage that overhead
// halves (measured: +2 to +9 % on the FLUX shapes against six 32 KB stages, bit-identical).
//
// Synchronisation (every cross-CTA signal names its one target barrier; no broadcast loads):
//   full[s]     lives in the leader; the leader arms it for both CTAs' bytes, both CTAs' TMA loads
//               (cta_group::2) complete on it; only the leader's MMA thread waits on it
//   empty[s]    one per CTA; after the MMAs reading stage s the leader signals both with ONE commit
//               whose CTA mask names both CTAs (two separate commits per stage cost 3-5 % of the
//               GEMM's throughput on every FLUX shape)
//   acc_full[a] one per CTA; the leader signals both (one masked commit) when accumulator a is complete
//   acc_empty[a] lives in the leader; every epilogue warp of both CTAs arrives on it (8 or 16)
//   rfull[w]    one per epilogue warp of each CTA: the warp's TMA boxes landed in its 4 KB staging
//               buffer (the residual of the gated residual, the RoPE tables of the QKV epilogue)
// Every wait is bounded (fb_common.cuh). The CTAs meet at cluster barriers after set-up and before
// TMEM is released, so neither leaves while the other may still signal it.
#include <cstdlib>

#include "gemm_common.cuh"

namespace fb {
namespace gemm_pair {

using namespace gemm;

constexpr int BM = 256;   // pair tile rows (128 per CTA)
constexpr int BN = 256;   // pair tile columns (W rows: 128 loaded by each CTA)
// warp 0 TMA, warp 1 MMA, then the epilogue warps: for the gated-residual and QKV epilogues two per
// TMEM lane quarter, each finishing one 128-column half of the tile's rows (the heavier epilogues of
// a K=3072 tile otherwise hold the accumulator past the next tile's mainloop: +5 % on the double
// block's QKV and proj shapes); for the light ones one per quarter (eight made MLP-in 2 % slower).
template <int EPI>
constexpr int epi_warps() {
  return (EPI == FB_EPI_GATED_RESIDUAL || EPI == FB_EPI_QKV) ? 8 : 4;
}
template <int EPI>
constexpr int threads_of() {
  return 64 + 32 * epi_warps<EPI>();
}
constexpr int kSub = 2;                       // 64-wide K blocks per stage
constexpr int kStages = 3;
constexpr int kBoxBytes = 128 * BK * 2;        // one 128-row x 64-column box: 16 KB
constexpr int kABytes = kSub * kBoxBytes;      // 32 KB
constexpr int kBBytes = kSub * kBoxBytes;      // 32 KB
constexpr int kStageBytes = kABytes + kBBytes;
// a 4 KB staging buffer per epilogue warp: the gated residual's 32-row x 32-column fp32 boxes
// (resid_row_tma), the QKV epilogue's RoPE table boxes (epilogue_qkv_group)
template <int EPI>
constexpr int resid_bytes() {
  return (EPI == FB_EPI_GATED_RESIDUAL || EPI == FB_EPI_QKV) ? epi_warps<EPI>() * kResidBoxBytes : 0;
}
template <int EPI>
constexpr int smem_of() {
  return kStages * kStageBytes + resid_bytes<EPI>() + 256 + 1024;
}
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kIdesc = idesc_bf16_f32(256, 256, false);

template <int EPI>
__global__ void __launch_bounds__(threads_of<EPI>(), 1) gemm_pair_kernel(const __grid_constant__ Args args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStages * kABytes;
  uint8_t* sR = sB + kStages * kBBytes;  // staging buffers (gated residual, QKV; 1024-byte aligned)
  uint64_t* full = reinterpret_cast<uint64_t*>(sR + resid_bytes<EPI>());
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint64_t* rfull = reinterpret_cast<uint64_t*>(tmem_slot + 2);  // [epilogue warp]: its staged boxes landed

  const int warp = warp_id();
  const int lane = lane_id();
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 2 * epi_warps<EPI>());  // every epilogue warp of the two CTAs
    }
    mbar_init(drain, 1);
    if constexpr (resid_bytes<EPI>() > 0) {
      for (int w = 0; w < epi_warps<EPI>(); ++w) mbar_init(&rfull[w], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    for (int p = 0; p < args.nprob; ++p) {
      tma_prefetch_desc(&args.prob[p].tma_a);
      tma_prefetch_desc(&args.prob[p].tma_b);
      if constexpr (EPI == FB_EPI_GATED_RESIDUAL) tma_prefetch_desc(&args.prob[p].tma_resid);
      if constexpr (EPI == FB_EPI_QKV) {
        tma_prefetch_desc(&args.prob[p].tma_cos);
        tma_prefetch_desc(&args.prob[p].tma_sin);
      }
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before_sync();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before either signals the other
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_parity[kStages];
      for (int s = 0; s < kStages; ++s) issued_parity[s] = 0xFFFFFFFFu;
      bool ok = true;
      for (int tile = pair; ok && tile < args.total_tiles; tile += npairs) {
        int p, mb, nb;
        decode_tile(args, tile, p, mb, nb);
        const Problem& P = args.prob[p];
        const int nstage = (P.num_kb + kSub - 1) / kSub;  // a K tail past the end is zero-filled by TMA
        for (int ks = 0; ks < nstage; ++ks) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, args.status, FB_DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * kStageBytes);
#pragma unroll
          for (int h = 0; h < kSub; ++h) {
            const int kx = (ks * kSub + h) * BK;
            tma_load_2d_pair(&P.tma_a, bar, sA + stage * kABytes + h * kBoxBytes, kx, mb * BM + 128 * static_cast<int>(rank));
            tma_load_2d_pair(&P.tma_b, bar, sB + stage * kBBytes + h * kBoxBytes, kx, nb * BN + 128 * static_cast<int>(rank));
          }
          issued_parity[stage] = phase;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && leader) {
        // every load of both CTAs completes on the leader's full barriers: let them land (bounded)
        for (int s = 0; s < kStages; ++s)
          if (issued_parity[s] != 0xFFFFFFFFu) mbar_wait_quiet(&full[s], issued_parity[s], kWaitBudgetNs);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (leader only)
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < args.total_tiles; tile += npairs) {
        int p, mb, nb;
        decode_tile(args, tile, p, mb, nb);
        const Problem& P = args.prob[p];
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, abort_flag, args.status, FB_DEV_TIMEOUT_EPI)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        const int nstage = (P.num_kb + kSub - 1) / kSub;
        for (int ks = 0; ks < nstage; ++ks) {
          if (!mbar_wait(&full[stage], phase, abort_flag, args.status, FB_DEV_TIMEOUT_TMA)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t a0 = smem_u32(sA + stage * kABytes);
          const uint32_t b0 = smem_u32(sB + stage * kBBytes);
#pragma unroll
          for (int h = 0; h < kSub; ++h) {
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) {
              umma_bf16_ss_pair(d_tmem, sdesc_kmajor_sw128(a0 + h * kBoxBytes + 32 * k),
                                sdesc_kmajor_sw128(b0 + h * kBoxBytes + 32 * k), kIdesc,
                                (ks > 0 || h > 0 || k > 0) ? 1u : 0u);
            }
          }
          const uint32_t e = smem_u32(&empty[stage]);
          umma_commit_pair_both(e);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        const uint32_t af = smem_u32(&acc_full[acc]);
        umma_commit_pair_both(af);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      umma_commit_pair(mapa_shared(smem_u32(drain), 0));
      mbar_wait_quiet(drain, 0, kWaitBudgetNs);
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2.., both CTAs)
    const int quarter = warp & 3;  // the TMEM lanes a warp may read are fixed by warp % 4
    constexpr int kParts = epi_warps<EPI>() / 4;  // column parts of a tile row
    const int part = (warp - 2) >> 2;
    const int row_in_tile = quarter * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    uint32_t rphase = 0;
    for (int tile = pair; tile < args.total_tiles; tile += npairs) {
      int p, mb, nb;
      decode_tile(args, tile, p, mb, nb);
      const Problem& P = args.prob[p];
      if (!mbar_wait(&acc_full[acc], acc_phase, abort_flag, args.status, FB_DEV_TIMEOUT_MMA)) break;
      tc_fence_after_sync();
      const uint32_t trow = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
      const int m = mb * BM + 128 * static_cast<int>(rank) + row_in_tile;
      if constexpr (EPI == FB_EPI_GATED_RESIDUAL) {
        const int ew = warp - 2;
        const int row0 = mb * BM + 128 * static_cast<int>(rank) + quarter * 32;
        if (!resid_row_tma<BN>(P, m, m < P.m, nb, trow, part * (BN / kParts) / 32, (part + 1) * (BN / kParts) / 32,
                               row0, sR + ew * kResidBoxBytes, &rfull[ew], rphase, abort_flag, args.status)) {
          mbar_wait_quiet(&rfull[ew], rphase, kWaitBudgetNs);  // the box in flight lands before the CTA exits
          break;
        }
      } else if constexpr (EPI == FB_EPI_QKV) {
        // the RoPE tables go through the warp's buffer when its 32 rows are 32 consecutive positions of
        // one image (image boundaries on multiples of 32 rows) and the first of them exists
        const int ew = warp - 2;
        const int row0 = mb * BM + 128 * static_cast<int>(rank) + quarter * 32;
        const bool stage_ok = row0 < P.m && P.rows_per_batch % 32 == 0;
        const int img0 = row0 / P.rows_per_batch;
        const RopeStage st{stage_ok, sR + ew * kResidBoxBytes, &rfull[ew], &rphase,
                           P.seq_offset + (row0 - img0 * P.rows_per_batch), abort_flag, args.status};
        if (!epilogue_row<BN, EPI>(P, m, m < P.m, nb, trow, part * (BN / kParts), (part + 1) * (BN / kParts), st)) {
          mbar_wait_quiet(&rfull[ew], rphase, kWaitBudgetNs);  // the boxes in flight land before the CTA exits
          break;
        }
      } else {
        epilogue_row<BN, EPI>(P, m, m < P.m, nb, trow, part * (BN / kParts), (part + 1) * (BN / kParts));
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(mapa_shared(smem_u32(&acc_empty[acc]), 0));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }

  tc_fence_before_sync();
  __syncthreads();
  cluster_sync_all();  // the peer no longer signals this CTA and nobody reads this CTA's TMEM
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

}  // namespace gemm_pair

std::string gemm_pair_setup() {
  using namespace gemm_pair;
  cudaError_t e = cudaSuccess;
  e = e ? e : cudaFuncSetAttribute(gemm_pair_kernel<FB_EPI_STORE_BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_of<FB_EPI_STORE_BF16>());
  e = e ? e : cudaFuncSetAttribute(gemm_pair_kernel<FB_EPI_STORE_F32>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_of<FB_EPI_STORE_F32>());
  e = e ? e : cudaFuncSetAttribute(gemm_pair_kernel<FB_EPI_GELU>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_of<FB_EPI_GELU>());
  e = e ? e : cudaFuncSetAttribute(gemm_pair_kernel<FB_EPI_GATED_RESIDUAL>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_of<FB_EPI_GATED_RESIDUAL>());
  e = e ? e : cudaFuncSetAttribute(gemm_pair_kernel<FB_EPI_QKV>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_of<FB_EPI_QKV>());
  return e == cudaSuccess ? std::string() : std::string("cudaFuncSetAttribute(gemm_pair): ") + cudaGetErrorString(e);
}

template <int EPI>
static cudaError_t launch_pair_t(const gemm::Args& args, int grid, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(gemm_pair::threads_of<EPI>(), 1, 1);
  cfg.dynamicSmemBytes = gemm_pair::smem_of<EPI>();
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemm_pair::gemm_pair_kernel<EPI>, args);
}

cudaError_t launch_gemm_pair(int epi, const gemm::Args& args, int grid, cudaStream_t st) {
  switch (epi) {
    case FB_EPI_STORE_BF16: return launch_pair_t<FB_EPI_STORE_BF16>(args, grid, st);
    case FB_EPI_STORE_F32: return launch_pair_t<FB_EPI_STORE_F32>(args, grid, st);
    case FB_EPI_GELU: return launch_pair_t<FB_EPI_GELU>(args, grid, st);
    case FB_EPI_GATED_RESIDUAL: return launch_pair_t<FB_EPI_GATED_RESIDUAL>(args, grid, st);
    default: return launch_pair_t<FB_EPI_QKV>(args, grid, st);
  }
}

bool gemm_pair_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("FLUX_B200_GEMM");
    return !(v && std::string(v) == "single");
  }();
  return on;
}

}  // namespace fb
