// vae.cu — the FLUX autoencoder decoder's kernels (selas/models/vae.py) on sm_100a.
//
// Activations are NHWC fp32 ([B, H, W, C], channels contiguous, a pixel stride >= C), so that a
// convolution is an implicit GEMM whose K dimension (input channels) is contiguous:
//
//   out[b, y, x, n] = bias[n] + sum_{r, s, c} in[b, y + r - R/2, x + s - R/2, c] * w[n, r, s, c]  (+ resid)
//
// conv_kernel — persistent, warp-specialised tcgen05 kernel, kind::tf32 (fp32 operands read as tf32,
// fp32 accumulation: the arithmetic torch uses for fp32 convolutions on tensor-core GPUs):
//   warp 0      TMA producer. The A tile of one K step is a 4-D box {32 channels, TW, TH, 1} of the
//               input at the tap's offset: 128 output pixels x 128 bytes, written in the 128-byte
//               swizzle layout the MMA reads as a K-major operand. Coordinates outside the image
//               (the 3x3 halo) are zero-filled by the TMA unit, which is exactly the conv's zero
//               padding. The B tile is {32, BN, 1} of the tap-major weights [R*R, Cout, Cin].
//   warp 1      TMEM allocation + MMA issue (one thread): 4 x tcgen05.mma M=128 N=BN K=8 per stage.
//   warps 2..5  epilogue: thread = TMEM lane = output pixel; bias, residual, tf32 rounding or the
//               final NCHW clamp, fp32 stores. Two TMEM accumulators: the epilogue of tile i overlaps
//               the mainloop of tile i+1.
// A 1x1 convolution is a plain GEMM, which is how the mid-block attention's products run too
// (S = Q K^T with Q, K column slices of the fused QKV output; O = P V with V transposed as the weights).
//
// strip_kernel — the 3x3 convolutions of images at least 128 pixels wide, BN = 128. A tile is two
// image rows x 128 pixels. For each kernel row r and 32-channel chunk, one stage holds the two input
// row segments the tile needs (130 pixels each: the 128 outputs' columns plus the halo) and the three
// taps (r, 0..2) of the weights; the three horizontal taps read the same A segment through descriptors
// shifted by s rows (128 B), so the TMA unit fetches 0.42 rows of 128 B per tensor-core cycle instead
// of 1.0 (the limiter of the tile-per-tap kernel at BN = 128).
//
// The memory-bound kernels around it: GroupNorm statistics (fp64 block partials, reduced in a fixed
// order: deterministic), GroupNorm apply (+ SiLU, + tf32 rounding for the conv that reads it), nearest
// 2x upsampling, the attention row softmax, a transpose, and the latent preparation (NCHW z / scale +
// shift -> NHWC, channels padded to 32).
#include "fb_internal.h"

namespace fb {
namespace vae {

constexpr int BM = 128;
constexpr int kThreads = 192;
constexpr int kEpiThreads = 128;

template <int BN>
struct Cfg {
  static constexpr int kStages = BN >= 256 ? 4 : (BN >= 128 ? 7 : 8);
  static constexpr int kABytes = BM * 128;
  static constexpr int kBBytes = BN * 128;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;
  static constexpr int kSmemBytes = kStages * kStageBytes + 256 + 1024;
  static constexpr uint32_t kIdesc = idesc_tf32_f32(BM, BN);
};

struct ConvArgs {
  CUtensorMap tma_in;  // {C, W, H, B}, box {32, tw, th, 1}
  CUtensorMap tma_w;   // {Cin, Cout, R*R}, box {32, BN, 1} (strip kernel: {32, 128, 3})
  const float* bias;   // [Cout] or null
  const float* resid;  // NHWC, pixel stride ld_resid, or null
  float* out;          // NHWC pixel stride ld_out, or NCHW [B, Cout, H, W] (kOutNchwClamp)
  int64_t ld_resid, ld_out;
  int batch, H, W, cin, cout, R;
  int tw, th, tiles_w, tiles_h, n_tiles;
  int total_tiles, num_kb, kb_per_tap;
  int flags;
  int* status;
};

constexpr int kRoundOut = 1;      // round the outputs to tf32 (they feed another tf32 product)
constexpr int kOutNchwClamp = 2;  // store NCHW, clamped to [-1, 1] (the decoder's last conv)
constexpr int kScalarIo = 4;      // internal: out / resid rows not 16-byte aligned, element stores

__device__ __forceinline__ void decode_tile(const ConvArgs& a, int tile, int& b, int& y0, int& x0, int& nb) {
  nb = tile % a.n_tiles;
  int t = tile / a.n_tiles;
  const int tx = t % a.tiles_w;
  t /= a.tiles_w;
  const int ty = t % a.tiles_h;
  b = t / a.tiles_h;
  y0 = ty * a.th;
  x0 = tx * a.tw;
}

template <int BN>
__device__ __forceinline__ void epilogue_chunk(const ConvArgs& a, const uint32_t* r, int ncols, int n0, int b, int y,
                                               int x, bool ok) {
  if (!ok) return;
  const int64_t pix = (static_cast<int64_t>(b) * a.H + y) * a.W + x;
  if (a.flags & kOutNchwClamp) {
    for (int j = 0; j < ncols; ++j) {
      const int n = n0 + j;
      if (n >= a.cout) break;
      float v = __uint_as_float(r[j]);
      if (a.bias) v = __fadd_rn(v, __ldg(a.bias + n));
      v = fminf(fmaxf(v, -1.0f), 1.0f);
      a.out[((static_cast<int64_t>(b) * a.cout + n) * a.H + y) * a.W + x] = v;
    }
    return;
  }
  float* dst = a.out + pix * a.ld_out + n0;
  const float* res = a.resid ? a.resid + pix * a.ld_resid + n0 : nullptr;
  const bool full = n0 + ncols <= a.cout && !(a.flags & kScalarIo);
#pragma unroll
  for (int j4 = 0; j4 < ncols / 4; ++j4) {
    float v[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int j = 4 * j4 + q;
      v[q] = __uint_as_float(r[j]);
      if (a.bias && (full || n0 + j < a.cout)) v[q] = __fadd_rn(v[q], __ldg(a.bias + n0 + j));
    }
    if (full) {
      if (res) {
        const float4 rr = __ldg(reinterpret_cast<const float4*>(res) + j4);
        v[0] = __fadd_rn(rr.x, v[0]);
        v[1] = __fadd_rn(rr.y, v[1]);
        v[2] = __fadd_rn(rr.z, v[2]);
        v[3] = __fadd_rn(rr.w, v[3]);
      }
      if (a.flags & kRoundOut) {
#pragma unroll
        for (int q = 0; q < 4; ++q) v[q] = tf32_round(v[q]);
      }
      reinterpret_cast<float4*>(dst)[j4] = make_float4(v[0], v[1], v[2], v[3]);
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int j = 4 * j4 + q;
        if (n0 + j >= a.cout) break;
        float w = v[q];
        if (res) w = __fadd_rn(res[j], w);
        if (a.flags & kRoundOut) w = tf32_round(w);
        dst[j] = w;
      }
    }
  }
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1) conv_kernel(const __grid_constant__ ConvArgs args) {
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
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kEpiThreads);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&args.tma_in);
    tma_prefetch_desc(&args.tma_w);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  const int pad = args.R / 2;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_parity[C::kStages];
      for (int s = 0; s < C::kStages; ++s) issued_parity[s] = 0xFFFFFFFFu;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < args.total_tiles; tile += gridDim.x) {
        int b, y0, x0, nb;
        decode_tile(args, tile, b, y0, x0, nb);
        for (int kb = 0; kb < args.num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, args.status, FB_DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          const int tap = kb / args.kb_per_tap;
          const int c0 = (kb - tap * args.kb_per_tap) * 32;
          const int r = tap / args.R, s = tap - (tap / args.R) * args.R;
          mbar_arrive_expect_tx(&full[stage], C::kStageBytes);
          tma_load_4d(&args.tma_in, &full[stage], sA + stage * C::kABytes, c0, x0 + s - pad, y0 + r - pad, b);
          tma_load_3d(&args.tma_w, &full[stage], sB + stage * C::kBBytes, c0, nb * BN, tap);
          issued_parity[stage] = phase;
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        for (int s = 0; s < C::kStages; ++s)
          if (issued_parity[s] != 0xFFFFFFFFu) mbar_wait_quiet(&full[s], issued_parity[s], kWaitBudgetNs);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < args.total_tiles; tile += gridDim.x) {
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, abort_flag, args.status, FB_DEV_TIMEOUT_EPI)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < args.num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, args.status, FB_DEV_TIMEOUT_TMA)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t a0 = smem_u32(sA + stage * C::kABytes);
          const uint32_t b0 = smem_u32(sB + stage * C::kBBytes);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_tf32_ss(d_tmem, sdesc_kmajor_sw128(a0 + 32 * k), sdesc_kmajor_sw128(b0 + 32 * k), C::kIdesc,
                         (kb > 0 || k > 0) ? 1u : 0u);
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
      umma_commit(drain);
      mbar_wait_quiet(drain, 0, kWaitBudgetNs);
    }
  } else {
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < args.total_tiles; tile += gridDim.x) {
      int b, y0, x0, nb;
      decode_tile(args, tile, b, y0, x0, nb);
      if (!mbar_wait(&acc_full[acc], acc_phase, abort_flag, args.status, FB_DEV_TIMEOUT_MMA)) break;
      tc_fence_after_sync();
      const int y = y0 + row / args.tw, x = x0 + row % args.tw;
      const bool ok = y < args.H && x < args.W;
      const uint32_t trow = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
      if constexpr (BN >= 32) {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(trow + 32 * c, r);
          tmem_ld_wait();
          epilogue_chunk<BN>(args, r, 32, nb * BN + 32 * c, b, y, x, ok);
        }
      } else {
        uint32_t r[16];
        tmem_ld_32x32b_x16(trow, r);
        tmem_ld_wait();
        epilogue_chunk<BN>(args, r, 16, nb * BN, b, y, x, ok);
      }
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

// ------------------------------------------------------------------------------------------ strip kernel

// Descriptor of a K-major SW128 operand whose start `addr` is shifted by whole 128-byte rows from the
// 1024-byte swizzle atom the TMA unit wrote. The MMA derives the swizzle phase of every row it reads
// from the shared-memory address itself (measured on sm_100a: the base-offset field must stay 0 for
// such a start; setting it to the row phase gives wrong products), so the plain descriptor at the
// shifted address reads rows s .. s + 127 of the segment.
__device__ __forceinline__ uint64_t sdesc_sw128_rowshift(uint32_t addr) { return sdesc_kmajor_sw128(addr); }

struct StripCfg {
  static constexpr int BN = 128;
  static constexpr int kARows = 130;                      // 128 output columns + the 3x3 halo
  static constexpr int kATx = kARows * 128;               // bytes one A box moves
  static constexpr int kABytes = 17 * 1024;               // one A segment, padded to the 1 KB atom
  static constexpr int kBBytes = 3 * BN * 128;            // taps (r, 0..2): [s][n][32 ch]
  static constexpr int kStageBytes = kBBytes + 2 * kABytes;
  static constexpr int kStageTx = kBBytes + 2 * kATx;
  static constexpr int kStages = 2;
  static constexpr int kTmemCols = 512;                   // 2 accumulators x 2 rows x 128 columns
  static constexpr int kSmemBytes = kStages * kStageBytes + 256 + 1024;
  static constexpr uint32_t kIdesc = idesc_tf32_f32(BM, BN);
};

__global__ void __launch_bounds__(kThreads, 1) strip_kernel(const __grid_constant__ ConvArgs args) {
  using C = StripCfg;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sB = smem;                                  // kStages x kBBytes
  uint8_t* sA = smem + C::kStages * C::kBBytes;        // kStages x 2 x kABytes
  uint64_t* full = reinterpret_cast<uint64_t*>(sA + C::kStages * 2 * C::kABytes);
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
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kEpiThreads);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&args.tma_in);
    tma_prefetch_desc(&args.tma_w);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  const int kb_per_tap = args.kb_per_tap;  // 32-channel chunks
  const int steps = 3 * kb_per_tap;        // (kernel row, chunk) stages per tile

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_parity[C::kStages];
      for (int s = 0; s < C::kStages; ++s) issued_parity[s] = 0xFFFFFFFFu;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < args.total_tiles; tile += gridDim.x) {
        int b, y0, x0, nb;
        decode_tile(args, tile, b, y0, x0, nb);
        for (int st = 0; st < steps; ++st) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, args.status, FB_DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          const int r = st / kb_per_tap;
          const int c0 = (st - r * kb_per_tap) * 32;
          uint8_t* a = sA + stage * 2 * C::kABytes;
          mbar_arrive_expect_tx(&full[stage], C::kStageTx);
          tma_load_4d(&args.tma_in, &full[stage], a, c0, x0 - 1, y0 + r - 1, b);
          tma_load_4d(&args.tma_in, &full[stage], a + C::kABytes, c0, x0 - 1, y0 + r, b);
          tma_load_3d(&args.tma_w, &full[stage], sB + stage * C::kBBytes, c0, nb * C::BN, 3 * r);
          issued_parity[stage] = phase;
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        for (int s = 0; s < C::kStages; ++s)
          if (issued_parity[s] != 0xFFFFFFFFu) mbar_wait_quiet(&full[s], issued_parity[s], kWaitBudgetNs);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < args.total_tiles; tile += gridDim.x) {
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, abort_flag, args.status, FB_DEV_TIMEOUT_EPI)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        for (int st = 0; st < steps; ++st) {
          if (!mbar_wait(&full[stage], phase, abort_flag, args.status, FB_DEV_TIMEOUT_TMA)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t a0 = smem_u32(sA + stage * 2 * C::kABytes);
          const uint32_t b0 = smem_u32(sB + stage * C::kBBytes);
#pragma unroll
          for (int t = 0; t < 2; ++t) {  // output row y0 + t reads input row y0 + t + r - 1 = segment t
            const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * 2 * C::BN + t * C::BN);
#pragma unroll
            for (int s = 0; s < 3; ++s) {
#pragma unroll
              for (int k = 0; k < 4; ++k)
                umma_tf32_ss(d_tmem, sdesc_sw128_rowshift(a0 + t * C::kABytes + 128 * s + 32 * k),
                             sdesc_kmajor_sw128(b0 + s * C::BN * 128 + 32 * k), C::kIdesc,
                             (st > 0 || s > 0 || k > 0) ? 1u : 0u);
            }
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
      umma_commit(drain);
      mbar_wait_quiet(drain, 0, kWaitBudgetNs);
    }
  } else {
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < args.total_tiles; tile += gridDim.x) {
      int b, y0, x0, nb;
      decode_tile(args, tile, b, y0, x0, nb);
      if (!mbar_wait(&acc_full[acc], acc_phase, abort_flag, args.status, FB_DEV_TIMEOUT_MMA)) break;
      tc_fence_after_sync();
      const int x = x0 + row;
#pragma unroll 1
      for (int t = 0; t < 2; ++t) {
        const int y = y0 + t;
        const bool ok = y < args.H && x < args.W;
        const uint32_t trow = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                              static_cast<uint32_t>(acc * 2 * C::BN + t * C::BN);
#pragma unroll 1
        for (int c = 0; c < C::BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(trow + 32 * c, r);
          tmem_ld_wait();
          epilogue_chunk<C::BN>(args, r, 32, nb * C::BN + 32 * c, b, y, x, ok);
        }
      }
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

// ------------------------------------------------------------------------------------------ GroupNorm

constexpr int kGnThreads = 256;
constexpr int kGnBlocksPerImage = 8 * kNumSms;  // statistics partials per image (upper bound)
constexpr int kGnUnroll = 4;

// Threads are laid out (pixel lane, channel float4): q = t % (C/4) is fixed per thread, so its group,
// gamma/beta and statistics are loaded once; the 256 / (C/4) pixel lanes of a block walk the block's
// span of pixels, kGnUnroll loads in flight per thread. C in {128, 256, 512, 1024}: C/4 divides 256 and
// a group (C/32 >= 4 channels) holds whole float4s.

// Per-block partial sums of x and x^2 of the 32 groups of one image, combined per group in a fixed
// order (deterministic).
__global__ void __launch_bounds__(kGnThreads) gn_stats_kernel(const float* __restrict__ x, int64_t hw, int c,
                                                              int64_t ld, double* __restrict__ partial) {
  __shared__ double s_su[kGnThreads], s_sq[kGnThreads];
  const int b = blockIdx.y;
  const int c4 = c / 4;
  const int lanes = kGnThreads / c4;
  const int q = threadIdx.x % c4, lane = threadIdx.x / c4;
  const int64_t per = (hw + gridDim.x - 1) / gridDim.x;
  const int64_t p0 = blockIdx.x * per, p1 = min(hw, p0 + per);
  const float4* base = reinterpret_cast<const float4*>(x + static_cast<int64_t>(b) * hw * ld) + q;
  const int64_t ld4 = ld / 4;
  double su = 0.0, sq = 0.0;
  int64_t p = p0 + lane;
  for (; p + (kGnUnroll - 1) * lanes < p1; p += kGnUnroll * lanes) {
    float4 v[kGnUnroll];
#pragma unroll
    for (int u = 0; u < kGnUnroll; ++u) v[u] = __ldg(base + (p + u * lanes) * ld4);
    float fs = 0.0f, fq = 0.0f;  // 16 values in fp32 (relative error ~1e-7), then fp64
#pragma unroll
    for (int u = 0; u < kGnUnroll; ++u) {
      fs += (v[u].x + v[u].y) + (v[u].z + v[u].w);
      fq += (v[u].x * v[u].x + v[u].y * v[u].y) + (v[u].z * v[u].z + v[u].w * v[u].w);
    }
    su += static_cast<double>(fs);
    sq += static_cast<double>(fq);
  }
  for (; p < p1; p += lanes) {
    const float4 v = __ldg(base + p * ld4);
    su += (static_cast<double>(v.x) + static_cast<double>(v.y)) + (static_cast<double>(v.z) + static_cast<double>(v.w));
    sq += (static_cast<double>(v.x) * v.x + static_cast<double>(v.y) * v.y) +
          (static_cast<double>(v.z) * v.z + static_cast<double>(v.w) * v.w);
  }
  s_su[threadIdx.x] = su;
  s_sq[threadIdx.x] = sq;
  __syncthreads();
  if (threadIdx.x < 32) {
    const int g = threadIdx.x;
    const int per_group = c4 / 32;  // float4s of one group within a pixel
    double a = 0.0, bq = 0.0;
    for (int l = 0; l < lanes; ++l) {
      for (int k = 0; k < per_group; ++k) {
        const int t = l * c4 + g * per_group + k;
        a += s_su[t];
        bq += s_sq[t];
      }
    }
    // group-major ([b][g][part][2]), so the finishing warp of a group reads its partials contiguously
    double* dst = partial + ((static_cast<int64_t>(b) * 32 + g) * gridDim.x + blockIdx.x) * 2;
    dst[0] = a;
    dst[1] = bq;
  }
}

// mean and 1/sqrt(var + eps) of each (image, group), from the partials in a fixed order: warp g of
// the image's block sums group g's partials lane-strided, then combines the 32 lanes by a fixed
// butterfly (deterministic).
__global__ void __launch_bounds__(1024) gn_finish_kernel(const double* __restrict__ partial, int parts, double count,
                                                         float eps, float* __restrict__ stats) {
  const int b = blockIdx.x, g = threadIdx.x >> 5, lane = threadIdx.x & 31;
  double su = 0.0, sq = 0.0;
  const double2* p = reinterpret_cast<const double2*>(partial) + (static_cast<int64_t>(b) * 32 + g) * parts;
  for (int i = lane; i < parts; i += 32) {
    const double2 v = p[i];
    su += v.x;
    sq += v.y;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    su += __shfl_xor_sync(0xffffffffu, su, o);
    sq += __shfl_xor_sync(0xffffffffu, sq, o);
  }
  if (lane == 0) {
    const double mean = su / count;
    const double var = fmax(sq / count - mean * mean, 0.0);
    stats[(b * 32 + g) * 2] = static_cast<float>(mean);
    stats[(b * 32 + g) * 2 + 1] = static_cast<float>(1.0 / sqrt(var + static_cast<double>(eps)));
  }
}

// SiLU with the fast exponential and division: a few ulp of fp32, far below the tf32 rounding that
// follows (the conv reads 10 mantissa bits); for v -> -inf, exp(-v) -> inf and the quotient -> 0.
__device__ __forceinline__ float silu_f32(float v) { return __fdividef(v, 1.0f + __expf(-v)); }

__device__ __forceinline__ float gn_one(float x, float mean, float rstd, float g, float b, int silu, int round) {
  float t = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x, mean), rstd), g), b);
  if (silu) t = silu_f32(t);
  return round ? tf32_round(t) : t;
}

// y = (x - mean) * rstd * gamma + beta, then SiLU if asked, then tf32 rounding if asked.
__global__ void __launch_bounds__(kGnThreads) gn_apply_kernel(const float* __restrict__ x, int64_t hw, int c, int64_t ld,
                                                              const float* __restrict__ stats,
                                                              const float* __restrict__ gamma,
                                                              const float* __restrict__ beta, float* __restrict__ out,
                                                              int64_t ld_out, int silu, int round) {
  const int b = blockIdx.y;
  const int c4 = c / 4;
  const int lanes = kGnThreads / c4;
  const int q = threadIdx.x % c4, lane = threadIdx.x / c4;
  const int g = q / (c4 / 32);
  const float mean = stats[(b * 32 + g) * 2], rstd = stats[(b * 32 + g) * 2 + 1];
  const float4 ga = __ldg(reinterpret_cast<const float4*>(gamma) + q);
  const float4 be = __ldg(reinterpret_cast<const float4*>(beta) + q);
  const float4* xb = reinterpret_cast<const float4*>(x + static_cast<int64_t>(b) * hw * ld) + q;
  float4* ob = reinterpret_cast<float4*>(out + static_cast<int64_t>(b) * hw * ld_out) + q;
  const int64_t ld4 = ld / 4, lo4 = ld_out / 4;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * lanes;
  int64_t p = static_cast<int64_t>(blockIdx.x) * lanes + lane;
  for (; p + (kGnUnroll - 1) * stride < hw; p += kGnUnroll * stride) {
    float4 v[kGnUnroll];
#pragma unroll
    for (int u = 0; u < kGnUnroll; ++u) v[u] = __ldg(xb + (p + u * stride) * ld4);
#pragma unroll
    for (int u = 0; u < kGnUnroll; ++u)
      ob[(p + u * stride) * lo4] =
          make_float4(gn_one(v[u].x, mean, rstd, ga.x, be.x, silu, round), gn_one(v[u].y, mean, rstd, ga.y, be.y, silu, round),
                      gn_one(v[u].z, mean, rstd, ga.z, be.z, silu, round), gn_one(v[u].w, mean, rstd, ga.w, be.w, silu, round));
  }
  for (; p < hw; p += stride) {
    const float4 v = __ldg(xb + p * ld4);
    ob[p * lo4] = make_float4(gn_one(v.x, mean, rstd, ga.x, be.x, silu, round), gn_one(v.y, mean, rstd, ga.y, be.y, silu, round),
                              gn_one(v.z, mean, rstd, ga.z, be.z, silu, round), gn_one(v.w, mean, rstd, ga.w, be.w, silu, round));
  }
}

// ------------------------------------------------------------------------------------------ glue

// out[b, 2y + i, 2x + j, :] = in[b, y, x, :] (nearest, factor 2), optionally tf32-rounded. Thread
// layout (pixel lane, channel float4) as in the GroupNorm kernels: C/4 divides 256.
__global__ void __launch_bounds__(256) upsample2_kernel(const float4* __restrict__ in, int64_t pixels_in, int w_in,
                                                        int c4, float4* __restrict__ out, int round) {
  const int lanes = 256 / c4;
  const int q = threadIdx.x % c4, lane = threadIdx.x / c4;
  const int64_t w_out = 2 * static_cast<int64_t>(w_in);
  for (int64_t p = static_cast<int64_t>(blockIdx.x) * lanes + lane; p < pixels_in;
       p += static_cast<int64_t>(gridDim.x) * lanes) {
    const int64_t row = p / w_in;  // b * h_in + y
    const int64_t xx = p - row * w_in;
    float4 v = __ldg(in + p * c4 + q);
    if (round) v = make_float4(tf32_round(v.x), tf32_round(v.y), tf32_round(v.z), tf32_round(v.w));
    const int64_t o0 = ((2 * row) * w_out + 2 * xx) * c4 + q;  // (b, 2y, 2x): output row 2 * row
    out[o0] = v;
    out[o0 + c4] = v;
    out[o0 + w_out * c4] = v;
    out[o0 + w_out * c4 + c4] = v;
  }
}

constexpr int kSmThreads = 512;

// In place: s[r, :n] = softmax(s[r, :n] * scale) (tf32-rounded for the P V product when asked). One
// block per row, the row held in registers (n <= kSmThreads * 4 * kSmMaxPer); a ragged last float4
// (n % 4 != 0) is masked: its extra columns are stored as 0.
constexpr int kSmMaxPer = 16;
// PER float4 per thread, the smallest power of two that holds the row: with 8 or fewer the kernel stays
// under 64 registers, so two 512-thread rows share an SM and one's loads overlap the other's reductions.
template <int PER>
__global__ void __launch_bounds__(kSmThreads, PER <= 8 ? 2 : 1) softmax_rows_kernel(float* __restrict__ s, int n,
                                                                                   int64_t ld, float scale, int round) {
  __shared__ float red[kSmThreads / 32];
  float* row = s + static_cast<int64_t>(blockIdx.x) * ld;
  const int n4 = (n + 3) / 4;
  float4 v[PER];
  float mx = -INFINITY;
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int i = threadIdx.x + k * kSmThreads;
    if (i < n4) {
      v[k] = reinterpret_cast<const float4*>(row)[i];
      if (4 * i + 4 > n) {  // the ragged end of the row (column 4i is always < n)
        if (4 * i + 1 >= n) v[k].y = -INFINITY;
        if (4 * i + 2 >= n) v[k].z = -INFINITY;
        if (4 * i + 3 >= n) v[k].w = -INFINITY;
      }
      mx = fmaxf(mx, fmaxf(fmaxf(v[k].x, v[k].y), fmaxf(v[k].z, v[k].w)));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = red[0];
  for (int w = 1; w < kSmThreads / 32; ++w) mx = fmaxf(mx, red[w]);
  __syncthreads();
  const float ms = __fmul_rn(mx, scale);
  float sum = 0.0f;
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int i = threadIdx.x + k * kSmThreads;
    if (i < n4) {  // exp(-inf) = 0 for the masked columns
      v[k].x = __expf(__fsub_rn(__fmul_rn(v[k].x, scale), ms));
      v[k].y = __expf(__fsub_rn(__fmul_rn(v[k].y, scale), ms));
      v[k].z = __expf(__fsub_rn(__fmul_rn(v[k].z, scale), ms));
      v[k].w = __expf(__fsub_rn(__fmul_rn(v[k].w, scale), ms));
      sum += (v[k].x + v[k].y) + (v[k].z + v[k].w);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
  __syncthreads();
  sum = 0.0f;
  for (int w = 0; w < kSmThreads / 32; ++w) sum += red[w];
  const float inv = __fdiv_rn(1.0f, sum);
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int i = threadIdx.x + k * kSmThreads;
    if (i < n4) {
      float4 p = make_float4(__fmul_rn(v[k].x, inv), __fmul_rn(v[k].y, inv), __fmul_rn(v[k].z, inv),
                             __fmul_rn(v[k].w, inv));
      if (round) p = make_float4(tf32_round(p.x), tf32_round(p.y), tf32_round(p.z), tf32_round(p.w));
      reinterpret_cast<float4*>(row)[i] = p;
    }
  }
}

// out[c, r] = in[r, c] for in [rows, cols] (row stride ld_in) -> out [cols, rows] (row stride ld_out).
__global__ void transpose_kernel(const float* __restrict__ in, int rows, int cols, int64_t ld_in, float* __restrict__ out,
                                 int64_t ld_out) {
  __shared__ float t[32][33];
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int r = r0 + k, c = c0 + threadIdx.x;
    if (r < rows && c < cols) t[k][threadIdx.x] = in[static_cast<int64_t>(r) * ld_in + c];
  }
  __syncthreads();
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int c = c0 + k, r = r0 + threadIdx.x;
    if (r < rows && c < cols) out[static_cast<int64_t>(c) * ld_out + r] = t[threadIdx.x][k];
  }
}

// z [B, zc, H, W] (NCHW) -> out [B, H, W, cpad] = tf32(z / scale + shift), zero channels zc..cpad.
__global__ void latent_prep_kernel(const float* __restrict__ z, int batch, int zc, int h, int w, int cpad, float scale,
                                   float shift, float* __restrict__ out) {
  const int64_t n = static_cast<int64_t>(batch) * h * w * cpad;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % cpad);
    const int64_t p = i / cpad;
    const int x = static_cast<int>(p % w);
    const int64_t t = p / w;
    const int y = static_cast<int>(t % h);
    const int b = static_cast<int>(t / h);
    float v = 0.0f;
    if (c < zc) v = tf32_round(__fadd_rn(__fdiv_rn(z[((static_cast<int64_t>(b) * zc + c) * h + y) * w + x], scale), shift));
    out[i] = v;
  }
}


// ------------------------------------------------------------------------------------------ norm_out + conv_out

// The decoder's last two layers, GroupNorm + SiLU (norm_out) then the 3x3 conv to the 3 image channels
// (conv_out), as one CUDA-core kernel. With 3 outputs the tensor-core conv is bound by fetching its A
// tiles, and the GroupNorm output it reads is the largest tensor of the decode (1024^2 x 128 fp32); here
// each CTA reads the pre-norm input once, as a halo tile, and keeps everything else on chip.
//   - CTA = 32 x 16 output pixels, 128 threads; a thread computes 4 consecutive rows of one column,
//     all 3 outputs (12 accumulators).
//   - Per 16-channel chunk: the 18 x 34 input halo, GroupNorm + SiLU + tf32 rounding applied as it is
//     loaded (the values the tensor-core path reads; pixels outside the image are the conv's zero
//     padding), stored channel-major with an odd plane stride; the chunk's tf32 weights as one float4
//     (the 3 outputs) per (tap, channel).
//   - Per channel and horizontal tap a thread reads the 6 input rows its 4 outputs need and each tap's
//     weights once (a broadcast): 27 shared-memory loads feed 108 FMAs. Products of two tf32 values are
//     exact in fp32, so only the summation order differs from the tensor-core conv.
//   - Output: bias, clamp to [-1, 1], NCHW.
constexpr int kNcTW = 32, kNcTH = 16, kNcRows = 4, kNcThreads = kNcTW * kNcTH / kNcRows;
constexpr int kNcPW = kNcTW + 2, kNcPH = kNcTH + 2;
constexpr int kNcPlane = kNcPW * kNcPH + 1;  // odd: consecutive channel planes start in different banks
constexpr int kNcChunk = 16;                 // channels per chunk

__global__ void __launch_bounds__(kNcThreads) gn_conv_out_kernel(const float* __restrict__ x, int h, int w,
                                                                 const float* __restrict__ stats,
                                                                 const float* __restrict__ gamma,
                                                                 const float* __restrict__ beta,
                                                                 const float* __restrict__ wt,  // [9][3][128]
                                                                 const float* __restrict__ bias,
                                                                 float* __restrict__ out) {
  constexpr int C = 128, kCpg = C / 32;
  __shared__ float s_in[kNcChunk * kNcPlane];
  __shared__ float4 s_w[9 * kNcChunk];
  const int b = blockIdx.z;
  const int x0 = blockIdx.x * kNcTW, y0 = blockIdx.y * kNcTH;
  const int tx = threadIdx.x % kNcTW, r0 = (threadIdx.x / kNcTW) * kNcRows;
  const float* xb = x + static_cast<int64_t>(b) * h * w * C;
  float acc[kNcRows][3];
#pragma unroll
  for (int p = 0; p < kNcRows; ++p) acc[p][0] = acc[p][1] = acc[p][2] = 0.f;
  for (int c0 = 0; c0 < C; c0 += kNcChunk) {
    __syncthreads();  // the previous chunk's reads are done
    for (int i = threadIdx.x; i < kNcPH * kNcPW * (kNcChunk / 4); i += kNcThreads) {
      const int pix = i / (kNcChunk / 4), q = i % (kNcChunk / 4);
      const int py = pix / kNcPW, px = pix - py * kNcPW;
      const int gy = y0 + py - 1, gx = x0 + px - 1;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (gy >= 0 && gy < h && gx >= 0 && gx < w) {
        const int ch = c0 + 4 * q;
        const float4 t = __ldg(reinterpret_cast<const float4*>(xb + (static_cast<int64_t>(gy) * w + gx) * C + ch));
        const float4 ga = __ldg(reinterpret_cast<const float4*>(gamma + ch));
        const float4 be = __ldg(reinterpret_cast<const float4*>(beta + ch));
        const int g = ch / kCpg;
        const float mean = stats[(b * 32 + g) * 2], rstd = stats[(b * 32 + g) * 2 + 1];
        v = make_float4(gn_one(t.x, mean, rstd, ga.x, be.x, 1, 1), gn_one(t.y, mean, rstd, ga.y, be.y, 1, 1),
                        gn_one(t.z, mean, rstd, ga.z, be.z, 1, 1), gn_one(t.w, mean, rstd, ga.w, be.w, 1, 1));
      }
      float* d = s_in + (4 * q) * kNcPlane + py * kNcPW + px;
      d[0] = v.x;
      d[kNcPlane] = v.y;
      d[2 * kNcPlane] = v.z;
      d[3 * kNcPlane] = v.w;
    }
    for (int i = threadIdx.x; i < 9 * kNcChunk; i += kNcThreads) {
      const int t = i / kNcChunk, k = i % kNcChunk;
      const float* src = wt + t * 3 * C + c0 + k;
      s_w[i] = make_float4(__ldg(src), __ldg(src + C), __ldg(src + 2 * C), 0.f);
    }
    __syncthreads();
#pragma unroll 2
    for (int k = 0; k < kNcChunk; ++k) {
      const float* sk = s_in + k * kNcPlane + r0 * kNcPW + tx;
#pragma unroll
      for (int dx = 0; dx < 3; ++dx) {
        float v[kNcRows + 2];
#pragma unroll
        for (int r = 0; r < kNcRows + 2; ++r) v[r] = sk[r * kNcPW + dx];
#pragma unroll
        for (int dy = 0; dy < 3; ++dy) {
          const float4 wv = s_w[(dy * 3 + dx) * kNcChunk + k];
#pragma unroll
          for (int p = 0; p < kNcRows; ++p) {
            acc[p][0] = fmaf(v[p + dy], wv.x, acc[p][0]);
            acc[p][1] = fmaf(v[p + dy], wv.y, acc[p][1]);
            acc[p][2] = fmaf(v[p + dy], wv.z, acc[p][2]);
          }
        }
      }
    }
  }
  const int gx = x0 + tx;
  if (gx >= w) return;
  const float b0 = bias ? bias[0] : 0.f, b1 = bias ? bias[1] : 0.f, b2 = bias ? bias[2] : 0.f;
#pragma unroll
  for (int p = 0; p < kNcRows; ++p) {
    const int gy = y0 + r0 + p;
    if (gy < h) {
      float* o = out + (static_cast<int64_t>(b) * 3 * h + gy) * w + gx;
      const int64_t plane = static_cast<int64_t>(h) * w;
      o[0] = fminf(fmaxf(acc[p][0] + b0, -1.f), 1.f);
      o[plane] = fminf(fmaxf(acc[p][1] + b1, -1.f), 1.f);
      o[2 * plane] = fminf(fmaxf(acc[p][2] + b2, -1.f), 1.f);
    }
  }
}

}  // namespace vae

// ============================================================================================ host

namespace {

int fail(int code, const std::string& msg) {
  set_last_error(msg);
  return code;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

int launched(const char* what) {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? FB_OK : fail(FB_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int encode(CUtensorMap* map, int rank, const void* base, const cuuint64_t* dims, const cuuint64_t* strides,
           const cuuint32_t* box, std::string& err) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) {
    err = "cuTensorMapEncodeTiled unavailable";
    return FB_ERR_INIT;
  }
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, rank, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    err = "cuTensorMapEncodeTiled failed (" + std::to_string(static_cast<int>(r)) + ")";
    return FB_ERR_CUDA;
  }
  return FB_OK;
}

template <int BN>
cudaError_t launch_conv_bn(const vae::ConvArgs& a, int sm, cudaStream_t st) {
  static bool attr = false;
  if (!attr) {
    const cudaError_t e = cudaFuncSetAttribute(vae::conv_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               vae::Cfg<BN>::kSmemBytes);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  const int grid = std::min(a.total_tiles, sm);
  vae::conv_kernel<BN><<<grid, vae::kThreads, vae::Cfg<BN>::kSmemBytes, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_strip(const vae::ConvArgs& a, int sm, cudaStream_t st) {
  static bool attr = false;
  if (!attr) {
    const cudaError_t e = cudaFuncSetAttribute(vae::strip_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               vae::StripCfg::kSmemBytes);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  vae::strip_kernel<<<std::min(a.total_tiles, sm), vae::kThreads, vae::StripCfg::kSmemBytes, st>>>(a);
  return cudaGetLastError();
}

}  // namespace
}  // namespace fb

using namespace fb;

extern "C" {

int32_t fb_vae_conv(const float* in, int64_t ld_in, int32_t batch, int32_t h, int32_t w, int32_t cin, const float* weight,
                    int64_t ld_w, int32_t cout, int32_t ksize, const float* bias, const float* resid, int64_t ld_resid,
                    float* out, int64_t ld_out, int32_t flags, void* stream) {
  std::string err;
  DeviceState* d = current_device(err);
  if (!d) return fail(FB_ERR_INIT, "fb_vae_conv: " + err);
  if (batch <= 0 || h <= 0 || w <= 0 || cin <= 0 || cin % 32 != 0 || cout <= 0 || (ksize != 1 && ksize != 3))
    return fail(FB_ERR_ARG, "fb_vae_conv: need batch, h, w > 0, cin % 32 == 0, cout > 0 and ksize 1 or 3");
  if (flags & ~(vae::kRoundOut | vae::kOutNchwClamp)) return fail(FB_ERR_ARG, "fb_vae_conv: unknown flags");
  if (!in || !weight || !out) return fail(FB_ERR_ARG, "fb_vae_conv: null in/weight/out");
  const bool nchw = flags & vae::kOutNchwClamp;
  if (ld_in < cin || ld_in % 4 || ld_w < cin || ld_w % 4 || (!nchw && ld_out < cout) ||
      (resid && (nchw || ld_resid < cout)))
    return fail(FB_ERR_ARG, "fb_vae_conv: in/weight strides multiples of 4, strides covering the rows, no resid "
                            "with the NCHW output");
  if (!aligned(in, 16) || !aligned(weight, 16) || !aligned(out, 16) || (resid && !aligned(resid, 16)) ||
      (bias && !aligned(bias, 4)))
    return fail(FB_ERR_ALIGN, "fb_vae_conv: in/weight/out/resid must be 16-byte aligned");
  vae::ConvArgs a;
  std::memset(&a, 0, sizeof(a));
  // the strip kernel: 3x3, rows of at least 128 pixels, whole 128-channel output blocks
  const bool strip = ksize == 3 && w >= 128 && cout % vae::StripCfg::BN == 0;
  int tw = 1;
  while (tw < w && tw < 16) tw <<= 1;
  a.tw = strip ? 128 : tw;
  a.th = strip ? 2 : vae::BM / tw;
  const int bn = strip ? vae::StripCfg::BN : (cout >= 256 ? 256 : (cout > 64 ? 128 : (cout > 16 ? 64 : 16)));
  {
    const cuuint64_t dims[4] = {static_cast<cuuint64_t>(cin), static_cast<cuuint64_t>(w), static_cast<cuuint64_t>(h),
                                static_cast<cuuint64_t>(batch)};
    const cuuint64_t strides[3] = {static_cast<cuuint64_t>(ld_in) * 4, static_cast<cuuint64_t>(ld_in) * 4 * w,
                                   static_cast<cuuint64_t>(ld_in) * 4 * w * h};
    const cuuint32_t box[4] = {32, static_cast<cuuint32_t>(strip ? vae::StripCfg::kARows : a.tw),
                               static_cast<cuuint32_t>(strip ? 1 : a.th), 1};
    if (int rc = encode(&a.tma_in, 4, in, dims, strides, box, err)) return fail(rc, "fb_vae_conv input map: " + err);
  }
  {
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(cin), static_cast<cuuint64_t>(cout),
                                static_cast<cuuint64_t>(ksize) * ksize};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld_w) * 4, static_cast<cuuint64_t>(ld_w) * 4 * cout};
    const cuuint32_t box[3] = {32, static_cast<cuuint32_t>(bn), strip ? 3u : 1u};
    if (int rc = encode(&a.tma_w, 3, weight, dims, strides, box, err)) return fail(rc, "fb_vae_conv weight map: " + err);
  }
  a.bias = bias;
  a.resid = resid;
  a.out = out;
  a.ld_resid = ld_resid;
  a.ld_out = ld_out;
  a.batch = batch;
  a.H = h;
  a.W = w;
  a.cin = cin;
  a.cout = cout;
  a.R = ksize;
  a.tiles_w = (w + a.tw - 1) / a.tw;
  a.tiles_h = (h + a.th - 1) / a.th;
  a.n_tiles = (cout + bn - 1) / bn;
  const int64_t tiles = static_cast<int64_t>(batch) * a.tiles_w * a.tiles_h * a.n_tiles;
  if (tiles > (1ll << 30)) return fail(FB_ERR_ARG, "fb_vae_conv: too many tiles");
  a.total_tiles = static_cast<int>(tiles);
  a.kb_per_tap = cin / 32;
  a.num_kb = ksize * ksize * a.kb_per_tap;
  a.flags = flags | ((ld_out % 4 || (resid && ld_resid % 4)) ? vae::kScalarIo : 0);
  a.status = d->status;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (strip) {
    e = launch_strip(a, d->sm_count, st);
  } else {
    switch (bn) {
      case 256: e = launch_conv_bn<256>(a, d->sm_count, st); break;
      case 128: e = launch_conv_bn<128>(a, d->sm_count, st); break;
      case 64: e = launch_conv_bn<64>(a, d->sm_count, st); break;
      default: e = launch_conv_bn<16>(a, d->sm_count, st); break;
    }
  }
  return e == cudaSuccess ? FB_OK : fail(FB_ERR_CUDA, std::string("fb_vae_conv: ") + cudaGetErrorString(e));
}

// GroupNorm statistics of x into work: fp64 partials, then [batch][32][mean, rstd] floats (returned).
static const float* gn_statistics(const float* x, int64_t ld, int batch, int64_t hw, int c, float eps, double* work,
                                  cudaStream_t st, int& parts) {
  // about 16 pixels per thread per kernel: 8 blocks per SM over the batch
  const int lanes = vae::kGnThreads / (c / 4);
  const int64_t want = std::max<int64_t>(1, (8 * kNumSms + batch - 1) / batch);
  parts = static_cast<int>(std::min<int64_t>({static_cast<int64_t>(vae::kGnBlocksPerImage), want,
                                              (hw + lanes - 1) / lanes}));
  double* partial = work;
  float* stats = reinterpret_cast<float*>(work + static_cast<int64_t>(batch) * parts * 64);
  vae::gn_stats_kernel<<<dim3(parts, batch), vae::kGnThreads, 0, st>>>(x, hw, c, ld, partial);
  vae::gn_finish_kernel<<<batch, 1024, 0, st>>>(partial, parts, static_cast<double>(hw) * (c / 32), eps, stats);
  return stats;
}

int32_t fb_vae_group_norm(const float* x, int64_t ld, int32_t batch, int64_t hw, int32_t c, const float* gamma,
                          const float* beta, float eps, int32_t silu, int32_t round_tf32, float* out, int64_t ld_out,
                          double* work, void* stream) {
  std::string err;
  if (!current_device(err)) return fail(FB_ERR_INIT, "fb_vae_group_norm: " + err);
  if (batch <= 0 || hw <= 0 || (c != 128 && c != 256 && c != 512 && c != 1024))
    return fail(FB_ERR_ARG, "fb_vae_group_norm: c must be 128, 256, 512 or 1024 (32 groups of >= 4 channels)");
  if (ld < c || ld % 4 || ld_out < c || ld_out % 4 || !x || !gamma || !beta || !out || !work)
    return fail(FB_ERR_ARG, "fb_vae_group_norm: bad strides or null pointer");
  if (!aligned(x, 16) || !aligned(out, 16) || !aligned(gamma, 16) || !aligned(beta, 16) || !aligned(work, 8))
    return fail(FB_ERR_ALIGN, "fb_vae_group_norm: x/out/gamma/beta must be 16-byte aligned");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  int parts = 0;
  const float* stats = gn_statistics(x, ld, batch, hw, c, eps, work, st, parts);
  vae::gn_apply_kernel<<<dim3(parts, batch), vae::kGnThreads, 0, st>>>(x, hw, c, ld, stats, gamma, beta, out, ld_out,
                                                                        silu, round_tf32);
  return launched("fb_vae_group_norm");
}

int32_t fb_vae_norm_out_conv(const float* x, int32_t batch, int32_t h, int32_t w, int32_t c, const float* gamma,
                             const float* beta, float eps, const float* weight, const float* bias, int32_t cout,
                             float* out, double* work, void* stream) {
  std::string err;
  if (!current_device(err)) return fail(FB_ERR_INIT, "fb_vae_norm_out_conv: " + err);
  if (c != 128 || cout != 3)
    return fail(FB_ERR_UNSUPPORTED, "fb_vae_norm_out_conv: built for 128 input and 3 output channels (FLUX's conv_out)");
  if (batch <= 0 || h <= 0 || w <= 0 || !x || !gamma || !beta || !weight || !out || !work)
    return fail(FB_ERR_ARG, "fb_vae_norm_out_conv: need positive sizes and non-null pointers");
  if (!aligned(x, 16) || !aligned(gamma, 16) || !aligned(beta, 16) || !aligned(work, 8))
    return fail(FB_ERR_ALIGN, "fb_vae_norm_out_conv: x, gamma, beta must be 16-byte aligned");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  int parts = 0;
  const float* stats = gn_statistics(x, c, batch, static_cast<int64_t>(h) * w, c, eps, work, st, parts);
  const dim3 grid((w + vae::kNcTW - 1) / vae::kNcTW, (h + vae::kNcTH - 1) / vae::kNcTH, batch);
  vae::gn_conv_out_kernel<<<grid, vae::kNcThreads, 0, st>>>(x, h, w, stats, gamma, beta, weight, bias, out);
  return launched("fb_vae_norm_out_conv");
}

int64_t fb_vae_group_norm_work_doubles(int32_t batch) {
  return static_cast<int64_t>(batch) * vae::kGnBlocksPerImage * 64 + static_cast<int64_t>(batch) * 32 + 2;
}

int32_t fb_vae_upsample2(const float* in, int32_t batch, int32_t h, int32_t w, int32_t c, int32_t round_tf32, float* out,
                         void* stream) {
  std::string err;
  if (!current_device(err)) return fail(FB_ERR_INIT, "fb_vae_upsample2: " + err);
  if (batch <= 0 || h <= 0 || w <= 0 || c <= 0 || c % 4 || c > 1024 || 256 % (c / 4) || !in || !out)
    return fail(FB_ERR_ARG, "fb_vae_upsample2: need positive sizes, c a power of two in [4, 1024]");
  if (!aligned(in, 16) || !aligned(out, 16)) return fail(FB_ERR_ALIGN, "fb_vae_upsample2: 16-byte aligned in/out");
  const int64_t pix = static_cast<int64_t>(batch) * h * w;
  const int64_t lanes = 256 / (c / 4);
  const int blocks = static_cast<int>(std::min<int64_t>((pix + lanes - 1) / lanes, 16 * kNumSms));
  vae::upsample2_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const float4*>(in), pix, w, c / 4, reinterpret_cast<float4*>(out), round_tf32);
  return launched("fb_vae_upsample2");
}

int32_t fb_vae_softmax_rows(float* s, int64_t rows, int32_t n, int64_t ld, float scale, int32_t round_tf32,
                            void* stream) {
  std::string err;
  if (!current_device(err)) return fail(FB_ERR_INIT, "fb_vae_softmax_rows: " + err);
  if (rows < 0 || n <= 0 || n > vae::kSmThreads * 4 * vae::kSmMaxPer || ld < (n + 3) / 4 * 4 || ld % 4 || !s)
    return fail(FB_ERR_ARG, "fb_vae_softmax_rows: need 0 < n <= 32768, ld >= n rounded up to 4, ld % 4 == 0");
  if (rows > 0x7fffffff) return fail(FB_ERR_ARG, "fb_vae_softmax_rows: too many rows");
  if (!aligned(s, 16)) return fail(FB_ERR_ALIGN, "fb_vae_softmax_rows: 16-byte aligned");
  if (rows == 0) return FB_OK;
  const int per = (n + 4 * vae::kSmThreads - 1) / (4 * vae::kSmThreads);  // float4 per thread
  const dim3 grid(static_cast<unsigned>(rows));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (per <= 1) vae::softmax_rows_kernel<1><<<grid, vae::kSmThreads, 0, st>>>(
      s, n, ld, scale, round_tf32);
  else if (per <= 2) vae::softmax_rows_kernel<2><<<grid, vae::kSmThreads, 0, st>>>(
      s, n, ld, scale, round_tf32);
  else if (per <= 4) vae::softmax_rows_kernel<4><<<grid, vae::kSmThreads, 0, st>>>(
      s, n, ld, scale, round_tf32);
  else if (per <= 8) vae::softmax_rows_kernel<8><<<grid, vae::kSmThreads, 0, st>>>(
      s, n, ld, scale, round_tf32);
  else vae::softmax_rows_kernel<16><<<grid, vae::kSmThreads, 0, st>>>(
      s, n, ld, scale, round_tf32);
  return launched("fb_vae_softmax_rows");
}

int32_t fb_vae_transpose(const float* in, int32_t rows, int32_t cols, int64_t ld_in, float* out, int64_t ld_out,
                         void* stream) {
  std::string err;
  if (!current_device(err)) return fail(FB_ERR_INIT, "fb_vae_transpose: " + err);
  if (rows <= 0 || cols <= 0 || ld_in < cols || ld_out < rows || !in || !out)
    return fail(FB_ERR_ARG, "fb_vae_transpose: bad shape");
  const dim3 grid((cols + 31) / 32, (rows + 31) / 32);
  vae::transpose_kernel<<<grid, dim3(32, 8), 0, static_cast<cudaStream_t>(stream)>>>(in, rows, cols, ld_in, out, ld_out);
  return launched("fb_vae_transpose");
}

int32_t fb_vae_latent_prep(const float* z, int32_t batch, int32_t zc, int32_t h, int32_t w, int32_t cpad, float scale,
                           float shift, float* out, void* stream) {
  std::string err;
  if (!current_device(err)) return fail(FB_ERR_INIT, "fb_vae_latent_prep: " + err);
  if (batch <= 0 || zc <= 0 || h <= 0 || w <= 0 || cpad < zc || !z || !out)
    return fail(FB_ERR_ARG, "fb_vae_latent_prep: bad shape");
  const int64_t n = static_cast<int64_t>(batch) * h * w * cpad;
  const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 8 * kNumSms));
  vae::latent_prep_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(z, batch, zc, h, w, cpad, scale, shift,
                                                                                  out);
  return launched("fb_vae_latent_prep");
}

}  // extern "C"
