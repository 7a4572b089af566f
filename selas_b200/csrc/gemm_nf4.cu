// gemm_nf4.cu — tcgen05 GEMM whose weight operand is stored compressed and decoded inside the mainloop,
// tile by tile, into the shared-memory operand of the MMA. The bf16 weight never exists in global
// memory. Two storage formats of selas's containers (FMT):
//
//   NF4       W[n, 2i] = bf16(code[p >> 4] * absmax), W[n, 2i+1] = bf16(code[p & 15] * absmax)
//             (p = packed byte (n * K + 2i) / 2, absmax = absmax[(n * K + 2i) / 64]; one fp32 multiply,
//             then a round-to-nearest-even cast: bit-identical to fb_nf4_dequant's output and to
//             selas/codecs.py:178-199)
//   int8_row  W[n, k] = bf16(float(q[n, k]) * float(bf16(scale[n]))) (selas/codecs.py:272-276)
//   fp8 raw   W[n, k] = bf16(f8[n, k]), e4m3fn or e5m2, exact (selas keeps fp8 sources raw and casts them
//             at use: convert.py:178-180, codecs.py:270-271)
//
//   y[m, n] = sum_k X[m, k] W[n, k] (+ bias[n])
//
// The structure is that of the CTA-pair bf16 GEMM (gemm_pair.cu): one tcgen05.mma.cta_group::2 per
// K=16 step computes a 256-token x 256-feature tile on two SMs; each CTA loads its 128 token rows of
// X with TMA, and each CTA's TMEM holds its 128 rows of the accumulator (256 fp32 columns,
// double-buffered), which the fused FLUX epilogues of gemm_common.cuh consume. The difference is the
// W operand: instead of a TMA load of bf16 rows, converter warps in each CTA turn the CTA's 128 stored
// W rows of the K step (loaded by TMA: 4 KB of NF4, 8 KB of int8 or fp8) into the 16 KB bf16 tile in the
// 128-byte-swizzled K-major layout the MMA reads.
//
// Warps (512 threads per CTA, four warpgroups with their own register budgets via setmaxnreg):
//   warps 0..3   epilogue (184 registers): one accumulator row (token) per thread; the gated
//                residual uses the lean form of gemm_common.cuh (no residual prefetch)
//   warp 4       TMA (104 registers, with warps 5-7): the X box and the packed W box of each K step
//   warp 5       TMEM allocator; in the leader, the MMA issuer (4 MMAs of K=16 per K step)
//   warps 6, 7   idle
//   warps 8..15  NF4 converters (112 registers), two warpgroups taking alternate K steps: one W row per
//                thread; the row's 64 weights of a K step share one absmax, so the thread builds that
//                block's 16 bf16 products once and looks the 64 nibbles up with byte permutes in
//                registers (no shared-memory lookup), then writes the 128-byte row of the W tile
//
// Synchronisation (every cross-CTA signal names its one target barrier; no broadcast loads):
//   x_full[s]    leader: both CTAs' X loads of stage s complete on it (TMA, cta_group::2)
//   w_full[s]    leader: the 4 converter warps of each CTA arrive on it after fence.proxy.async
//   empty[s]     each CTA: the leader's MMA commits to both after reading stage s; the TMA warp and
//                the converters of each CTA wait on it before refilling the X and W halves
//   p_full/p_empty  each CTA: the packed-W ring between its TMA warp and its converters
//   acc_full[a]  each CTA: the leader commits to both when accumulator a is complete
//   acc_empty[a] leader: the 4 epilogue warps of each CTA arrive on it
//   rfull[w]     each CTA (NF4 gated residual): epilogue warp w's residual box landed in its 4 KB buffer
// Every wait is bounded (fb_common.cuh).
//
// Requirements (checked on the host): N % 32 == 0; NF4: K % 256 == 0 (whole float4 groups of absmax
// per row), blocksize 64, 16-byte aligned absmax; int8_row and fp8: K % 64 == 0.
#include "gemm_common.cuh"

namespace fb {
namespace gemm_nf4 {

using namespace gemm;

constexpr int BM = 256;  // tokens per pair tile (128 loaded by each CTA)
constexpr int BN = 256;  // W rows per pair tile (128 decoded by each CTA)
constexpr int kThreads = 512;
// setmaxnreg budgets per warpgroup; their sum times 128 threads must stay within the 128 x 512
// registers the block is launched with (the kernel is compiled to exactly 128 per thread).
constexpr uint32_t kRegEpi = 184, kRegCtl = 104, kRegConv = 112;
constexpr int kLaunchRegs = 128;
static_assert((kRegEpi + kRegCtl + 2 * kRegConv) * 128 <= kLaunchRegs * kThreads, "register split exceeds the launch budget");
constexpr int kStages = 5;   // X + W operand stages
constexpr int kPStages = 8;  // packed W stages
constexpr int kXBytes = 128 * BK * 2;  // 16 KB
constexpr int kWBytes = 128 * BK * 2;  // 16 KB
constexpr int kFmtNf4 = 1, kFmtInt8 = 2, kFmtFp8 = 3;  // weight formats (fb_linear: w_nf4 / w_i8 / w_f8)
// one K step of the CTA's 128 W rows as stored: NF4 32 bytes per row, int8_row and fp8 64 bytes per row
template <int FMT>
constexpr int packed_bytes() { return FMT == kFmtNf4 ? 128 * BK / 2 : 128 * BK; }
constexpr uint32_t kTmemCols = 512;
constexpr int kNumBars = 3 * kStages + 2 * kPStages + 2 + 2 + 1;
// The gated residual of NF4 weights takes the residual by TMA, one 4 KB box per epilogue warp
// (resid_row_tma); int8_row and fp8, whose packed ring is twice as large, leave no room for it and use
// the lean epilogue, which loads the residual straight from global memory.
template <int EPI, int FMT>
constexpr bool tma_resid() {
  return EPI == FB_EPI_GATED_RESIDUAL && FMT == kFmtNf4;
}
template <int EPI, int FMT>
constexpr int smem_bytes() {
  return kStages * (kXBytes + kWBytes) + kPStages * packed_bytes<FMT>() + (tma_resid<EPI, FMT>() ? 4 * kResidBoxBytes : 0) +
         kNumBars * 8 + 16 + 4 * 8 + 1024;
}
constexpr uint32_t kIdesc = idesc_bf16_f32(256, BN, false);

__device__ __forceinline__ uint64_t mul_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__device__ __forceinline__ uint64_t add_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__device__ __forceinline__ uint64_t pack_f32x2(float lo, float hi) {
  return (static_cast<uint64_t>(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
}

// Decode the 64 weights of one row and K step (32 packed bytes in w, one absmax block s) into 32 bf16
// pairs: o[j] = bf16(code[e_2j] * s) | bf16(code[e_2j+1] * s) << 16.
//
// The 16 possible products are computed once (8 packed FP32x2 multiplies, 8 RNE conversions) and
// split into byte planes: LB[r] holds the low bytes of entries 4r..4r+3, HB[r] the high bytes. A byte
// permute selects, for four nibbles at once, among 8 entries (two plane registers); two permutes cover
// entries 0-7 and 8-15, and a third picks per byte by the nibble's top bit. The nibbles of a 16-bit
// half-word come in the order (e1, e0, e3, e2) (high nibble = even element), which the final
// interleaving permutes undo. Every selector has bit 3 of each nibble clear.
__device__ __forceinline__ void decode_row64(const uint32_t (&w)[8], float s, const float (&c)[16],
                                             uint32_t (&o)[32]) {
  const uint64_t s2 = pack_f32x2(s, s);
  uint32_t t[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint64_t p = mul_f32x2(pack_f32x2(c[2 * j], c[2 * j + 1]), s2);
    t[j] = pack_bf16x2(__uint_as_float(static_cast<uint32_t>(p)), __uint_as_float(static_cast<uint32_t>(p >> 32)));
  }
  uint32_t lb[4], hb[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    lb[r] = __byte_perm(t[2 * r], t[2 * r + 1], 0x6420);
    hb[r] = __byte_perm(t[2 * r], t[2 * r + 1], 0x7531);
  }
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    const uint32_t s7 = w[g] & 0x77777777u;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t sel = h ? (s7 >> 16) : s7;
      const uint32_t pick = ((w[g] >> (1 + 16 * h)) & 0x4444u) | 0x3210u;
      const uint32_t rl = __byte_perm(__byte_perm(lb[0], lb[1], sel), __byte_perm(lb[2], lb[3], sel), pick);
      const uint32_t rh = __byte_perm(__byte_perm(hb[0], hb[1], sel), __byte_perm(hb[2], hb[3], sel), pick);
      o[4 * g + 2 * h] = __byte_perm(rl, rh, 0x4051);
      o[4 * g + 2 * h + 1] = __byte_perm(rl, rh, 0x6273);
    }
  }
}

// Decode the 64 int8 weights of one row and K step (16 words, little-endian bytes = consecutive k)
// with the row's scale s = float(bf16(scale)): o[j] = bf16(float(q_2j) * s) | bf16(float(q_2j+1) * s)
// << 16. An int8 becomes an exact float by placing (q + 128) in the mantissa of 2^23 (byte permute)
// and subtracting 2^23 + 128; the product of an 8-bit integer and a bf16 is exact in fp32, so the
// final RNE cast is the only rounding, as in selas's q.to(bf16) * scale.to(bf16) (codecs.py:272-276).
__device__ __forceinline__ void decode_row64_i8(const uint32_t (&w)[16], float s, uint32_t (&o)[32]) {
  const uint64_t s2 = pack_f32x2(s, s);
  const uint64_t bias2 = pack_f32x2(-8388736.0f, -8388736.0f);
#pragma unroll
  for (int u = 0; u < 16; ++u) {
    const uint32_t x = w[u] ^ 0x80808080u;
    const uint64_t lo = pack_f32x2(__uint_as_float(__byte_perm(x, 0x4B000000u, 0x7540)),
                                   __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7541)));
    const uint64_t hi = pack_f32x2(__uint_as_float(__byte_perm(x, 0x4B000000u, 0x7542)),
                                   __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7543)));
    const uint64_t a = mul_f32x2(add_f32x2(lo, bias2), s2);
    const uint64_t b = mul_f32x2(add_f32x2(hi, bias2), s2);
    o[2 * u] = pack_bf16x2(__uint_as_float(static_cast<uint32_t>(a)), __uint_as_float(static_cast<uint32_t>(a >> 32)));
    o[2 * u + 1] = pack_bf16x2(__uint_as_float(static_cast<uint32_t>(b)), __uint_as_float(static_cast<uint32_t>(b >> 32)));
  }
}

// Decode the 64 fp8 weights of one row and K step (16 words, little-endian bytes = consecutive k) to bf16
// pairs: the hardware conversion of two fp8 values to f16x2 is exact (e4m3fn and e5m2 both fit f16),
// and so is f16 -> f32 -> bf16 (at most 3 mantissa bits, exponents inside bf16's range).
template <bool E5M2>
__device__ __forceinline__ uint32_t fp8x2_to_bf16x2(uint32_t two) {
  uint32_t h;
  if constexpr (E5M2) {
    asm("{\n\t.reg .b16 t;\n\tcvt.u16.u32 t, %1;\n\tcvt.rn.f16x2.e5m2x2 %0, t;\n\t}" : "=r"(h) : "r"(two));
  } else {
    asm("{\n\t.reg .b16 t;\n\tcvt.u16.u32 t, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, t;\n\t}" : "=r"(h) : "r"(two));
  }
  const __half2 hv = *reinterpret_cast<const __half2*>(&h);
  const float2 f = __half22float2(hv);
  return pack_bf16x2(f.x, f.y);
}

template <bool E5M2>
__device__ __forceinline__ void decode_row64_f8(const uint32_t (&w)[16], uint32_t (&o)[32]) {
#pragma unroll
  for (int u = 0; u < 16; ++u) {
    o[2 * u] = fp8x2_to_bf16x2<E5M2>(w[u] & 0xFFFFu);
    o[2 * u + 1] = fp8x2_to_bf16x2<E5M2>(w[u] >> 16);
  }
}

// Work item w: tile w % total_tiles, the K steps [kb0, kb1) of split w / total_tiles (every problem's
// K steps divide into args.splits ranges of a multiple of 4 steps, the NF4 absmax group).
__device__ __forceinline__ void decode_work(const Args& a, int w, int& p, int& mb, int& nb, int& kb0, int& kb1) {
  const int split = w / a.total_tiles;
  decode_tile(a, w - split * a.total_tiles, p, mb, nb);
  const int per = a.prob[p].num_kb / a.splits;
  kb0 = split * per;
  kb1 = kb0 + per;
}

// Split-K completion of one CTA's 128 accumulator rows (the 4 epilogue warps, 128 threads): each split
// stores its fp32 partial rows; the CTA that arrives last for the tile (no CTA ever waits for another)
// sums all splits' partials in split order — the same order whichever arrives last, so the result is
// run-to-run deterministic — into its TMEM accumulator and runs the epilogue. Returns whether this CTA
// completes the tile.
__device__ __forceinline__ bool splitk_reduce(const Args& a, int w, uint32_t rank, int row, uint32_t trow,
                                              volatile int* last_flag) {
  const int tiles = a.total_tiles;
  const int tile = w % tiles;
  float* mine = a.splitk_ws + ((static_cast<int64_t>(w) * 2 + rank) * 128 + row) * BN;
#pragma unroll 1
  for (int c = 0; c < BN / 16; ++c) {  // 16 columns at a time: few live registers next to the epilogue
    uint32_t v[16];
    tmem_ld_32x32b_x16(trow + 16 * c, v);
    tmem_ld_wait();
    uint4* dst = reinterpret_cast<uint4*>(mine + 16 * c);
#pragma unroll
    for (int i = 0; i < 4; ++i) __stcg(dst + i, make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]));
  }
  __threadfence();
  asm volatile("bar.sync 8, 128;" ::: "memory");  // the CTA's 128 epilogue threads have stored
  if (row == 0) {
    int* cnt = a.splitk_count + tile * 2 + rank;
    const int old = atomicAdd(cnt, 1);
    const bool last = old == a.splits - 1;
    if (last) *cnt = 0;  // every split has arrived: ready for the next launch
    __threadfence();
    *last_flag = last ? 1 : 0;
  }
  asm volatile("bar.sync 8, 128;" ::: "memory");
  if (!*last_flag) return false;
#pragma unroll 1
  for (int c = 0; c < BN / 16; ++c) {
    float acc[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) acc[j] = 0.f;
#pragma unroll 1
    for (int sp = 0; sp < a.splits; ++sp) {
      const uint4* src = reinterpret_cast<const uint4*>(
          a.splitk_ws + ((static_cast<int64_t>(sp * tiles + tile) * 2 + rank) * 128 + row) * BN + 16 * c);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 u = __ldcg(src + i);
        acc[4 * i] += __uint_as_float(u.x);
        acc[4 * i + 1] += __uint_as_float(u.y);
        acc[4 * i + 2] += __uint_as_float(u.z);
        acc[4 * i + 3] += __uint_as_float(u.w);
      }
    }
    uint32_t o[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j] = __float_as_uint(acc[j]);
    tmem_st_32x32b_x16(trow + 16 * c, o);
  }
  tmem_st_wait();
  return true;
}

template <int EPI, int FMT>
__global__ void __launch_bounds__(kThreads, 1) gemm_nf4_kernel(const __grid_constant__ Args args) {
  constexpr int kPBytes = packed_bytes<FMT>();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sX = smem;                         // kStages x 16 KB token rows
  uint8_t* sW = sX + kStages * kXBytes;       // kStages x 16 KB decoded W rows
  uint8_t* sPk = sW + kStages * kWBytes;      // kPStages x 4 KB packed W rows
  uint8_t* sR = sPk + kPStages * kPBytes;     // residual boxes, one per epilogue warp (tma_resid only)
  uint64_t* x_full = reinterpret_cast<uint64_t*>(sR + (tma_resid<EPI, FMT>() ? 4 * kResidBoxBytes : 0));
  uint64_t* w_full = x_full + kStages;
  uint64_t* empty = w_full + kStages;
  uint64_t* p_full = empty + kStages;
  uint64_t* p_empty = p_full + kPStages;
  uint64_t* acc_full = p_empty + kPStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* split_last = abort_flag + 1;  // split-K: this CTA completes the current tile
  uint64_t* rfull = reinterpret_cast<uint64_t*>(tmem_slot + 4);  // [epilogue warp]: its residual box landed
  const int total_work = args.total_tiles * args.splits;

  const int warp = warp_id();
  const int lane = lane_id();
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&x_full[s], 1);
      mbar_init(&w_full[s], 8);  // 4 converter warps in each CTA
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < kPStages; ++s) {
      mbar_init(&p_full[s], 1);
      mbar_init(&p_empty[s], 128);  // every thread of the converter warpgroup that took the K step
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 8);  // 4 epilogue warps in each CTA
    }
    mbar_init(drain, 1);
    if constexpr (tma_resid<EPI, FMT>()) {
      for (int w = 0; w < 4; ++w) mbar_init(&rfull[w], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 4 && lane == 0) {
    for (int p = 0; p < args.nprob; ++p) {
      tma_prefetch_desc(&args.prob[p].tma_a);
      tma_prefetch_desc(&args.prob[p].tma_b);
      if constexpr (tma_resid<EPI, FMT>()) tma_prefetch_desc(&args.prob[p].tma_resid);
    }
  }
  if (warp == 5) {
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
  const int wg = warp >> 2;
  if (wg == 0) {
    reg_alloc<kRegEpi>();
  } else if (wg == 1) {
    reg_dealloc<kRegCtl>();
  } else {
    reg_dealloc<kRegConv>();
  }

  if (warp == 4) {
    // ------------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int xs = 0, ps = 0;
      uint32_t xph = 0, pph = 0;
      uint32_t x_issued[kStages], p_issued[kPStages];
      for (int s = 0; s < kStages; ++s) x_issued[s] = 0xFFFFFFFFu;
      for (int s = 0; s < kPStages; ++s) p_issued[s] = 0xFFFFFFFFu;
      bool ok = true;
      for (int w = pair; ok && w < total_work; w += npairs) {
        int p, mb, nb, kb0, kb1;
        decode_work(args, w, p, mb, nb, kb0, kb1);
        const Problem& P = args.prob[p];
        for (int kb = kb0; kb < kb1; ++kb) {
          // packed W first: the converters run ahead of the MMA by up to kStages K steps
          if (!mbar_wait(&p_empty[ps], pph ^ 1u, abort_flag, args.status, FB_DEV_TIMEOUT_EPI)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&p_full[ps], kPBytes);
          tma_load_2d(&P.tma_b, &p_full[ps], sPk + ps * kPBytes, kb * (kPBytes / 128), nb * BN + 128 * static_cast<int>(rank));
          p_issued[ps] = pph;
          if (++ps == kPStages) {
            ps = 0;
            pph ^= 1u;
          }
          if (!mbar_wait(&empty[xs], xph ^ 1u, abort_flag, args.status, FB_DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&x_full[xs], 2 * kXBytes);
          tma_load_2d_pair(&P.tma_a, mapa_shared(smem_u32(&x_full[xs]), 0), sX + xs * kXBytes, kb * BK,
                           mb * BM + 128 * static_cast<int>(rank));
          x_issued[xs] = xph;
          if (++xs == kStages) {
            xs = 0;
            xph ^= 1u;
          }
        }
      }
      if (!ok) {
        // let every issued load land (bounded) before the CTA can leave: the packed loads complete on
        // this CTA's barriers, the X loads of both CTAs on the leader's
        for (int s = 0; s < kPStages; ++s)
          if (p_issued[s] != 0xFFFFFFFFu) mbar_wait_quiet(&p_full[s], p_issued[s], kWaitBudgetNs);
        if (leader)
          for (int s = 0; s < kStages; ++s)
            if (x_issued[s] != 0xFFFFFFFFu) mbar_wait_quiet(&x_full[s], x_issued[s], kWaitBudgetNs);
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------------ MMA issuer (leader only)
    if (lane == 0 && leader) {
      int s = 0, acc = 0;
      uint32_t ph = 0, acc_phase = 0;
      bool ok = true;
      for (int w = pair; ok && w < total_work; w += npairs) {
        int p, mb, nb, kb0, kb1;
        decode_work(args, w, p, mb, nb, kb0, kb1);
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, abort_flag, args.status, FB_DEV_TIMEOUT_EPI)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          ok = mbar_wait(&x_full[s], ph, abort_flag, args.status, FB_DEV_TIMEOUT_TMA) &&
               mbar_wait(&w_full[s], ph, abort_flag, args.status, FB_DEV_TIMEOUT_EPI);
          if (!ok) break;
          tc_fence_after_sync();
          const uint32_t x0 = smem_u32(sX + s * kXBytes);
          const uint32_t w0 = smem_u32(sW + s * kWBytes);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_bf16_ss_pair(d_tmem, sdesc_kmajor_sw128(x0 + 32 * k), sdesc_kmajor_sw128(w0 + 32 * k), kIdesc,
                              (kb > kb0 || k > 0) ? 1u : 0u);
          const uint32_t e = smem_u32(&empty[s]);
          umma_commit_pair_both(e);
          if (++s == kStages) {
            s = 0;
            ph ^= 1u;
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
  } else if (warp < 4) {
    // ------------------------------------------------------------------ epilogue (warps 0..3, both CTAs)
    const int quarter = warp;
    const int row_in_tile = quarter * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    uint32_t rphase = 0;
    if (args.splits == 1) {
      for (int w = pair; w < total_work; w += npairs) {
        int p, mb, nb;
        decode_tile(args, w, p, mb, nb);
        const Problem& P = args.prob[p];
        if (!mbar_wait(&acc_full[acc], acc_phase, abort_flag, args.status, FB_DEV_TIMEOUT_MMA)) break;
        tc_fence_after_sync();
        const uint32_t trow = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
        const int m = mb * BM + 128 * static_cast<int>(rank) + row_in_tile;
        if constexpr (tma_resid<EPI, FMT>()) {
          const int row0 = mb * BM + 128 * static_cast<int>(rank) + quarter * 32;
          if (!resid_row_tma<BN, 2>(P, m, m < P.m, nb, trow, 0, BN / 32, row0, sR + quarter * kResidBoxBytes,
                                 &rfull[quarter], rphase, abort_flag, args.status)) {
            mbar_wait_quiet(&rfull[quarter], rphase, kWaitBudgetNs);  // the box in flight lands before the CTA exits
            break;
          }
        } else {
          epilogue_row<BN, EPI, true>(P, m, m < P.m, nb, trow);  // lean: fits the 184-register budget
        }
        tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(mapa_shared(smem_u32(&acc_empty[acc]), 0));
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    } else {
      // split-K: the CTA that completes a tile sums the splits into its accumulator, then the epilogue
      for (int w = pair; w < total_work; w += npairs) {
        if (!mbar_wait(&acc_full[acc], acc_phase, abort_flag, args.status, FB_DEV_TIMEOUT_MMA)) break;
        tc_fence_after_sync();
        const uint32_t trow = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
        if (splitk_reduce(args, w, rank, row_in_tile, trow, split_last)) {
          int p, mb, nb, kb0, kb1;
          decode_work(args, w, p, mb, nb, kb0, kb1);
          const Problem& P = args.prob[p];
          const int m = mb * BM + 128 * static_cast<int>(rank) + row_in_tile;
          epilogue_row<BN, EPI, true>(P, m, m < P.m, nb, trow);
        }
        tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(mapa_shared(smem_u32(&acc_empty[acc]), 0));
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
  } else if (warp >= 8) {
    // ------------------------------------------------------------------ NF4 converters (warps 8..15)
    // Warpgroup `set` takes the K steps of its parity. Every problem has a multiple of 4 K steps, so
    // the parity of a tile's K step equals that of this CTA's running K-step count gk, which also
    // indexes the operand stages (gk % kStages) and the packed ring (gk % kPStages).
    const uint32_t set = static_cast<uint32_t>(wg & 1);
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // the W row of the CTA's 128 this thread decodes
    const uint32_t swz = static_cast<uint32_t>(r & 7);
    uint32_t gk0 = 0;
    bool ok = true;
    for (int w = pair; ok && w < total_work; w += npairs) {
      int p, mb, nb, kb0, kb1;
      decode_work(args, w, p, mb, nb, kb0, kb1);
      const Problem& P = args.prob[p];
      const int n = nb * BN + 128 * static_cast<int>(rank) + r;
      const bool valid = n < P.n;
      float code[16];
      float s_row = 0.f;
      if constexpr (FMT == kFmtNf4) {
#pragma unroll
        for (int i = 0; i < 16; ++i) code[i] = __ldg(P.code16 + i);
      } else if constexpr (FMT == kFmtInt8) {
        s_row = valid ? bf16_round(__ldg(P.absmax + n)) : 0.f;  // int8_row: absmax holds the row scales
      }
      // NF4: absmax arrives four K steps at a time (one float4 per row), with the next group in flight
      const float4* am4 = reinterpret_cast<const float4*>(P.absmax + static_cast<int64_t>(n) * P.absmax_per_row);
      const float4 zero4 = make_float4(0.f, 0.f, 0.f, 0.f);
      float4 cur = zero4, nxt = zero4;
      int cur_g = kb0 >> 2;
      if constexpr (FMT == kFmtNf4) {
        cur = valid ? __ldg(am4 + cur_g) : zero4;
        nxt = (valid && 4 * (cur_g + 1) < kb1) ? __ldg(am4 + cur_g + 1) : zero4;
      }
      for (int kb = kb0 + static_cast<int>(set); kb < kb1; kb += 2) {
        const uint32_t gk = gk0 + static_cast<uint32_t>(kb - kb0);
        const uint32_t ps = gk & (kPStages - 1), pph = (gk / kPStages) & 1u;
        const uint32_t s = gk % kStages, ph = (gk / kStages) & 1u;
        uint32_t o[32];
        if constexpr (FMT == kFmtNf4) {
          const int g = kb >> 2;
          if (g != cur_g) {
            cur_g = g;
            cur = nxt;
            nxt = (valid && 4 * (g + 1) < kb1) ? __ldg(am4 + g + 1) : zero4;
          }
          const int q = kb & 3;
          const float s_cur = q == 0 ? cur.x : q == 1 ? cur.y : q == 2 ? cur.z : cur.w;
          if (!mbar_wait(&p_full[ps], pph, abort_flag, args.status, FB_DEV_TIMEOUT_TMA)) {
            ok = false;
            break;
          }
          // the row's 32 packed bytes as two 16-byte loads; threads 4-7 of every 8 take the halves in
          // the other order, so each load instruction touches all eight 16-byte bank groups once per 8 rows
          const uint8_t* pk = sPk + ps * kPBytes + r * 32;
          const uint32_t h0 = static_cast<uint32_t>((r >> 2) & 1) << 4;
          const uint4 wa = *reinterpret_cast<const uint4*>(pk + h0);
          const uint4 wb = *reinterpret_cast<const uint4*>(pk + (h0 ^ 16u));
          mbar_arrive(&p_empty[ps]);
          const uint4 w0 = h0 ? wb : wa;
          const uint4 w1 = h0 ? wa : wb;
          const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
          decode_row64(words, s_cur, code, o);
        } else {
          if (!mbar_wait(&p_full[ps], pph, abort_flag, args.status, FB_DEV_TIMEOUT_TMA)) {
            ok = false;
            break;
          }
          // the row's 64 bytes; the TMA wrote them with the 64-byte swizzle (16-byte chunk c of row r at
          // position c ^ ((r >> 1) & 3)), so reading chunk c touches all eight bank groups across a warp
          const uint8_t* pk = sPk + ps * kPBytes + r * 64;
          const uint32_t x = static_cast<uint32_t>((r >> 1) & 3);
          uint32_t words[16];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint4 v = *reinterpret_cast<const uint4*>(pk + ((static_cast<uint32_t>(c) ^ x) << 4));
            words[4 * c] = v.x;
            words[4 * c + 1] = v.y;
            words[4 * c + 2] = v.z;
            words[4 * c + 3] = v.w;
          }
          mbar_arrive(&p_empty[ps]);
          if constexpr (FMT == kFmtInt8) {
            decode_row64_i8(words, s_row, o);
          } else if (P.fp8_e5m2) {
            decode_row64_f8<true>(words, o);
          } else {
            decode_row64_f8<false>(words, o);
          }
        }
        // the MMA that last read stage s must be done before its W half is overwritten
        if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, args.status, FB_DEV_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        uint8_t* rowp = sW + s * kWBytes + r * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c)  // 16-byte chunk c of the row goes to position c ^ (row & 7)
          *reinterpret_cast<uint4*>(rowp + ((static_cast<uint32_t>(c) ^ swz) << 4)) =
              make_uint4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(mapa_shared(smem_u32(&w_full[s]), 0));
      }
      gk0 += static_cast<uint32_t>(kb1 - kb0);
    }
  }

  tc_fence_before_sync();
  __syncthreads();
  cluster_sync_all();  // the peer no longer signals this CTA and nobody reads this CTA's TMEM
  if (warp == 5) {
    tc_fence_after_sync();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

template <int EPI, int FMT>
static cudaError_t launch_t(const gemm::Args& args, int grid, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem_bytes<EPI, FMT>();
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemm_nf4_kernel<EPI, FMT>, args);
}

}  // namespace gemm_nf4

template <int EPI, int FMT>
static std::string setup_one() {
  // setmaxnreg.inc only completes if the block was launched with the registers the split assumes
  cudaFuncAttributes a;
  cudaError_t e = cudaFuncGetAttributes(&a, gemm_nf4::gemm_nf4_kernel<EPI, FMT>);
  if (e != cudaSuccess) return std::string("cudaFuncGetAttributes(gemm_nf4): ") + cudaGetErrorString(e);
  if (a.numRegs != gemm_nf4::kLaunchRegs)
    return "gemm_nf4: compiled to " + std::to_string(a.numRegs) + " registers per thread, the register split needs " +
           std::to_string(gemm_nf4::kLaunchRegs);
  e = cudaFuncSetAttribute(gemm_nf4::gemm_nf4_kernel<EPI, FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           gemm_nf4::smem_bytes<EPI, FMT>());
  return e == cudaSuccess ? std::string() : std::string("cudaFuncSetAttribute(gemm_nf4): ") + cudaGetErrorString(e);
}

template <int FMT>
static std::string setup_fmt() {
  for (const std::string& m : {setup_one<FB_EPI_STORE_BF16, FMT>(), setup_one<FB_EPI_STORE_F32, FMT>(),
                               setup_one<FB_EPI_GELU, FMT>(), setup_one<FB_EPI_GATED_RESIDUAL, FMT>(),
                               setup_one<FB_EPI_QKV, FMT>()})
    if (!m.empty()) return m;
  return std::string();
}

std::string gemm_nf4_setup() {
  std::string m = setup_fmt<gemm_nf4::kFmtNf4>();
  if (m.empty()) m = setup_fmt<gemm_nf4::kFmtInt8>();
  return m.empty() ? setup_fmt<gemm_nf4::kFmtFp8>() : m;
}

template <int FMT>
static cudaError_t launch_fmt(int epi, const gemm::Args& args, int grid, cudaStream_t st) {
  using namespace gemm_nf4;
  switch (epi) {
    case FB_EPI_STORE_BF16: return launch_t<FB_EPI_STORE_BF16, FMT>(args, grid, st);
    case FB_EPI_STORE_F32: return launch_t<FB_EPI_STORE_F32, FMT>(args, grid, st);
    case FB_EPI_GELU: return launch_t<FB_EPI_GELU, FMT>(args, grid, st);
    case FB_EPI_GATED_RESIDUAL: return launch_t<FB_EPI_GATED_RESIDUAL, FMT>(args, grid, st);
    default: return launch_t<FB_EPI_QKV, FMT>(args, grid, st);
  }
}

cudaError_t launch_gemm_decode(int wfmt, int epi, const gemm::Args& args, int grid, cudaStream_t st) {
  return wfmt == gemm_nf4::kFmtNf4    ? launch_fmt<gemm_nf4::kFmtNf4>(epi, args, grid, st)
         : wfmt == gemm_nf4::kFmtInt8 ? launch_fmt<gemm_nf4::kFmtInt8>(epi, args, grid, st)
                                      : launch_fmt<gemm_nf4::kFmtFp8>(epi, args, grid, st);
}

}  // namespace fb
