// attention.cu — flash-attention forward on tcgen05 for FLUX's joint attention (head_dim 128,
// non-causal, no mask): out[b, l, h*128 + d] = softmax(q k^T * scale) v, written straight into the
// token-major [B, L, H*128] layout the next Linear reads (no transpose copy).
//
// One CTA per (256 queries = two 128-row tiles A and B, head, image); 320 threads:
//   warp 0      TMA: Q_A and Q_B once; K_j and V_j (two slots each) per 128-key tile, 128-byte
//               swizzle, 3-D maps so a tile never reads past its own (image, head) rows. With one K
//               slot, K_{j+1} could only be fetched once S_B(j) had read K_j, and its L2 latency stood
//               between PV_A(j) and S_A(j+1); two slots fetch it a tile ahead.
//   warp 1      TMEM allocator + MMA issuer (one thread), ping-pong between the two tiles:
//                 S_A(0), S_B(0), then per KV tile j:  O_A += P_A V_j,  S_A(j+1),  O_B += P_B V_j,  S_B(j+1)
//               where O += P V is issued in two halves of 64 keys: the first as soon as the softmax has
//               stored P for keys 0..63, so it runs while the softmax works on keys 64..127.
//               S = Q K^T is M=128, N=128 keys, K=128; O += P V is M=128, N=128 dims, K=128 keys with V
//               as an MN-major operand. While one warpgroup runs its softmax the tensor core works on
//               the other tile.
//   warps 2..5  softmax of tile A, warps 6..9 softmax of tile B: thread = one query row (TMEM lane).
//               Reads S, masks keys >= L, keeps a running max in the log2 domain and rescales O (in
//               TMEM) only when the max grows by more than 8 (2^8 headroom), writes
//               P = exp2(s*scale*log2e - m) as bf16 pairs back into TMEM over the S columns it has
//               consumed (keys 2c, 2c+1 in column c), and finally writes O / l.
// O += P V reads P from TMEM (the A operand) and V from shared memory, so shared memory carries only
// Q, K and V. S(j+1) overwrites the P(j) columns only after O += P(j) V has read them: the MMA thread
// issues the two in that order, and tcgen05.mma operations from one thread execute in issue order.
// Waits are bounded (fb_common.cuh); the kernel returns with a status code instead of hanging.
#include "fb_internal.h"

namespace fb {
namespace attn {

constexpr int BQ = 128;           // queries per tile; a CTA owns two tiles (A, B)
constexpr int BKV = 128;          // keys per KV tile
constexpr int HD = 128;
constexpr int kRowsPerCta = 2 * BQ;
constexpr int kThreads = 320;     // warp 0 TMA, warp 1 MMA, warps 2-5 softmax A, warps 6-9 softmax B
constexpr int kTileBytes = 128 * HD * 2;  // 32 KB: one 128 x 128 bf16 tile (two 64-column boxes)
constexpr int kHalf = kTileBytes / 2;     // 16 KB: one 128-row x 64-column box
// shared memory: Q_A, Q_B, K[2], V[2] (6 tiles) + barriers + alignment slack
constexpr int kSmemBytes = 6 * kTileBytes + 256 + 1024;
constexpr uint32_t kIdescS = idesc_bf16_f32(128, 128, false);
constexpr uint32_t kIdescO = idesc_bf16_f32(128, 128, true);
constexpr uint32_t kTmemCols = 512;  // S_A [0,128), S_B [128,256), O_A [256,384), O_B [384,512)

struct Args {
  CUtensorMap tq, tk, tv;  // 3-D maps over [B*H, L, 128]
  uint16_t* out0;  // rows [0, split) of each image: out0[(b * split + l) * ld0 + h * 128 + d]
  int64_t ld0;
  uint16_t* out1;  // rows [split, seq): out1[(b * (seq - split) + l - split) * ld1 + h * 128 + d]
  int64_t ld1;
  int split;
  int seq, heads;
  float scale_log2;
  int* status;
  // sequence parallel (sp_world > 0, one image): row t of the gathered sequence belongs to rank
  // t / sp_ll, its local token t % sp_ll; it is stored to sp_out[t / sp_ll] + (t % sp_ll) * sp_ld +
  // sp_col0 + h * 128 (this rank's head group's columns of that rank's next-Linear input, over NVLink)
  uint16_t* sp_out[8];
  int sp_world, sp_ll, sp_col0;
  int64_t sp_ld;
};

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// --- packed FP32x2 arithmetic (two fp32 lanes in one 64-bit register, one instruction for both)
__device__ __forceinline__ uint64_t f2(float a, float b) {
  return static_cast<uint64_t>(__float_as_uint(a)) | (static_cast<uint64_t>(__float_as_uint(b)) << 32);
}
__device__ __forceinline__ float f2_lo(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v)); }
__device__ __forceinline__ float f2_hi(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v >> 32)); }
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x for a pair of lanes on the FMA pipe instead of the MUFU pipe, so that both pipes share the
// softmax's exponentials. Range reduction after Cody and Waite: x = j + f with j = round(x) (obtained
// by adding 1.5 * 2^23) and f in [-0.5, 0.5]; 2^f from a degree-4 polynomial fitted here by
// least squares on Chebyshev nodes (max relative error 2.7e-6, below the bf16 rounding of P);
// 2^j added to the exponent field. x is clamped at -126 so the result stays a normal float (a
// masked key then weighs 2^-126 instead of 0, far below anything bf16 P can carry next to the max).
__device__ __forceinline__ void exp2_poly_x2(uint64_t x, float& e0, float& e1) {
  x = f2(fmaxf(f2_lo(x), -126.f), fmaxf(f2_hi(x), -126.f));
  const uint64_t t = f2_add(x, f2(12582912.f, 12582912.f));
  const uint64_t j = f2_add(t, f2(-12582912.f, -12582912.f));
  const uint64_t f = f2_fma(j, f2(-1.f, -1.f), x);
  uint64_t p = f2_fma(f, f2(0.009570097550749779f, 0.009570097550749779f), f2(0.05591785907745361f, 0.05591785907745361f));
  p = f2_fma(p, f, f2(0.240247443318367f, 0.240247443318367f));
  p = f2_fma(p, f, f2(0.6931217908859253f, 0.6931217908859253f));
  p = f2_fma(p, f, f2(0.9999992847442627f, 0.9999992847442627f));
  const uint32_t tl = static_cast<uint32_t>(t), th = static_cast<uint32_t>(t >> 32);
  e0 = __uint_as_float(static_cast<uint32_t>(p) + ((tl - 0x4B400000u) << 23));
  e1 = __uint_as_float(static_cast<uint32_t>(p >> 32) + ((th - 0x4B400000u) << 23));
}

// Which of the 32 exponential pairs of a 64-key half take the FMA-pipe polynomial: 2 of 32. Measured at
// L = 4608 (1x24 heads): 0/32 1040, 2/32 1041, 4/32 1039, 8/32 1028, 12/32 995, 16/32 945 TFLOP/s —
// the MUFU pipe is not what bounds the softmax, so the polynomial only pays at a small share.
__device__ __forceinline__ constexpr bool poly_pair(int i) { return (i & 15) == 15; }

// One softmax warpgroup: owns query tile `x` (rows q_base .. q_base+127), S in TMEM columns s_col
// (P overwrites the first 64 of them), O in o_col.
__device__ __forceinline__ void softmax_tile(const Args& args, int nkv, int q_base, uint32_t tmem, uint32_t s_col,
                                             uint32_t o_col, uint64_t* s_full, uint64_t* p_half, uint64_t* p_full,
                                             uint64_t* pv_done, volatile int* abort_flag) {
  const int warp = warp_id();
  const int lane = lane_id();
  const int quarter = warp & 3;
  const int row = quarter * 32 + lane;
  const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
  const float sl2 = args.scale_log2;
  float m_run = -INFINITY;
  float l_run = 0.f;
  bool ok = true;
  for (int j = 0; j < nkv; ++j) {
    if (!mbar_wait(s_full, j & 1, abort_flag, args.status, FB_DEV_TIMEOUT_MMA)) {
      ok = false;
      break;
    }
    tc_fence_after_sync();
    // Pass 1: the row max, reading S from TMEM in two 64-column halves; four independent running
    // maxima keep the dependency chain short. Keys 64..127 are read first and keys 0..63 last, and
    // those stay in registers for the first half of pass 2: three TMEM round trips per tile, not four.
    const int valid = args.seq - j * BKV;  // keys of this tile that exist (>= 1)
    float mxa = -INFINITY, mxb = -INFINITY, mxc = -INFINITY, mxd = -INFINITY;
    // keys 64..127 first; keys 0..63 last, kept in registers for the first half of pass 2
    uint32_t keep[2][32];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int h = 1 - hh;
      uint32_t tmp[2][32];
      uint32_t (&sr)[2][32] = h == 0 ? keep : tmp;
      tmem_ld_32x32b_x32(tmem + lane_base + s_col + 64 * h, sr[0]);
      tmem_ld_32x32b_x32(tmem + lane_base + s_col + 64 * h + 32, sr[1]);
      tmem_ld_wait();
      if (valid < BKV) {  // only the last KV tile has keys past the sequence end
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (64 * h + i >= valid) sr[i >> 5][i & 31] = __float_as_uint(-INFINITY);
      }
#pragma unroll
      for (int i = 0; i < 64; i += 8) {
        mxa = max3(mxa, __uint_as_float(sr[i >> 5][i & 31]), __uint_as_float(sr[i >> 5][(i + 1) & 31]));
        mxb = max3(mxb, __uint_as_float(sr[i >> 5][(i + 2) & 31]), __uint_as_float(sr[i >> 5][(i + 3) & 31]));
        mxc = max3(mxc, __uint_as_float(sr[i >> 5][(i + 4) & 31]), __uint_as_float(sr[i >> 5][(i + 5) & 31]));
        mxd = max3(mxd, __uint_as_float(sr[i >> 5][(i + 6) & 31]), __uint_as_float(sr[i >> 5][(i + 7) & 31]));
      }
    }
    const float m_tile = fmaxf(fmaxf(mxa, mxb), fmaxf(mxc, mxd)) * sl2;
    float factor = 1.f;
    bool rescale = false;
    if (j == 0) {
      m_run = m_tile;
    } else if (m_tile > m_run + 8.0f) {
      factor = fast_exp2(m_run - m_tile);
      m_run = m_tile;
      rescale = true;
    }
    if (j > 0) {
      // PV_{j-1} must be complete: it reads this tile's P buffer and updates O. (It finished before
      // S_j did, since the tensor core runs in issue order, so this wait is normally immediate.)
      if (!mbar_wait(pv_done, (j - 1) & 1, abort_flag, args.status, FB_DEV_TIMEOUT_MMA)) {
        ok = false;
        break;
      }
      tc_fence_after_sync();
      if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          const uint32_t taddr = tmem + lane_base + o_col + 32 * c;
          tmem_ld_32x32b_x32(taddr, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * factor);
          tmem_st_32x32b_x32(taddr, r);
        }
        tmem_st_wait();
      }
    }
    // Pass 2, per 64-key half: P = exp2(s * scale * log2(e) - m) as packed bf16 pairs into TMEM
    // columns s_col + 32h .. +31 (half 1's S columns are read again before its P is stored; half 0's P
    // lands on S columns already consumed); the row sum keeps the fp32 values. poly_pair() pairs take the FMA-pipe
    // exponential, the rest the MUFU one.
    uint64_t psum[4] = {0, 0, 0, 0};  // four independent packed partial row sums
    const uint64_t sl2x2 = f2(sl2, sl2), negm = f2(-m_run, -m_run);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t tmp[2][32];
      uint32_t (&sr)[2][32] = h == 0 ? keep : tmp;  // keys 0..63 are still in registers from pass 1
      if (h == 1) {
        tmem_ld_32x32b_x32(tmem + lane_base + s_col + 64, sr[0]);
        tmem_ld_32x32b_x32(tmem + lane_base + s_col + 96, sr[1]);
        tmem_ld_wait();
        if (valid < BKV) {
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (64 + i >= valid) sr[i >> 5][i & 31] = __float_as_uint(-INFINITY);
        }
      }
      uint32_t p[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float a = __uint_as_float(sr[i >> 4][(2 * i) & 31]);
        const float b = __uint_as_float(sr[i >> 4][(2 * i + 1) & 31]);
        const uint64_t x = f2_fma(f2(a, b), sl2x2, negm);
        float e0, e1;
        if (poly_pair(i)) {
          exp2_poly_x2(x, e0, e1);
        } else {
          e0 = fast_exp2(f2_lo(x));
          e1 = fast_exp2(f2_hi(x));
        }
        psum[i & 3] = f2_add(psum[i & 3], f2(e0, e1));
        p[i] = pack_bf16x2(e0, e1);
      }
      tmem_st_32x32b_x32(tmem + lane_base + s_col + 32 * h, p);
      if (h == 0) {  // P for keys 0..63 is in place: the MMA may start O += P V on them
        tmem_st_wait();
        tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_half);
      }
    }
    const uint64_t ps = f2_add(f2_add(psum[0], psum[1]), f2_add(psum[2], psum[3]));
    l_run = l_run * factor + (f2_lo(ps) + f2_hi(ps));
    tmem_st_wait();
    tc_fence_before_sync();
    __syncwarp();
    if (lane == 0) mbar_arrive(p_full);
  }
  if (ok && mbar_wait(pv_done, (nkv - 1) & 1, abort_flag, args.status, FB_DEV_TIMEOUT_MMA)) {
    tc_fence_after_sync();
    const float inv = 1.0f / l_run;
    const int q = q_base + row;
    const bool row_ok = q < args.seq;
    const int64_t b = blockIdx.z;
    uint16_t* dst;
    if (args.sp_world > 0) {
      const int src = row_ok ? q / args.sp_ll : 0;
      dst = args.sp_out[src] + static_cast<int64_t>(q - src * args.sp_ll) * args.sp_ld + args.sp_col0;
    } else {
      dst = q < args.split ? args.out0 + (b * args.split + q) * args.ld0
                           : args.out1 + (b * (args.seq - args.split) + (q - args.split)) * args.ld1;
    }
    dst += static_cast<int64_t>(blockIdx.y) * HD;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(tmem + lane_base + o_col + 32 * c, r);
      tmem_ld_wait();
      if (row_ok) {
        uint4* d = reinterpret_cast<uint4*>(dst + 32 * c);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float* f = reinterpret_cast<const float*>(r) + 8 * i;
          d[i] = make_uint4(pack_bf16x2(f[0] * inv, f[1] * inv), pack_bf16x2(f[2] * inv, f[3] * inv),
                            pack_bf16x2(f[4] * inv, f[5] * inv), pack_bf16x2(f[6] * inv, f[7] * inv));
        }
      }
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1) attention_kernel(const __grid_constant__ Args args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                    // Q_A, Q_B
  uint8_t* sK = smem + 2 * kTileBytes;   // two slots
  uint8_t* sV = smem + 4 * kTileBytes;   // two slots
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 6 * kTileBytes);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [2]
  uint64_t* k_empty = bars + 3;   // [2]
  uint64_t* v_full = bars + 5;    // [2]
  uint64_t* v_empty = bars + 7;   // [2]
  uint64_t* s_full = bars + 9;    // [A, B]
  uint64_t* p_full = bars + 11;   // [A, B]
  uint64_t* pv_done = bars + 13;  // [A, B]
  uint64_t* drain = bars + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint64_t* p_half = bars + 17;   // [A, B]: P for the first 64 keys stored

  const int warp = warp_id();
  const int lane = lane_id();
  const int q0 = blockIdx.x * kRowsPerCta;
  const int bh = blockIdx.z * args.heads + blockIdx.y;
  const int nkv = (args.seq + BKV - 1) / BKV;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], 4);
      mbar_init(&p_half[s], 4);
      mbar_init(&pv_done[s], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&args.tq);
    tma_prefetch_desc(&args.tk);
    tma_prefetch_desc(&args.tv);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA
    if (lane == 0) {
      bool ok = true;
      int k_pending[2] = {-1, -1};  // parity of the last load into each slot, -1 = none
      int v_pending[2] = {-1, -1};
      mbar_arrive_expect_tx(q_full, 2 * kTileBytes);
      tma_load_3d(&args.tq, q_full, sQ, 0, q0, bh);
      tma_load_3d(&args.tq, q_full, sQ + kHalf, 64, q0, bh);
      tma_load_3d(&args.tq, q_full, sQ + kTileBytes, 0, q0 + BQ, bh);
      tma_load_3d(&args.tq, q_full, sQ + kTileBytes + kHalf, 64, q0 + BQ, bh);
      for (int j = 0; j < nkv; ++j) {
        const int ks = j & 1;
        if (j >= 2 && !mbar_wait(&k_empty[ks], ((j >> 1) - 1) & 1, abort_flag, args.status, FB_DEV_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        uint8_t* k_dst = sK + ks * kTileBytes;
        mbar_arrive_expect_tx(&k_full[ks], kTileBytes);
        tma_load_3d(&args.tk, &k_full[ks], k_dst, 0, j * BKV, bh);
        tma_load_3d(&args.tk, &k_full[ks], k_dst + kHalf, 64, j * BKV, bh);
        k_pending[ks] = (j >> 1) & 1;
        const int vs = j & 1;
        if (j >= 2 && !mbar_wait(&v_empty[vs], ((j >> 1) - 1) & 1, abort_flag, args.status, FB_DEV_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        uint8_t* v_dst = sV + vs * kTileBytes;
        mbar_arrive_expect_tx(&v_full[vs], kTileBytes);
        tma_load_3d(&args.tv, &v_full[vs], v_dst, 0, j * BKV, bh);
        tma_load_3d(&args.tv, &v_full[vs], v_dst + kHalf, 64, j * BKV, bh);
        v_pending[vs] = (j >> 1) & 1;
      }
      if (!ok) {
        // let the copies in flight land before the CTA exits (bounded)
        mbar_wait_quiet(q_full, 0, kWaitBudgetNs);
        for (int s = 0; s < 2; ++s) {
          if (k_pending[s] >= 0) mbar_wait_quiet(&k_full[s], static_cast<uint32_t>(k_pending[s]), kWaitBudgetNs);
          if (v_pending[s] >= 0) mbar_wait_quiet(&v_full[s], static_cast<uint32_t>(v_pending[s]), kWaitBudgetNs);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA
    if (lane == 0) {
      // Descriptors are built once; a K step adds its byte offset / 16 to the start-address field
      // (every address stays below 256 KB, so the 14-bit field never carries into the next one).
      const uint64_t dqa = sdesc_kmajor_sw128(smem_u32(sQ)), dqb = sdesc_kmajor_sw128(smem_u32(sQ + kTileBytes));
      const uint64_t dk0 = sdesc_kmajor_sw128(smem_u32(sK)), dk1 = sdesc_kmajor_sw128(smem_u32(sK + kTileBytes));
      const uint64_t dv0 = sdesc_mnmajor_sw128(smem_u32(sV), kHalf);
      const uint64_t dv1 = sdesc_mnmajor_sw128(smem_u32(sV + kTileBytes), kHalf);
      auto issue_s = [&](uint64_t dq, uint64_t dk, uint32_t s_col) {
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint64_t off = static_cast<uint64_t>(((kk >> 2) * kHalf + (kk & 3) * 32) >> 4);
          umma_bf16_ss(tmem + s_col, dq + off, dk + off, kIdescS, kk > 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [&](uint32_t p_col, uint64_t dvs, uint32_t o_col, bool acc, int half) {
#pragma unroll
        for (int k4 = 0; k4 < BKV / 32; ++k4) {  // 16 keys = 8 TMEM columns of P, 2 KB of V rows
          const int kk = half * (BKV / 32) + k4;
          umma_bf16_ts(tmem + o_col, tmem + p_col + 8 * kk, dvs + static_cast<uint64_t>((kk * 16 * 128) >> 4), kIdescO,
                       (acc || kk > 0) ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(q_full, 0, abort_flag, args.status, FB_DEV_TIMEOUT_TMA) &&
                mbar_wait(&k_full[0], 0, abort_flag, args.status, FB_DEV_TIMEOUT_TMA);
      if (ok) {
        tc_fence_after_sync();
        issue_s(dqa, dk0, 0);
        umma_commit(&s_full[0]);
        issue_s(dqb, dk0, 128);
        umma_commit(&s_full[1]);
        umma_commit(&k_empty[0]);
      }
      for (int j = 0; ok && j < nkv; ++j) {
        const int vs = j & 1;

        const bool more = j + 1 < nkv;
        const int kn = (j + 1) & 1;  // K slot of tile j + 1
        const uint64_t dkn = kn ? dk1 : dk0;
        // tile A: O_A += P_A V_j, then S_A(j+1)
        ok = mbar_wait(&v_full[vs], (j >> 1) & 1, abort_flag, args.status, FB_DEV_TIMEOUT_TMA) &&
             mbar_wait(&p_half[0], j & 1, abort_flag, args.status, FB_DEV_TIMEOUT_EPI);
        if (!ok) break;
        tc_fence_after_sync();
        issue_pv(0, vs ? dv1 : dv0, 256, j > 0, 0);
        ok = mbar_wait(&p_full[0], j & 1, abort_flag, args.status, FB_DEV_TIMEOUT_EPI);
        if (!ok) break;
        tc_fence_after_sync();
        issue_pv(0, vs ? dv1 : dv0, 256, true, 1);
        umma_commit(&pv_done[0]);
        if (more) {
          ok = mbar_wait(&k_full[kn], ((j + 1) >> 1) & 1, abort_flag, args.status, FB_DEV_TIMEOUT_TMA);
          if (!ok) break;
          tc_fence_after_sync();
          issue_s(dqa, dkn, 0);
          umma_commit(&s_full[0]);
        }
        // tile B: O_B += P_B V_j, then S_B(j+1)
        ok = mbar_wait(&p_half[1], j & 1, abort_flag, args.status, FB_DEV_TIMEOUT_EPI);
        if (!ok) break;
        tc_fence_after_sync();
        issue_pv(128, vs ? dv1 : dv0, 384, j > 0, 0);
        ok = mbar_wait(&p_full[1], j & 1, abort_flag, args.status, FB_DEV_TIMEOUT_EPI);
        if (!ok) break;
        tc_fence_after_sync();
        issue_pv(128, vs ? dv1 : dv0, 384, true, 1);
        umma_commit(&pv_done[1]);
        umma_commit(&v_empty[vs]);
        if (more) {
          issue_s(dqb, dkn, 128);
          umma_commit(&s_full[1]);
          umma_commit(&k_empty[kn]);
        }
      }
      umma_commit(drain);
      mbar_wait_quiet(drain, 0, kWaitBudgetNs);
    }
  } else {
    const int x = warp >= 6 ? 1 : 0;  // warps 2-5: tile A, warps 6-9: tile B (one call site: one copy of the code)
    softmax_tile(args, nkv, q0 + x * BQ, tmem, 128u * x, 256u + 128u * x, &s_full[x], &p_half[x], &p_full[x],
                 &pv_done[x],
                 abort_flag);
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace attn

std::string attention_setup() {
  const cudaError_t e =
      cudaFuncSetAttribute(attn::attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, attn::kSmemBytes);
  return e == cudaSuccess ? std::string() : std::string("cudaFuncSetAttribute(attention): ") + cudaGetErrorString(e);
}

static int encode_qkv_map(CUtensorMap* map, const uint16_t* base, int bh, int seq, std::string& err) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) {
    err = "cuTensorMapEncodeTiled unavailable (fb_init not run?)";
    return FB_ERR_INIT;
  }
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(attn::HD), static_cast<cuuint64_t>(seq),
                              static_cast<cuuint64_t>(bh)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(attn::HD) * 2,
                                 static_cast<cuuint64_t>(seq) * attn::HD * 2};
  const cuuint32_t box[3] = {64, 128, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<uint16_t*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    err = "cuTensorMapEncodeTiled(attention) failed (" + std::to_string(static_cast<int>(r)) + ")";
    return FB_ERR_CUDA;
  }
  return FB_OK;
}

int launch_attention_sp(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* const* out_peers,
                        int64_t ld_out, int col0, int heads, int seq_local, int sp_world, int head_dim, float scale,
                        cudaStream_t st, std::string& err) {
  if (head_dim != attn::HD) {
    err = "fb_attention_sp: head_dim must be 128";
    return FB_ERR_UNSUPPORTED;
  }
  if (sp_world < 1 || sp_world > 8 || heads <= 0 || heads > 65535 || seq_local < 0 || !out_peers) {
    err = "fb_attention_sp: need 1 <= sp_world <= 8, heads > 0, seq_local >= 0 and the output table";
    return FB_ERR_ARG;
  }
  if (ld_out % 8 != 0 || col0 % 8 != 0 || col0 < 0 || ld_out < col0 + static_cast<int64_t>(heads) * attn::HD) {
    err = "fb_attention_sp: ld_out and col0 multiples of 8 with col0 + heads*128 <= ld_out";
    return FB_ERR_ALIGN;
  }
  uintptr_t any = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v);
  for (int g = 0; g < sp_world; ++g) {
    if (!out_peers[g]) {
      err = "fb_attention_sp: null output pointer";
      return FB_ERR_ARG;
    }
    any |= reinterpret_cast<uintptr_t>(out_peers[g]);
  }
  if (any & 15u) {
    err = "fb_attention_sp: q, k, v and outputs must be 16-byte aligned";
    return FB_ERR_ALIGN;
  }
  const int seq = sp_world * seq_local;
  if (seq == 0) return FB_OK;
  std::string derr;
  DeviceState* dev = current_device(derr);
  if (!dev) {
    err = derr;
    return FB_ERR_INIT;
  }
  attn::Args args;
  memset(&args, 0, sizeof(args));
  int rc = encode_qkv_map(&args.tq, q, heads, seq, err);
  if (!rc) rc = encode_qkv_map(&args.tk, k, heads, seq, err);
  if (!rc) rc = encode_qkv_map(&args.tv, v, heads, seq, err);
  if (rc) return rc;
  args.split = 0;
  args.seq = seq;
  args.heads = heads;
  args.scale_log2 = scale * 1.4426950408889634f;
  args.status = dev->status;
  args.sp_world = sp_world;
  args.sp_ll = seq_local;
  args.sp_col0 = col0;
  args.sp_ld = ld_out;
  for (int g = 0; g < sp_world; ++g) args.sp_out[g] = out_peers[g];
  const dim3 grid((seq + attn::kRowsPerCta - 1) / attn::kRowsPerCta, heads, 1);
  attn::attention_kernel<<<grid, attn::kThreads, attn::kSmemBytes, st>>>(args);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    err = std::string("attention launch: ") + cudaGetErrorString(e);
    return FB_ERR_CUDA;
  }
  return FB_OK;
}

int launch_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out0, int64_t ld0,
                     uint16_t* out1, int64_t ld1, int split, int batch, int heads, int seq, int head_dim, float scale,
                     cudaStream_t st, std::string& err) {
  if (head_dim != attn::HD) {
    err = "fb_attention: head_dim must be 128";
    return FB_ERR_UNSUPPORTED;
  }
  if (batch < 0 || heads <= 0 || seq < 0 || heads > 65535 || batch > 65535) {
    err = "fb_attention: bad shape";
    return FB_ERR_ARG;
  }
  if (split < 0 || split > seq || (split > 0 && out0 == nullptr) || (split < seq && out1 == nullptr)) {
    err = "fb_attention: split must be in [0, seq] with an output for each non-empty part";
    return FB_ERR_ARG;
  }
  const int64_t need = static_cast<int64_t>(heads) * attn::HD;
  if ((split > 0 && (ld0 < need || ld0 % 8 != 0)) || (split < seq && (ld1 < need || ld1 % 8 != 0))) {
    err = "fb_attention: output row strides must be >= heads*128 and multiples of 8";
    return FB_ERR_ALIGN;
  }
  const uintptr_t any = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                        reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(out0) |
                        reinterpret_cast<uintptr_t>(out1);
  if (any & 15u) {
    err = "fb_attention: q, k, v and outputs must be 16-byte aligned";
    return FB_ERR_ALIGN;
  }
  if (batch == 0 || seq == 0) return FB_OK;
  std::string derr;
  DeviceState* dev = current_device(derr);
  if (!dev) {
    err = derr;
    return FB_ERR_INIT;
  }
  attn::Args args;
  memset(&args, 0, sizeof(args));
  int rc = encode_qkv_map(&args.tq, q, batch * heads, seq, err);
  if (!rc) rc = encode_qkv_map(&args.tk, k, batch * heads, seq, err);
  if (!rc) rc = encode_qkv_map(&args.tv, v, batch * heads, seq, err);
  if (rc) return rc;
  args.out0 = out0;
  args.ld0 = ld0;
  args.out1 = out1;
  args.ld1 = ld1;
  args.split = split;
  args.seq = seq;
  args.heads = heads;
  args.scale_log2 = scale * 1.4426950408889634f;
  args.status = dev->status;
  const dim3 grid((seq + attn::kRowsPerCta - 1) / attn::kRowsPerCta, heads, batch);
  attn::attention_kernel<<<grid, attn::kThreads, attn::kSmemBytes, st>>>(args);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    err = std::string("attention launch: ") + cudaGetErrorString(e);
    return FB_ERR_CUDA;
  }
  return FB_OK;
}

}  // namespace fb
