// gemm_common.cuh — what the tcgen05 GEMM kernels share: the per-problem launch arguments, the
// persistent tile raster, and the fused epilogues that turn one accumulator row (one TMEM lane = one
// output row) into the outputs of a FLUX Linear.
#pragma once

#include "fb_internal.h"

namespace fb {
namespace gemm {

constexpr int BK = 64;

struct alignas(64) Problem {
  CUtensorMap tma_a;
  CUtensorMap tma_b;
  CUtensorMap tma_resid;  // pair kernel, gated residual: fp32 [m, n] rows of `resid`, 32 x 32 boxes
  CUtensorMap tma_cos;    // pair kernel, QKV: the RoPE tables, fp32 [seq_total, 64], 32-row x 16-column boxes
  CUtensorMap tma_sin;
  const uint16_t* bias;
  void* out;
  const float* resid;
  const uint16_t* gate;
  const float* q_scale;
  const float* k_scale;
  const float* rope_cos;
  const float* rope_sin;
  uint16_t* q;
  uint16_t* k;
  uint16_t* v;
  int64_t ld_out, ld_resid, gate_bstride;
  int m, n, num_kb, tiles_m, tiles_n, tile_begin, tile_end;
  int rows_per_batch, guard;
  int heads, seq_total, seq_offset, qkv_cols, gelu_col0;
  int n_offset;  // QKV epilogue: column `n` of this problem is column `n_offset + n` of the full Linear
  // decoded weights (gemm_nf4.cu): NF4 - tma_b maps the packed bytes [n, k/2], absmax holds k/64 values
  // per row; int8_row - tma_b maps the int8 rows [n, k], absmax holds one scale per row
  const float* absmax;
  const float* code16;
  int absmax_per_row;
  int fp8_e5m2;  // fp8 weights: 1 = e5m2, 0 = e4m3fn
  // QKV epilogue, sequence-parallel scatter (sp_world > 0, one image): head h of this rank's seq_total
  // tokens goes to rank g = h / (heads / sp_world), buffer sp_dst[g] laid out [3][heads/sp_world]
  // [sp_world * seq_total][128] (q, k, v; the head within the group; the gathered token = sp_rank *
  // seq_total + position): the all-to-all of Ulysses attention done by the epilogue's stores over NVLink.
  uint16_t* sp_dst[8];
  int sp_world, sp_rank;
};

struct Args {
  Problem prob[2];
  int nprob;
  int total_tiles;
  int* status;
  // split-K (decoding GEMM only): work item w covers tile w % total_tiles, K steps of split
  // w / total_tiles; partial rows in splitk_ws, arrivals per (tile, CTA) in splitk_count
  int splits;
  float* splitk_ws;
  int* splitk_count;
};

// Raster: groups of group_m(P) M-tiles, M fastest inside a group. Narrow outputs (at most 16 column
// tiles: proj, MLP-out, linear2 at N = 3072) take groups of 4, so that the tiles running at once share
// more A rows (linear2: DRAM bytes per launch 676 -> 586 MB at the same speed); wide ones (QKV, MLP-in,
// linear1) keep 16, where groups of 4 cost up to 5 %.
constexpr int kGroupM = 16;
constexpr int kGroupMNarrow = 4;
__device__ __forceinline__ int group_m(const Problem& P) { return P.tiles_n <= 16 ? kGroupMNarrow : kGroupM; }

__device__ __forceinline__ void decode_tile(const Args& a, int tile, int& p, int& mb, int& nb) {
  p = (a.nprob > 1 && tile >= a.prob[1].tile_begin) ? 1 : 0;
  const Problem& P = a.prob[p];
  const int local = tile - P.tile_begin;
  const int g = group_m(P);
  const int per_group = g * P.tiles_n;
  const int group = local / per_group;
  const int first_m = group * g;
  const int gm = min(P.tiles_m - first_m, g);
  const int in_group = local - group * per_group;
  mb = first_m + in_group % gm;
  nb = in_group / gm;
}

// 32 consecutive bf16 bias values (or zeros).
__device__ __forceinline__ void load_bias32(const uint16_t* bias, int n0, float (&b)[32]) {
  if (bias == nullptr) {
#pragma unroll
    for (int j = 0; j < 32; ++j) b[j] = 0.f;
    return;
  }
  const uint4* p = reinterpret_cast<const uint4*>(bias + n0);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint4 u = __ldg(p + i);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      b[8 * i + 2 * j] = __uint_as_float(w[j] << 16);
      b[8 * i + 2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
    }
  }
}

// 8 * NQ consecutive bf16 values kept packed (4 * NQ registers instead of 8 * NQ), zeros for a null
// pointer; bf16_at() widens element e (a compile-time index after unrolling).
template <int NQ>
__device__ __forceinline__ void load_bf16_packed(const uint16_t* p, int n0, uint4 (&q)[NQ]) {
#pragma unroll
  for (int i = 0; i < NQ; ++i) q[i] = p ? __ldg(reinterpret_cast<const uint4*>(p + n0) + i) : make_uint4(0, 0, 0, 0);
}
__device__ __forceinline__ void load_bf16x32_packed(const uint16_t* p, int n0, uint4 (&q)[4]) { load_bf16_packed<4>(p, n0, q); }
template <int NQ>
__device__ __forceinline__ float bf16_at(const uint4 (&q)[NQ], int e) {
  const uint4 u = q[e >> 3];
  const int w = (e >> 1) & 3;
  const uint32_t v = w == 0 ? u.x : w == 1 ? u.y : w == 2 ? u.z : u.w;
  return __uint_as_float((e & 1) ? (v & 0xFFFF0000u) : (v << 16));
}

// Store 32 fp32 values as bf16 (64 contiguous bytes).
__device__ __forceinline__ void store_bf16x32(uint16_t* dst, const float (&v)[32]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    d[i] = make_uint4(pack_bf16x2(v[8 * i], v[8 * i + 1]), pack_bf16x2(v[8 * i + 2], v[8 * i + 3]),
                      pack_bf16x2(v[8 * i + 4], v[8 * i + 5]), pack_bf16x2(v[8 * i + 6], v[8 * i + 7]));
  }
}

template <int EPI>
__device__ __forceinline__ void epilogue_chunk(const Problem& P, int m, bool row_ok, int n0, const uint32_t (&r)[32]) {
  float b[32];
  load_bias32(P.bias, n0, b);
  float y[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) y[j] = bf16_round(__fadd_rn(__uint_as_float(r[j]), b[j]));
  if (!row_ok) return;
  if constexpr (EPI == FB_EPI_STORE_BF16) {
    store_bf16x32(static_cast<uint16_t*>(P.out) + static_cast<int64_t>(m) * P.ld_out + n0, y);
  } else if constexpr (EPI == FB_EPI_STORE_F32) {
    float4* d = reinterpret_cast<float4*>(static_cast<float*>(P.out) + static_cast<int64_t>(m) * P.ld_out + n0);
#pragma unroll
    for (int i = 0; i < 8; ++i) d[i] = make_float4(y[4 * i], y[4 * i + 1], y[4 * i + 2], y[4 * i + 3]);
  } else if constexpr (EPI == FB_EPI_GELU) {
#pragma unroll
    for (int j = 0; j < 32; ++j) y[j] = gelu_tanh_f32(y[j]);
    store_bf16x32(static_cast<uint16_t*>(P.out) + static_cast<int64_t>(m) * P.ld_out + n0, y);
  } else if constexpr (EPI == FB_EPI_GATED_RESIDUAL) {
    const int64_t img = m / P.rows_per_batch;
    float g[32];
    load_bias32(P.gate + img * P.gate_bstride, n0, g);
    const float4* x = reinterpret_cast<const float4*>(P.resid + static_cast<int64_t>(m) * P.ld_resid + n0);
    float4* d = reinterpret_cast<float4*>(static_cast<float*>(P.out) + static_cast<int64_t>(m) * P.ld_out + n0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 xv = x[i];
      float t[4] = {y[4 * i], y[4 * i + 1], y[4 * i + 2], y[4 * i + 3]};
      if (P.guard) {
#pragma unroll
        for (int j = 0; j < 4; ++j) t[j] = fminf(fmaxf(t[j], -65504.0f), 65504.0f);
      }
      d[i] = make_float4(__fadd_rn(xv.x, __fmul_rn(g[4 * i], t[0])), __fadd_rn(xv.y, __fmul_rn(g[4 * i + 1], t[1])),
                         __fadd_rn(xv.z, __fmul_rn(g[4 * i + 2], t[2])), __fadd_rn(xv.w, __fmul_rn(g[4 * i + 3], t[3])));
    }
  }
}

// Gated-residual epilogue of one tile row: out = resid + gate * f32(bf16(acc + bias)), 32 columns per
// step, over the tile's 32-column chunks [c_lo, c_hi). The residual of step c+1 is loaded while step c
// waits for its accumulator columns, so the global-memory latency of the residual overlaps the TMEM
// loads and the math.
template <int BN>
__device__ __forceinline__ void epilogue_resid_row(const Problem& P, int m, bool row_ok, int nb, uint32_t trow,
                                                   int c_lo = 0, int c_hi = BN / 32) {
  const int nchunks = min(c_hi, (P.n - nb * BN) / 32);
  // Rows past M (padding of the last tile) still run the TMEM loads, but must not compute an image
  // index past the last image: their gate reads would leave the modulation tensor.
  const int64_t img = row_ok ? m / P.rows_per_batch : 0;
  const float4* xrow = reinterpret_cast<const float4*>(P.resid + static_cast<int64_t>(m) * P.ld_resid + nb * BN);
  float4* orow = reinterpret_cast<float4*>(static_cast<float*>(P.out) + static_cast<int64_t>(m) * P.ld_out + nb * BN);
  const uint16_t* grow = P.gate + img * P.gate_bstride;
  float4 xa[8];
  if (row_ok && c_lo < nchunks) {
#pragma unroll
    for (int i = 0; i < 8; ++i) xa[i] = xrow[8 * c_lo + i];
  }
#pragma unroll 1
  for (int c = c_lo; c < nchunks; ++c) {
    float4 xb[8];
    if (row_ok && c + 1 < nchunks) {
#pragma unroll
      for (int i = 0; i < 8; ++i) xb[i] = xrow[8 * (c + 1) + i];
    }
    const int n0 = nb * BN + 32 * c;
    uint32_t r[32];
    tmem_ld_32x32b_x32(trow + 32 * c, r);
    uint4 bq[4], gq[4];  // bias and gate stay packed bf16 until used
    load_bf16x32_packed(P.bias, n0, bq);
    load_bf16x32_packed(grow, n0, gq);
    tmem_ld_wait();
    if (row_ok) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float t[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          t[j] = bf16_round(__fadd_rn(__uint_as_float(r[4 * i + j]), bf16_at(bq, 4 * i + j)));
          if (P.guard) t[j] = fminf(fmaxf(t[j], -65504.0f), 65504.0f);
        }
        orow[8 * c + i] = make_float4(__fadd_rn(xa[i].x, __fmul_rn(bf16_at(gq, 4 * i), t[0])),
                                      __fadd_rn(xa[i].y, __fmul_rn(bf16_at(gq, 4 * i + 1), t[1])),
                                      __fadd_rn(xa[i].z, __fmul_rn(bf16_at(gq, 4 * i + 2), t[2])),
                                      __fadd_rn(xa[i].w, __fmul_rn(bf16_at(gq, 4 * i + 3), t[3])));
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) xa[i] = xb[i];
  }
}

// One 32-row x 32-column fp32 box of the residual (TMA, 128-byte swizzle): 4 KB.
constexpr int kResidBoxBytes = 32 * 32 * 4;

// Gated-residual epilogue of one tile row over the tile's 32-column chunks [c_lo, c_hi):
// out = resid + gate * f32(bf16(acc + bias)). The warp's 32 x 32 box of the residual arrives by TMA
// (128-byte swizzle) into `buf` while the chunk before it is finished, and each thread reads its row
// from shared memory: a row per thread read straight from global memory costs 32 L1 wavefronts per
// 16-byte load, which the mainloop's shared-memory traffic then waits for. A chunk is finished in SUB
// steps of 32 / SUB columns (SUB = 2 halves the registers it holds, for kernels compiled to 128 per
// thread). `row0` is the warp's first row; `buf` (kResidBoxBytes, 1024-byte aligned) and `bar` are the
// warp's own, `phase` tracks `bar`. Needs P.tma_resid. Returns false if a wait gave up; the load it
// waited for may then still be in flight (the caller lets it land).
template <int BN, int SUB = 1>
__device__ __forceinline__ bool resid_row_tma(const Problem& P, int m, bool row_ok, int nb, uint32_t trow, int c_lo,
                                              int c_hi, int row0, uint8_t* buf, uint64_t* bar, uint32_t& phase,
                                              volatile int* abort_flag, int* status) {
  static_assert(SUB == 1 || SUB == 2, "32 or 16 columns per step");
  constexpr int NC = 32 / SUB;  // columns per step
  constexpr int NV = NC / 4;    // float4 per step
  const int lane = lane_id();
  const int nchunks = min(c_hi, (P.n - nb * BN) / 32);
  if (c_lo >= nchunks) return true;
  // Rows past M (padding of the last tile) still run the TMEM loads, but must not compute an image
  // index past the last image: their gate reads would leave the modulation tensor.
  const int64_t img = row_ok ? m / P.rows_per_batch : 0;
  float4* orow = reinterpret_cast<float4*>(static_cast<float*>(P.out) + static_cast<int64_t>(m) * P.ld_out + nb * BN);
  const uint16_t* grow = P.gate + img * P.gate_bstride;
  if (lane == 0) {
    mbar_arrive_expect_tx(bar, kResidBoxBytes);
    tma_load_2d(&P.tma_resid, bar, buf, nb * BN + 32 * c_lo, row0);
  }
  const uint8_t* myrow = buf + lane * 128;  // this thread's row: 8 chunks of 16 bytes, swizzled by row % 8
  const int sw = lane & 7;
#pragma unroll 1
  for (int c = c_lo; c < nchunks; ++c) {
#pragma unroll
    for (int h = 0; h < SUB; ++h) {
      const int n0 = nb * BN + 32 * c + NC * h;
      uint32_t r[NC];
      if constexpr (NC == 32) {
        tmem_ld_32x32b_x32(trow + 32 * c, r);
      } else {
        tmem_ld_32x32b_x16(trow + 32 * c + NC * h, r);
      }
      uint4 bq[NC / 8], gq[NC / 8];  // bias and gate stay packed bf16 until used
      load_bf16_packed<NC / 8>(P.bias, n0, bq);
      load_bf16_packed<NC / 8>(grow, n0, gq);
      if (h == 0 && !mbar_wait(bar, phase, abort_flag, status, FB_DEV_TIMEOUT_TMA)) {
        tmem_ld_wait();
        return false;
      }
      float4 xa[NV];
#pragma unroll
      for (int i = 0; i < NV; ++i) xa[i] = *reinterpret_cast<const float4*>(myrow + (((NV * h + i) ^ sw) << 4));
      if (h == SUB - 1) {
        phase ^= 1u;
        __syncwarp();  // every lane has its row before the next box overwrites the buffer
        if (c + 1 < nchunks && lane == 0) {
          fence_proxy_async_smem();
          mbar_arrive_expect_tx(bar, kResidBoxBytes);
          tma_load_2d(&P.tma_resid, bar, buf, nb * BN + 32 * (c + 1), row0);
        }
      }
      tmem_ld_wait();
      if (row_ok) {
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          float t[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            t[j] = bf16_round(__fadd_rn(__uint_as_float(r[4 * i + j]), bf16_at(bq, 4 * i + j)));
            if (P.guard) t[j] = fminf(fmaxf(t[j], -65504.0f), 65504.0f);
          }
          orow[8 * c + NV * h + i] = make_float4(__fadd_rn(xa[i].x, __fmul_rn(bf16_at(gq, 4 * i), t[0])),
                                                 __fadd_rn(xa[i].y, __fmul_rn(bf16_at(gq, 4 * i + 1), t[1])),
                                                 __fadd_rn(xa[i].z, __fmul_rn(bf16_at(gq, 4 * i + 2), t[2])),
                                                 __fadd_rn(xa[i].w, __fmul_rn(bf16_at(gq, 4 * i + 3), t[3])));
        }
      }
    }
  }
  return true;
}

// Where the QKV epilogue reads the RoPE tables from. Global (tab == nullptr): each thread loads its row's
// cos/sin as float4 straight from global memory (32 lines per warp instruction). Staged: the warp's 32
// rows of the 16 table columns a 32-column chunk needs arrive by TMA (a 2 KB box of cos and one of
// sin, 64-byte swizzle) into the warp's 4 KB buffer, the next chunk's boxes while the current chunk is
// finished. Needs P.tma_cos / P.tma_sin and 32 consecutive table rows for the warp's 32 output rows.
// Passed by value (all inlined) so that it stays in registers.
struct RopeStage {
  bool on;          // false: the tables come from global memory
  uint8_t* buf;     // 4 KB, 1024-byte aligned: cos box, then sin box
  uint64_t* bar;    // the warp's barrier
  uint32_t* phase;  // its phase bit
  int pos0;         // table row of the warp's first output row
  volatile int* abort_flag;
  int* status;
};

__device__ __forceinline__ void rope_stage_issue(const Problem& P, const RopeStage& t, int chunk) {
  fence_proxy_async_smem();
  mbar_arrive_expect_tx(t.bar, 2 * 32 * 16 * 4);
  tma_load_2d(&P.tma_cos, t.bar, t.buf, 16 * chunk, t.pos0);
  tma_load_2d(&P.tma_sin, t.bar, t.buf + 2048, 16 * chunk, t.pos0);
}

// QKV epilogue for one 128-column group (one head of q, k or v): RMSNorm + RoPE for q/k.
// `local0` indexes this problem's columns (bias, bounds); `col0` is the column of the full Linear
// (which of q/k/v and which head). Two passes over the accumulator columns in TMEM keep the register
// footprint small: pass 1 accumulates the sum of squares (sequentially over the 128 values), pass 2
// re-reads each 32-column chunk, normalises, rotates and stores it. `tab.on` (warp-uniform) stages the
// RoPE tables through shared memory; returns false only if a staged wait gave up (the box it waited
// for may still be in flight).
__device__ __forceinline__ bool epilogue_qkv_group(const Problem& P, int m, bool row_ok, int local0, int col0,
                                                   uint32_t taddr, RopeStage tab = RopeStage{}) {
  constexpr int HD = 128;
  const int hd_all = P.heads * HD;
  const int part = col0 / hd_all;  // 0 = q, 1 = k, 2 = v
  const bool staged = tab.on && part < 2;
  const int lane = lane_id();
  if (staged && lane == 0) rope_stage_issue(P, tab, 0);  // lands while pass 1 runs
  float rr = 1.f;
  if (part < 2) {
    float ss = 0.f;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(taddr + 32 * c, r);
      float b[32];
      load_bias32(P.bias, local0 + 32 * c, b);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float y = bf16_round(__fadd_rn(__uint_as_float(r[j]), b[j]));
        ss = __fadd_rn(ss, __fmul_rn(y, y));
      }
    }
    rr = rsqrtf(ss / static_cast<float>(HD) + 1e-6f);
  }
  const int head = (col0 - part * hd_all) / HD;
  const int img = row_ok ? m / P.rows_per_batch : 0;
  const int pos = P.seq_offset + (m - img * P.rows_per_batch);
  uint16_t* out;
  if (P.sp_world > 0) {
    const int hp = P.heads / P.sp_world;
    const int64_t ltot = static_cast<int64_t>(P.sp_world) * P.seq_total;
    out = P.sp_dst[head / hp] + ((static_cast<int64_t>(part) * hp + head % hp) * ltot +
                                 static_cast<int64_t>(P.sp_rank) * P.seq_total + pos) * HD;
  } else {
    const int64_t dst = ((static_cast<int64_t>(img) * P.heads + head) * P.seq_total + pos) * HD;
    out = (part == 0 ? P.q : part == 1 ? P.k : P.v) + dst;
  }
  // scale, cos and sin are read as float4 (16-byte aligned rows): a quarter of the load instructions
  // of scalar reads, which matters because every lane reads a different cos/sin row.
  const float4* sc4 = reinterpret_cast<const float4*>(part == 0 ? P.q_scale : P.k_scale);
  const float4* cs4 = reinterpret_cast<const float4*>(P.rope_cos + static_cast<int64_t>(pos) * (HD / 2));
  const float4* sn4 = reinterpret_cast<const float4*>(P.rope_sin + static_cast<int64_t>(pos) * (HD / 2));
  // staged: this thread's table row in the 64-byte-swizzled boxes (16-byte unit u of row r sits at unit
  // u ^ ((r >> 1) & 3) of its 64 bytes)
  const uint8_t* crow = staged ? tab.buf + lane * 64 : nullptr;
  const int sw = (lane >> 1) & 3;
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(taddr + 32 * c, r);
    float b[32];
    load_bias32(P.bias, local0 + 32 * c, b);
    float4 ct[4], st[4];
    if (staged) {
      if (!mbar_wait(tab.bar, *tab.phase, tab.abort_flag, tab.status, FB_DEV_TIMEOUT_TMA)) {
        tmem_ld_wait();
        return false;
      }
#pragma unroll
      for (int i4 = 0; i4 < 4; ++i4) {
        ct[i4] = *reinterpret_cast<const float4*>(crow + ((i4 ^ sw) << 4));
        st[i4] = *reinterpret_cast<const float4*>(crow + 2048 + ((i4 ^ sw) << 4));
      }
      *tab.phase ^= 1u;
      __syncwarp();  // every lane has its row before the next boxes overwrite the buffer
      if (c + 1 < 4 && lane == 0) rope_stage_issue(P, tab, c + 1);
    }
    tmem_ld_wait();
    float f[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) f[j] = bf16_round(__fadd_rn(__uint_as_float(r[j]), b[j]));
    if (part < 2 && row_ok) {
#pragma unroll
      for (int i4 = 0; i4 < 4; ++i4) {  // 4 rotation pairs (8 dims) per step; pair index 16c + 4 i4 + p
        const float4 c4 = staged ? ct[i4] : __ldg(cs4 + 4 * c + i4);
        const float4 s4 = staged ? st[i4] : __ldg(sn4 + 4 * c + i4);
        const float4 sa = __ldg(sc4 + 8 * c + 2 * i4), sb = __ldg(sc4 + 8 * c + 2 * i4 + 1);
        const float cv[4] = {c4.x, c4.y, c4.z, c4.w};
        const float sv[4] = {s4.x, s4.y, s4.z, s4.w};
        const float gv[8] = {sa.x, sa.y, sa.z, sa.w, sb.x, sb.y, sb.z, sb.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int i = 4 * i4 + q;
          const float e = __fmul_rn(__fmul_rn(f[2 * i], rr), gv[2 * q]);
          const float o = __fmul_rn(__fmul_rn(f[2 * i + 1], rr), gv[2 * q + 1]);
          f[2 * i] = __fsub_rn(__fmul_rn(e, cv[q]), __fmul_rn(o, sv[q]));
          f[2 * i + 1] = __fadd_rn(__fmul_rn(e, sv[q]), __fmul_rn(o, cv[q]));
        }
      }
    }
    if (row_ok) store_bf16x32(out + 32 * c, f);
  }
  return true;
}

// The epilogue of one accumulator row of one tile: `trow` addresses this thread's TMEM lane at the
// tile's first accumulator column; `m` is the output row, `nb` the tile's column block (BN wide).
// [col_lo, col_hi) is the part of the tile's columns this thread finishes (multiples of 128 when BN
// is, so that a head of the QKV epilogue never straddles two threads; the whole tile by default).
// kLean: a lower-register variant of the gated-residual epilogue (no prefetch of the next chunk's
// residual), for kernels that run more warps per CTA. `tab`: the QKV epilogue's RoPE tables staged
// through shared memory (epilogue_qkv_group). Returns false only if a staged wait gave up.
template <int BN, int EPI, bool kLean = false>
__device__ __forceinline__ bool epilogue_row(const Problem& P, int m, bool row_ok, int nb, uint32_t trow,
                                             int col_lo = 0, int col_hi = BN, RopeStage tab = RopeStage{}) {
  if constexpr (EPI == FB_EPI_QKV) {
#pragma unroll 1
    for (int g = col_lo / 128; g < col_hi / 128; ++g) {
      const int local0 = nb * BN + g * 128;
      if (local0 >= P.n) break;
      const int col0 = P.n_offset + local0;
      if (col0 < P.qkv_cols) {
        if (!epilogue_qkv_group(P, m, row_ok, local0, col0, trow + 128 * g, tab)) return false;
      } else {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(trow + 128 * g + 32 * c, r);
          tmem_ld_wait();
          float b[32];
          load_bias32(P.bias, local0 + 32 * c, b);
          float y[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) y[j] = gelu_tanh_f32(bf16_round(__fadd_rn(__uint_as_float(r[j]), b[j])));
          if (row_ok)
            store_bf16x32(static_cast<uint16_t*>(P.out) + static_cast<int64_t>(m) * P.ld_out + P.gelu_col0 +
                              (col0 + 32 * c - P.qkv_cols),
                          y);
        }
      }
    }
  } else if constexpr (EPI == FB_EPI_GATED_RESIDUAL && !kLean) {
    epilogue_resid_row<BN>(P, m, row_ok, nb, trow, col_lo / 32, col_hi / 32);
  } else {
#pragma unroll 1
    for (int c = col_lo / 32; c < col_hi / 32; ++c) {
      const int n0 = nb * BN + 32 * c;
      if (n0 >= P.n) break;
      uint32_t r[32];
      tmem_ld_32x32b_x32(trow + 32 * c, r);
      tmem_ld_wait();
      epilogue_chunk<EPI>(P, m, row_ok, n0, r);
    }
  }
  return true;
}

}  // namespace gemm

// The fused decode GEMM (gemm_nf4.cu): one-time attribute set-up and launch. wfmt 1 = NF4 (tma_b maps
// the packed bytes, absmax/code16 set), 2 = int8_row (tma_b maps the int8 rows, absmax = row scales),
// 3 = fp8 raw (tma_b maps the fp8 rows, fp8_e5m2 selects the format).
std::string gemm_nf4_setup();
cudaError_t launch_gemm_decode(int wfmt, int epilogue, const gemm::Args& args, int grid, cudaStream_t st);
// The CTA-pair bf16 GEMM (gemm_pair.cu): 256 x 256 tiles on clusters of two CTAs. Enabled unless
// the environment sets FLUX_B200_GEMM=single (read once), which selects the one-CTA kernel.
std::string gemm_pair_setup();
cudaError_t launch_gemm_pair(int epilogue, const gemm::Args& args, int grid, cudaStream_t st);
bool gemm_pair_enabled();

}  // namespace fb
