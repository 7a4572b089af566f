/*
 * flux_b200.h — C-ABI of libflux_b200.so, the sm_100a (B200) kernels behind selas's FLUX
 * transformer step.
 *
 * Conventions
 *   - Every entry point returns int32_t status: 0 = ok, > 0 = an FB_ERR_* code; the message is
 *     available from fb_last_error() (thread-local).
 *   - All pointers are device pointers owned by the caller. The library allocates no device memory
 *     on any call below (fb_init allocates one small status word per device, once).
 *   - bf16 tensors are passed as uint16_t*; fp32 as float*. Strides are in elements.
 *   - `stream` is a cudaStream_t passed as void*; every launch goes on it and nothing synchronizes
 *     the host, so calls may be captured in a CUDA graph.
 *   - Shapes and alignments are validated on the host before launching; a violation returns
 *     FB_ERR_ARG / FB_ERR_ALIGN and launches nothing.
 *   - Kernels that wait on mbarriers give up after a bounded time, set the device status word and
 *     return; fb_device_status() reads (and optionally clears) it.
 *
 * The reference (tcox-coding/selas) is pure Python; each entry point names the reference function
 * whose arithmetic it implements.
 */
#ifndef FLUX_B200_H
#define FLUX_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum fb_error {
  FB_OK = 0,
  FB_ERR_ARG = 1,          /* bad shape / argument */
  FB_ERR_ALIGN = 2,        /* pointer or stride alignment the kernels need */
  FB_ERR_CUDA = 3,         /* a CUDA runtime or driver call failed */
  FB_ERR_UNSUPPORTED = 4,  /* a configuration these kernels do not implement */
  FB_ERR_INIT = 5,         /* fb_init failed (no sm_100 device, missing driver entry point) */
  FB_ERR_DEVICE = 6        /* a kernel reported a device-side error (see fb_device_status) */
};

enum fb_dtype { FB_F32 = 0, FB_F16 = 1, FB_BF16 = 2 };

/* Device-side status codes written by the kernels (first error wins). */
enum fb_device_code {
  FB_DEV_OK = 0,
  FB_DEV_TIMEOUT_TMA = 1,    /* a wait for a TMA load gave up */
  FB_DEV_TIMEOUT_MMA = 2,    /* a wait for tensor-core work gave up */
  FB_DEV_TIMEOUT_EPI = 3,    /* a wait for the epilogue / softmax warps gave up */
  FB_DEV_BAD_SHAPE = 4,      /* a kernel saw a shape its host check should have rejected */
  FB_DEV_TIMEOUT_PEER = 5    /* fb_peer_barrier gave up waiting for another rank */
};

/* Epilogues of fb_linear_grouped (all problems of one call share one). */
enum fb_epilogue {
  FB_EPI_STORE_BF16 = 0,     /* out bf16 = bf16(acc + bias)                         (F.linear, store.py:289-293) */
  FB_EPI_STORE_F32 = 1,      /* out f32 = f32(bf16(acc + bias))         (F.linear(...).float(), flux.py:343, :536) */
  FB_EPI_GELU = 2,           /* out bf16 = bf16(gelu_tanh(bf16(acc + bias)))           (flux.py:194-195 after :319) */
  FB_EPI_GATED_RESIDUAL = 3, /* out f32 = resid + gate[b] * f32(bf16(acc + bias))         (flux.py:169-171, :141-143) */
  FB_EPI_QKV = 4             /* QK-RMSNorm + RoPE into q/k, v copied, heads split; columns >= qkv_cols
                                go through GELU into out (flux.py:179-191, :331-336) */
};

/* One Linear y = A W^T (+ bias) with a fused epilogue. */
typedef struct fb_linear {
  /* operands */
  const uint16_t* a; int64_t lda;      /* bf16 activations [m, k], row stride lda (multiple of 8) */
  const uint16_t* w; int64_t ldw;      /* bf16 weight [n, k] (nn.Linear layout); NULL when NF4 */
  const uint8_t* w_nf4;                /* NF4 weight: packed [n*k/2], high nibble = even element */
  const float* absmax;                 /* NF4: fp32 absmax, one per `blocksize` consecutive elements */
  const float* code16;                 /* NF4: the 16-entry fp32 code table (runtime input) */
  int32_t blocksize;                   /* NF4 block size (64 in selas) */
  const uint16_t* bias;                /* bf16 [n] or NULL */
  int32_t m, n, k;
  int32_t rows_per_batch;              /* tokens per image (row / rows_per_batch = image index) */
  /* STORE_BF16 / STORE_F32 / GELU, and the GELU part of QKV */
  void* out; int64_t ld_out;
  /* GATED_RESIDUAL */
  const float* resid; int64_t ld_resid;
  const uint16_t* gate; int64_t gate_batch_stride;   /* bf16 gate[b * stride + col] */
  int32_t guard;                       /* clamp the Linear output to +-65504 first (fp16 guard) */
  /* QKV */
  const float* q_scale; const float* k_scale;        /* fp32 [head_dim] RMSNorm scales */
  const float* rope_cos; const float* rope_sin;      /* fp32 [seq_total, head_dim/2] */
  uint16_t* q; uint16_t* k_out; uint16_t* v;         /* bf16 [batch, heads, seq_total, head_dim] */
  int32_t heads, head_dim, seq_total, seq_offset;    /* this stream's rows land at seq_offset.. */
  int32_t qkv_cols;                                  /* 3 * heads * head_dim */
  int32_t gelu_col0;                                 /* GELU columns land at out[:, gelu_col0 + (n - qkv_cols)] */
  /* int8_row weight (selas --quant int8 containers): q int8 [n, k] row-major and one fp32 scale per
   * row; decoded in the GEMM mainloop as w = bf16(float(q) * float(bf16(scale[row]))), bit-identical to
   * selas/codecs.py:272-276. w and w_nf4 NULL; k % 64 == 0. */
  const int8_t* w_i8;
  const float* w_scale;
  /* fp8 weight stored raw (selas keeps fp8 sources as-is and casts at use, convert.py:178-180): [n, k]
   * row-major bytes, e4m3fn (w_f8_e5m2 = 0) or e5m2 (1); decoded exactly to bf16 in the GEMM mainloop.
   * w, w_nf4 and w_i8 NULL; k % 64 == 0. */
  const uint8_t* w_f8;
  int32_t w_f8_e5m2;
  /* QKV, sequence parallel (Ulysses over sp_world ranks, one image; 0 = off): instead of q/k/v, head h
   * of this rank's tokens is stored straight into rank g = h / (heads / sp_world)'s buffer sp_qkv_dst[g]
   * (a peer pointer, e.g. from fb_ipc_open), laid out [3][heads/sp_world][sp_world * seq_total][head_dim]
   * with this rank's tokens at rows sp_rank * seq_total + position: the all-to-all before attention,
   * done by the epilogue's stores over NVLink. */
  uint16_t* sp_qkv_dst[8];
  int32_t sp_world, sp_rank;
} fb_linear;

/* One-time set-up (thread-safe, idempotent): checks for an sm_100 device, resolves the driver's
 * cuTensorMapEncodeTiled, raises the kernels' shared-memory limits, allocates the status word. */
int32_t fb_init(void);
const char* fb_last_error(void);
/* Synchronously reads the current device's status word (an fb_device_code); clears it if asked. */
int32_t fb_device_status(int32_t* code, int32_t clear);
/* Library build identifier ("flux_b200 sm_100a <date>"). */
const char* fb_version(void);
/* Self-test of the device-side failure path (no counterpart in the reference): launches one kernel
 * whose bounded wait on an mbarrier that nothing completes runs out after budget_ms (1..1000); it
 * records FB_DEV_TIMEOUT_EPI in the status word and returns, leaving the context usable, exactly as a
 * real kernel's timed-out wait does. Read the code with fb_device_status. */
int32_t fb_selftest_wait_timeout(int32_t budget_ms, void* stream);

/* NF4 decode, bit-exact: out[2i] = cast(code[p[i] >> 4] * absmax[2i / bs]), out[2i+1] with p[i] & 15.
 * Replaces selas/codecs.py:178-199 (nf4_dequant_torch) and :207-228 (the Triton kernel).
 * out_dtype: FB_F32 / FB_F16 / FB_BF16. blocksize even; n_bytes * 2 divisible by blocksize. */
int32_t fb_nf4_dequant(const uint8_t* packed, const float* absmax, const float* code16, int64_t n_bytes,
                       int32_t blocksize, void* out, int32_t out_dtype, void* stream);

/* out = bf16(LayerNorm(x) * (1 + scale[b]) + shift[b]), eps 1e-6, no affine; x fp32 [rows, dim].
 * Replaces the `_mod_in` segment, selas/models/flux.py:164-166 (with `_ln`, :146-147).
 * shift/scale are bf16 rows indexed by b = row / rows_per_batch with stride mod_batch_stride. */
int32_t fb_ln_mod(const float* x, int64_t rows, int32_t dim, int32_t rows_per_batch, const uint16_t* shift,
                  const uint16_t* scale, int64_t mod_batch_stride, uint16_t* out, void* stream);

/* One fb_ln_mod problem (the arguments of fb_ln_mod, field for field). */
typedef struct fb_ln_mod_problem {
  const float* x;
  int64_t rows;
  int32_t dim;
  int32_t rows_per_batch;
  const uint16_t* shift;
  const uint16_t* scale;
  int64_t mod_batch_stride;
  uint16_t* out;
} fb_ln_mod_problem;

/* `count` (1 or 2) fb_ln_mod problems, in one launch when both have dim 3072: the `_mod_in` calls of
 * a double block's img and txt streams, selas/models/flux.py:306-307 and :318/:321 (through
 * `_gated_add_mod`, :174-176). Same arithmetic and checks as fb_ln_mod for each problem. */
int32_t fb_ln_mod_grouped(const fb_ln_mod_problem* problems, int32_t count, void* stream);

/* `count` (1 or 2) Linears in one persistent tcgen05 launch, all with epilogue `epilogue`.
 * Replaces UnitView.linear (selas/store.py:289-293) plus the segment that follows it in
 * double_block / single_block / final_layer (flux.py:300-343). */
int32_t fb_linear_grouped(const fb_linear* problems, int32_t count, int32_t epilogue, void* stream);

/* One NF4 Linear (problem->w_nf4 / absmax / code16 / blocksize set, problem->w NULL) with epilogue
 * `epilogue`. The weight is decoded bit-exactly (as fb_nf4_dequant) into the caller's `workspace` as bf16,
 * whole 256-row chunks of output features at a time when it does not fit at once (workspace_bytes >=
 * min(n, 256) * k * 2 required; 16-byte aligned), and each chunk runs through the tcgen05 GEMM.
 * Replaces UnitView.linear on an NF4 unit: JIT decode (selas/store.py:265-281, codecs.py:260-266)
 * followed by F.linear (store.py:289-293). The workspace is scratch: its contents are overwritten. */
int32_t fb_linear_nf4(const fb_linear* problem, int32_t epilogue, void* workspace, int64_t workspace_bytes,
                      void* stream);

/* fb_linear_nf4 for callers that cannot allocate device memory. It has no counterpart in the
 * reference: selas always lets torch allocate the decoded weight. Here the decode workspace and the
 * status word live in one fixed 16 MiB array of device memory built into the library, so nothing is
 * allocated (no cudaMalloc, no fb_init status word, no workspace argument). Limits: min(n, 256) * k * 2
 * bytes must fit in that array (k <= 32767 for n >= 256); larger problems return FB_ERR_ARG before
 * launching. All calls share the array: calls whose work overlaps on the GPU race, so keep them on
 * one stream. The first call on a device does the set-up; make it before any stream capture.
 * A kernel of this path that gives up on a bounded wait records its fb_device_code in the array's
 * first word (not in the word fb_device_status reads); read it with fb_linear_nf4_static_status. */
int32_t fb_linear_nf4_static(const fb_linear* problem, int32_t epilogue, void* stream);
/* The status word of fb_linear_nf4_static (no counterpart in the reference), read without allocating:
 * waits for all work on the current device (cudaDeviceSynchronize), copies the word from the fixed
 * array and clears it if `clear` is set. *code = 0 when no call of this path timed out since the last
 * clearing read (or none ran on this device). The word is sticky: calls never clear it, so read it
 * after the calls whose results you are about to use, outside any stream capture. */
int32_t fb_linear_nf4_static_status(int32_t* code, int32_t clear);
/* Self-test of that status word (no counterpart in the reference): fb_selftest_wait_timeout's kernel,
 * recording its FB_DEV_TIMEOUT_EPI in the fixed array's status word instead of fb_device_status's. */
int32_t fb_selftest_static_wait_timeout(int32_t budget_ms, void* stream);

/* Flash attention forward, non-causal, no mask: out[b, l, h*Dh + d] = softmax(q k^T * scale) v.
 * q, k, v bf16 [batch, heads, seq, head_dim]; out row stride ld_out (elements). head_dim = 128.
 * Replaces `_attention`, selas/models/flux.py:135-138 (SDPA + transpose + reshape). */
int32_t fb_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out, int64_t ld_out,
                     int32_t batch, int32_t heads, int32_t seq, int32_t head_dim, float scale, void* stream);

/* Same, with the output rows of each image split in two: rows [0, split) go to
 * out0[(b * split + l) * ld0 + h*Dh + d] and rows [split, seq) to out1[(b * (seq - split) + l - split) * ld1 + ...].
 * The double block's txt (first L_txt rows) and img streams land in separate per-stream buffers
 * (selas/models/flux.py:314-316: attn[:, :lt], attn[:, lt:]). */
int32_t fb_attention_split(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out0, int64_t ld0,
                           uint16_t* out1, int64_t ld1, int32_t split, int32_t batch, int32_t heads, int32_t seq,
                           int32_t head_dim, float scale, void* stream);

/* Elementwise segments, for callers that keep selas's segment-level structure. */
/* out = x + g[b] * f32(y) (y clamped to +-65504 when guard); flux.py:169-171. x,out fp32; y,g bf16. */
int32_t fb_gated_add(const float* x, const uint16_t* g, const uint16_t* y, float* out, int64_t rows, int32_t dim,
                     int32_t rows_per_batch, int64_t g_batch_stride, int32_t guard, void* stream);
/* out = bf16(gelu_tanh(f32(h))) over n elements; flux.py:194-195. */
int32_t fb_gelu_tanh(const uint16_t* h, uint16_t* out, int64_t n, void* stream);
/* QK-RMSNorm + RoPE + head split of one stream's qkv [batch, rows, 3*heads*hd] (row stride ld_qkv)
 * into q/k/v [batch, heads, seq_total, hd] at rows seq_offset..; flux.py:179-191. */
int32_t fb_qk_norm_rope(const uint16_t* qkv, int64_t ld_qkv, int32_t batch, int32_t rows, int32_t heads,
                        int32_t head_dim, const float* q_scale, const float* k_scale, const float* rope_cos,
                        const float* rope_sin, uint16_t* q, uint16_t* k, uint16_t* v, int32_t seq_total,
                        int32_t seq_offset, void* stream);

/* ---- sequence parallelism over NVLink (Ulysses, one image; no counterpart in the reference, which has
 * no multi-GPU path). Buffers are shared between the ranks' processes with CUDA IPC; the two
 * all-to-alls of Ulysses attention are done by the kernels' own stores into the peers' buffers, with
 * fb_peer_barrier between the steps. */

/* Attention over the gathered sequence of sp_world * seq_local tokens (q/k/v [heads, sp_world *
 * seq_local, head_dim] bf16, this rank's head group) whose output row t is stored straight into rank
 * t / seq_local's buffer: out_peers[t / seq_local] + (t % seq_local) * ld_out + col0 + h*Dh + d. */
int32_t fb_attention_sp(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* const* out_peers,
                        int64_t ld_out, int32_t col0, int32_t heads, int32_t seq_local, int32_t sp_world,
                        int32_t head_dim, float scale, void* stream);

/* CUDA IPC of a device buffer: export writes the 64-byte handle of the allocation that holds ptr and
 * the offset of ptr inside it; open maps another process's buffer (peer_ptr = its base + offset;
 * peer_base is what close takes). */
int32_t fb_ipc_export(const void* ptr, void* handle64, int64_t* offset);
int32_t fb_ipc_open(const void* handle64, int64_t offset, void** peer_ptr, void** peer_base);
int32_t fb_ipc_close(void* peer_base);

/* Device-side barrier of `world` ranks, stream-ordered: flags[r] points to rank r's int32 flag array
 * (world entries; a peer pointer for r != rank, zero-initialised once). The kernel stores `epoch` (which
 * must grow by one per barrier) into every rank's flags[rank] with release semantics, then waits with
 * acquire loads until its own array holds `epoch` from every rank; a wait longer than timeout_ms records
 * FB_DEV_TIMEOUT_PEER in the status word and returns. */
int32_t fb_peer_barrier(int32_t* const* flags, int32_t world, int32_t rank, int32_t epoch, int32_t timeout_ms,
                        void* stream);

/* ---- weight encoders (conversion time), bit-exact with selas's torch encoders ----
 * NF4 (selas/codecs.py:99-119): w (n values, FB_F32 / FB_BF16 / FB_F16) in blocks of `blocksize` (even,
 * dividing n) -> packed [n / 2] (first value of a pair in the high nibble) and absmax [n / blocksize];
 * code index = number of midpoints (code16[i] + code16[i+1]) / 2 strictly below w / absmax. */
int32_t fb_nf4_encode(const void* w, int32_t w_dtype, int64_t n, int32_t blocksize, const float* code16,
                      uint8_t* packed, float* absmax, void* stream);
/* int8_row (selas/codecs.py:87-97): w [rows, cols] -> q int8 [rows, cols] = clamp(round_half_even(w / scale),
 * -127, 127), scale [rows] = absmax / 127 (1 for an all-zero row). */
int32_t fb_int8_row_encode(const void* w, int32_t w_dtype, int64_t rows, int64_t cols, int8_t* q, float* scale,
                           void* stream);

/* ---- step cache (selas/stepcache.py): the probe distance and the residual arithmetic ----
 * Replaces the torch expressions of StepCache.decide (selas/stepcache.py:127-129), _Hist.predict
 * (:84-94) and the residual captures / adds of FluxRunner.step (selas/models/flux.py:548, 553, 559-580).
 * All arrays are contiguous with n % 4 == 0 elements; f32 arrays 16-byte aligned. */
#define FB_PROBE_WORK_DOUBLES 4096

/* r = x - x_in (x_in NULL: r = x), stored to resid when it is not NULL. With ref: work[0] = sum |r - ref|,
 * work[1] = sum |ref| (fp64; work = FB_PROBE_WORK_DOUBLES doubles of device memory), so that the
 * reference's distance is (work[0] / n) / max(work[1] / n, 1e-12). */
int32_t fb_probe_distance(const float* x, const float* x_in, const float* ref, float* resid, int64_t n, double* work,
                          void* stream);

/* p = r1 + a * (r1 - r0) (r0 NULL: p = r1), out = x + p (x NULL: out = p); r1/r0 FB_F32 or FB_BF16,
 * every operation an fp32 operation rounded once. */
int32_t fb_residual_predict(const float* x, const void* r1, const void* r0, int32_t r_dtype, float a, float* out,
                            int64_t n, void* stream);

/* r = x - x0, stored as FB_F32 or FB_BF16 (round to nearest even). */
int32_t fb_residual_diff(const float* x, const float* x0, void* r, int32_t r_dtype, int64_t n, void* stream);

/* ---- FLUX autoencoder decoder (selas/models/vae.py:42-96) ----
 * Activations are NHWC fp32: [B, H, W, C] with a pixel stride ld >= C (a multiple of 4 floats); every
 * pointer 16-byte aligned. The products run on the tensor cores as tf32 x tf32 -> fp32 (the arithmetic
 * of torch's fp32 convolutions on tensor-core GPUs). */
enum fb_vae_conv_flags {
  FB_VAE_ROUND_OUT = 1,       /* round the outputs to tf32 (they feed another tensor-core product) */
  FB_VAE_OUT_NCHW_CLAMP = 2   /* store NCHW [B, Cout, H, W] clamped to [-1, 1] (the last conv, vae.py:95-96) */
};

/* F.conv2d(x, w, b, padding=ksize/2) (vae.py:51-52), stride 1, ksize 1 or 3, as an implicit GEMM:
 * out[b,y,x,n] = bias[n] + sum_{r,s,c} in[b, y+r-k/2, x+s-k/2, c] * weight[r*k+s][n][c] (+ resid[b,y,x,n]).
 * weight is tap-major [ksize*ksize][cout][cin] (row stride ld_w >= cin, tap stride cout * ld_w), i.e.
 * torch's [cout, cin, k, k] permuted to [k, k, cout, cin]; cin % 32 == 0 (pad with zero channels);
 * bias and resid may be NULL. */
int32_t fb_vae_conv(const float* in, int64_t ld_in, int32_t batch, int32_t h, int32_t w, int32_t cin, const float* weight,
                    int64_t ld_w, int32_t cout, int32_t ksize, const float* bias, const float* resid, int64_t ld_resid,
                    float* out, int64_t ld_out, int32_t flags, void* stream);

/* F.group_norm(x, 32, gamma, beta, eps) (vae.py:54-55), then SiLU when silu != 0 (vae.py:58, 60, 94), then
 * tf32 rounding when round_tf32 != 0; c in {128, 256, 512, 1024}; hw = H*W pixels per image. work: device
 * memory of fb_vae_group_norm_work_doubles(batch) doubles. Statistics in fp64, reduced in a fixed order. */
int32_t fb_vae_group_norm(const float* x, int64_t ld, int32_t batch, int64_t hw, int32_t c, const float* gamma,
                          const float* beta, float eps, int32_t silu, int32_t round_tf32, float* out, int64_t ld_out,
                          double* work, void* stream);
int64_t fb_vae_group_norm_work_doubles(int32_t batch);

/* The decoder's last two layers in one call: F.group_norm(x, 32, gamma, beta, eps) and SiLU (norm_out,
 * vae.py:94), then the 3x3 conv to the image channels with its bias (conv_out, vae.py:95), clamped to
 * [-1, 1] and written NCHW fp32 [batch, 3, h, w]. x is NHWC fp32 [batch, h, w, 128], contiguous. The
 * conv reads the normalised values rounded to tf32, as fb_vae_group_norm + fb_vae_conv would give it.
 * weight: the tap-major tf32 weights [9][3][128] as fb_vae_conv takes them; bias: 3 values or NULL.
 * work as for fb_vae_group_norm. c must be 128 and cout 3 (FLUX's decoder); other shapes return
 * FB_ERR_UNSUPPORTED. */
int32_t fb_vae_norm_out_conv(const float* x, int32_t batch, int32_t h, int32_t w, int32_t c, const float* gamma,
                             const float* beta, float eps, const float* weight, const float* bias, int32_t cout,
                             float* out, double* work, void* stream);

/* F.interpolate(x, scale_factor=2, mode="nearest") (vae.py:90): [B, H, W, C] -> [B, 2H, 2W, C], c % 4 == 0. */
int32_t fb_vae_upsample2(const float* in, int32_t batch, int32_t h, int32_t w, int32_t c, int32_t round_tf32, float* out,
                         void* stream);

/* In place, per row: s = softmax(s * scale) over n columns (the softmax of the mid-block attention,
 * vae.py:71); n % 4 == 0, n <= 32768. */
int32_t fb_vae_softmax_rows(float* s, int64_t rows, int32_t n, int64_t ld, float scale, int32_t round_tf32,
                            void* stream);

/* out[c, r] = in[r, c]: in [rows, cols] (row stride ld_in) -> out [cols, rows] (row stride ld_out). */
int32_t fb_vae_transpose(const float* in, int32_t rows, int32_t cols, int64_t ld_in, float* out, int64_t ld_out,
                         void* stream);

/* z [B, zc, H, W] NCHW -> [B, H, W, cpad] NHWC of tf32(z / scale + shift), channels zc..cpad zero (vae.py:82). */
int32_t fb_vae_latent_prep(const float* z, int32_t batch, int32_t zc, int32_t h, int32_t w, int32_t cpad, float scale,
                           float shift, float* out, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* FLUX_B200_H */
