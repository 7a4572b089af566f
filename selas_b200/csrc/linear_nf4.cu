// linear_nf4.cu — an NF4 Linear as one call: decode the packed weight into a bf16 workspace with the
// bit-exact NF4 kernel, then run the tcgen05 GEMM (with the problem's fused epilogue) on it. This is
// selas's just-in-time decode point (store.py:265-281 -> codecs.py:260-266 -> F.linear) moved onto
// the device behind the C-ABI. When the workspace cannot hold the whole weight, the output features
// are processed in chunks of whole 256-row tiles.
#include "fb_internal.h"

namespace fb {

int launch_linear_nf4(const fb_linear& L, int epi, void* ws, int64_t ws_bytes, int* status, int sm_count,
                      cudaStream_t st, std::string& err) {
  if (!L.w_nf4 || !L.absmax || !L.code16) {
    err = "fb_linear_nf4: w_nf4, absmax and code16 are required";
    return FB_ERR_ARG;
  }
  const int64_t n = L.n, k = L.k, bs = L.blocksize;
  if (n <= 0 || k <= 0 || L.m < 0 || bs <= 0 || bs % 2 != 0 || (n * k) % bs != 0 || k % 8 != 0) {
    err = "fb_linear_nf4: need n, k > 0, k % 8 == 0 and an even blocksize dividing n*k";
    return FB_ERR_ARG;
  }
  if (!ws || (reinterpret_cast<uintptr_t>(ws) & 15u) != 0) {
    err = "fb_linear_nf4: the workspace must be a 16-byte aligned device pointer";
    return FB_ERR_ALIGN;
  }
  const int64_t fit = ws_bytes / (k * 2);
  const int64_t rows = fit >= n ? n : (fit / 256) * 256;
  if (rows <= 0) {
    err = "fb_linear_nf4: workspace too small: it must hold at least min(n, 256) * k bf16 values (" +
          std::to_string(std::min<int64_t>(n, 256) * k * 2) + " bytes)";
    return FB_ERR_ARG;
  }
  if (rows < n && (rows * k) % bs != 0) {
    err = "fb_linear_nf4: a chunked decode needs whole NF4 blocks per chunk (256 * k % blocksize == 0)";
    return FB_ERR_ARG;
  }
  const size_t out_esize = (epi == FB_EPI_STORE_F32 || epi == FB_EPI_GATED_RESIDUAL) ? 4 : 2;
  for (int64_t n0 = 0; n0 < n; n0 += rows) {
    const int64_t r = std::min(rows, n - n0);
    cudaError_t e = launch_nf4_dequant(L.w_nf4 + n0 * k / 2, L.absmax + n0 * k / bs, L.code16, r * k / 2,
                                       static_cast<int>(bs), ws, FB_BF16, st);
    if (e != cudaSuccess) {
      err = std::string("fb_linear_nf4: decode launch: ") + cudaGetErrorString(e);
      return FB_ERR_CUDA;
    }
    fb_linear sub = L;
    sub.w = static_cast<const uint16_t*>(ws);
    sub.ldw = k;
    sub.w_nf4 = nullptr;
    sub.n = static_cast<int32_t>(r);
    sub.bias = L.bias ? L.bias + n0 : nullptr;
    if (epi != FB_EPI_QKV) {
      sub.out = L.out ? static_cast<char*>(L.out) + n0 * out_esize : nullptr;
      sub.resid = L.resid ? L.resid + n0 : nullptr;
      sub.gate = L.gate ? L.gate + n0 : nullptr;
    }
    const int off = static_cast<int>(n0);
    const int rc = launch_linear_on(&sub, 1, epi, &off, status, sm_count, st, err);
    if (rc) return rc;
  }
  return FB_OK;
}

}  // namespace fb
