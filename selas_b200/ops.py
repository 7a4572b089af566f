"""Tensor-level wrappers over the C-ABI: validate torch tensors, pass raw pointers and the current
stream. Every function launches on ``torch.cuda.current_stream()`` and never synchronises.

The wrappers raise ``FluxB200Error`` for anything the kernels do not handle; there is no CPU path.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _lib
from . import profile as _prof
from ._lib import FluxB200Error

BF16, F32 = torch.bfloat16, torch.float32
_DTYPE_CODE = {torch.float32: _lib.FB_F32, torch.float16: _lib.FB_F16, torch.bfloat16: _lib.FB_BF16}


_launches = 0


def launch_count_reset() -> None:
    global _launches
    _launches = 0


def launch_count() -> int:
    """Kernels launched through this module since the last reset (one per C-ABI compute call)."""
    return _launches


def _count() -> None:
    global _launches
    _launches += 1


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _need(cond: bool, msg: str) -> None:
    if not cond:
        raise FluxB200Error(msg)


def _cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise FluxB200Error("libflux_b200 tensors must be CUDA tensors (there is no CPU path)")


# ------------------------------------------------------------------------------------------ NF4


def nf4_dequant(packed: torch.Tensor, absmax: torch.Tensor, blocksize: int, code, shape, dtype: torch.dtype,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """Bit-exact NF4 decode with the signature of ``selas.codecs.nf4_dequant`` (codecs.py:260-266)."""
    _cuda(packed, absmax)
    _need(packed.dtype == torch.uint8 and absmax.dtype == F32, "nf4_dequant: packed uint8 and absmax fp32 required")
    _need(dtype in _DTYPE_CODE, f"nf4_dequant: unsupported output dtype {dtype}")
    packed = packed.contiguous()
    absmax = absmax.contiguous()
    code_t = code if isinstance(code, torch.Tensor) else torch.tensor(tuple(code), dtype=F32)
    code_t = code_t.to(device=packed.device, dtype=F32).contiguous()
    _need(code_t.numel() == 16, "nf4_dequant: the code table needs 16 entries")
    n_bytes = packed.numel()
    if out is None:
        out = torch.empty(n_bytes * 2, dtype=dtype, device=packed.device)
    _need(out.numel() == 2 * n_bytes and out.is_contiguous() and out.dtype == dtype, "nf4_dequant: bad out tensor")
    _need(absmax.numel() * int(blocksize) == 2 * n_bytes, "nf4_dequant: absmax size does not match the blocksize")
    if n_bytes:
        with _prof.region("nf4_dequant", 0.0, n_bytes * (1 + 2 * out.element_size()) + absmax.numel() * 4):
            _lib.check(_lib.lib().fb_nf4_dequant(packed.data_ptr(), absmax.data_ptr(), code_t.data_ptr(), n_bytes,
                                                 int(blocksize), out.data_ptr(), _DTYPE_CODE[dtype], _stream()),
                       "fb_nf4_dequant")
        _count()
    return out.view(tuple(shape))


# ------------------------------------------------------------------------------------------ glue


def _mod_rows(v: torch.Tensor, batch: int, dim: int) -> tuple[torch.Tensor, int]:
    """A [B, dim] (or [B, 1, dim]) bf16 view whose rows may be strided: returns (tensor, batch stride)."""
    v = v.reshape(v.shape[0], -1) if v.dim() == 3 else v
    _need(v.dtype == BF16, "modulation vectors must be bf16")
    _need(v.shape[-1] == dim and v.stride(-1) == 1, "modulation row must be contiguous with the model width")
    _need(v.shape[0] in (1, batch), "modulation batch does not match")
    stride = v.stride(0) if v.shape[0] > 1 else 0
    return v, stride


def ln_mod(x: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """bf16(LayerNorm(x) * (1 + scale) + shift) for x fp32 [B, L, D]; shift/scale bf16 [B, D] views
    (the ``_mod_in`` segment, flux.py:164-166)."""
    _cuda(x, shift, scale)
    _need(x.dtype == F32 and x.is_contiguous() and x.dim() == 3, "ln_mod: x must be contiguous fp32 [B, L, D]")
    b, l, d = x.shape
    sh, s_sh = _mod_rows(shift, b, d)
    sc, s_sc = _mod_rows(scale, b, d)
    _need(s_sh == s_sc, "ln_mod: shift and scale must share a batch stride")
    if out is None:
        out = torch.empty(b, l, d, dtype=BF16, device=x.device)
    with _prof.region("ln_mod", 0.0, b * l * d * 6 + 2 * b * d * 2):
        _lib.check(_lib.lib().fb_ln_mod(x.data_ptr(), b * l, d, max(l, 1), sh.data_ptr(), sc.data_ptr(), s_sh,
                                        out.data_ptr(), _stream()), "fb_ln_mod")
    _count()
    return out


def ln_mod_grouped(items: list) -> list[torch.Tensor]:
    """``ln_mod`` of each (x, shift, scale) in ``items`` (one or two), in one launch when the two share
    dim 3072 (``fb_ln_mod_grouped``): the img and txt streams of a double block."""
    _need(1 <= len(items) <= 2, "ln_mod_grouped: one or two problems")
    probs, outs, nbytes = [], [], 0
    for x, shift, scale in items:
        _cuda(x, shift, scale)
        _need(x.dtype == F32 and x.is_contiguous() and x.dim() == 3, "ln_mod: x must be contiguous fp32 [B, L, D]")
        b, l, d = x.shape
        sh, s_sh = _mod_rows(shift, b, d)
        sc, s_sc = _mod_rows(scale, b, d)
        _need(s_sh == s_sc, "ln_mod: shift and scale must share a batch stride")
        out = torch.empty(b, l, d, dtype=BF16, device=x.device)
        probs.append(_lib.FbLnModProblem(x.data_ptr(), b * l, d, max(l, 1), sh.data_ptr(), sc.data_ptr(), s_sh,
                                         out.data_ptr()))
        outs.append(out)
        nbytes += b * l * d * 6 + 2 * b * d * 2
    arr = (_lib.FbLnModProblem * len(probs))(*probs)
    with _prof.region("ln_mod", 0.0, nbytes):
        _lib.check(_lib.lib().fb_ln_mod_grouped(ctypes.addressof(arr), len(probs), _stream()), "fb_ln_mod_grouped")
    _count()
    return outs


def gated_add(x: torch.Tensor, g: torch.Tensor, y: torch.Tensor, guard: bool) -> torch.Tensor:
    """x + g * f32(y) (the ``_gated_add`` segment, flux.py:169-171): x fp32 [B, L, D], y bf16, g bf16 [B, 1, D]."""
    _cuda(x, g, y)
    _need(x.dtype == F32 and x.is_contiguous() and x.dim() == 3, "gated_add: x must be contiguous fp32 [B, L, D]")
    _need(y.dtype == BF16 and y.is_contiguous() and y.shape == x.shape, "gated_add: y must be contiguous bf16 like x")
    b, l, d = x.shape
    gv, gs = _mod_rows(g, b, d)
    out = torch.empty_like(x)
    with _prof.region("gated_add", 0.0, b * l * d * 10):
        _lib.check(_lib.lib().fb_gated_add(x.data_ptr(), gv.data_ptr(), y.data_ptr(), out.data_ptr(), b * l, d, max(l, 1),
                                           gs, int(bool(guard)), _stream()), "fb_gated_add")
    _count()
    return out


def gelu_tanh(h: torch.Tensor) -> torch.Tensor:
    """bf16 GELU (tanh approximation) of a bf16 tensor (the ``_gelu`` segment, flux.py:194-195)."""
    _cuda(h)
    _need(h.dtype == BF16 and h.is_contiguous() and h.numel() % 8 == 0, "gelu_tanh: contiguous bf16, numel % 8 == 0")
    out = torch.empty_like(h)
    with _prof.region("gelu", 0.0, h.numel() * 4):
        _lib.check(_lib.lib().fb_gelu_tanh(h.data_ptr(), out.data_ptr(), h.numel(), _stream()), "fb_gelu_tanh")
    _count()
    return out


def qk_norm_rope(qkv: torch.Tensor, heads: int, q_scale: torch.Tensor, k_scale: torch.Tensor, cos: torch.Tensor,
                 sin: torch.Tensor, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, seq_offset: int) -> None:
    """QK-RMSNorm + RoPE + head split of one stream's qkv [B, Ls, 3*H*hd] (a view with unit column
    stride) into q/k/v [B, H, L, hd] at rows seq_offset.. (flux.py:179-191)."""
    _cuda(qkv, q_scale, k_scale, cos, sin, q, k, v)
    b, ls, c = qkv.shape
    hd = c // (3 * heads)
    _need(qkv.dtype == BF16 and qkv.stride(2) == 1 and qkv.stride(0) == ls * qkv.stride(1),
          "qk_norm_rope: qkv must be bf16 rows with a uniform row stride")
    for t in (q, k, v):
        _need(t.dtype == BF16 and t.is_contiguous() and t.shape[0] == b and t.shape[1] == heads and t.shape[3] == hd,
              "qk_norm_rope: q/k/v must be contiguous bf16 [B, H, L, hd]")
    with _prof.region("qk_norm_rope", 0.0, b * ls * c * 4):
        _lib.check(_lib.lib().fb_qk_norm_rope(qkv.data_ptr(), qkv.stride(1), b, ls, heads, hd, q_scale.data_ptr(),
                                              k_scale.data_ptr(), cos.data_ptr(), sin.data_ptr(), q.data_ptr(),
                                              k.data_ptr(), v.data_ptr(), q.shape[2], seq_offset, _stream()),
                   "fb_qk_norm_rope")
    _count()


# ------------------------------------------------------------------------------------------ attention


def attention_sp(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out_peers: list[int], ld_out: int, col0: int,
                 seq_local: int) -> None:
    """``fb_attention_sp``: attention over the gathered sequence (q/k/v [hp, P * seq_local, 128], this
    rank's head group) whose output row t is stored into rank t // seq_local's buffer out_peers[...]
    at row t % seq_local, columns col0 .. col0 + hp*128 (selas/models/flux.py:135-138 per head)."""
    _cuda(q, k, v)
    hp, l, hd = q.shape
    for t in (q, k, v):
        _need(t.dtype == BF16 and t.is_contiguous() and tuple(t.shape) == (hp, l, hd), "attention_sp: q/k/v layout")
    world = len(out_peers)
    _need(l == world * seq_local, "attention_sp: sequence must be world * seq_local")
    arr = (ctypes.c_void_p * world)(*out_peers)
    flops = 4.0 * hp * l * l * hd
    with _prof.region("attention", flops, 4.0 * hp * l * hd * 2):
        _lib.check(_lib.lib().fb_attention_sp(q.data_ptr(), k.data_ptr(), v.data_ptr(), arr, int(ld_out), int(col0),
                                              hp, int(seq_local), world, hd, 1.0 / math.sqrt(hd), _stream()),
                   "fb_attention_sp")
    _count()


def peer_barrier(flag_ptrs: list[int], rank: int, epoch: int, timeout_ms: int) -> None:
    """``fb_peer_barrier``: stream-ordered device-side barrier of the ranks whose flag arrays are given."""
    arr = (ctypes.c_void_p * len(flag_ptrs))(*flag_ptrs)
    _lib.check(_lib.lib().fb_peer_barrier(arr, len(flag_ptrs), int(rank), int(epoch), int(timeout_ms), _stream()),
               "fb_peer_barrier")
    _count()



def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor | None = None,
              split: int | None = None, out_first: torch.Tensor | None = None) -> torch.Tensor:
    """softmax(q k^T / sqrt(hd)) v for q/k/v bf16 [B, H, L, 128] into out [B, L, H*128] (a view whose
    rows may be strided, e.g. the first columns of the single block's linear2 input). With ``split``,
    rows [0, split) of each image go to ``out_first`` [B, split, H*128] instead (flux.py:135-138, :314-316)."""
    _cuda(q, k, v)
    b, h, l, hd = q.shape
    for t in (q, k, v):
        _need(t.dtype == BF16 and t.is_contiguous() and tuple(t.shape) == (b, h, l, hd), "attention: q/k/v layout")
    split = 0 if split is None else int(split)
    if out is None:
        out = torch.empty(b, l - split, h * hd, dtype=BF16, device=q.device)

    def rows(t, n):
        _need(t.dtype == BF16 and t.shape[-1] == h * hd and t.stride(-1) == 1, "attention: output rows")
        if b > 1:
            _need(t.stride(0) == n * t.stride(1), "attention: output rows must be uniformly strided across images")
        return t.stride(1)

    ld1 = rows(out, l - split)
    flops = 4.0 * b * h * l * l * hd
    with _prof.region("attention", flops, 4.0 * b * h * l * hd * 2):
        _attention_launch(q, k, v, out, ld1, split, out_first, rows, b, h, l, hd)
    _count()
    return out


def _attention_launch(q, k, v, out, ld1, split, out_first, rows, b, h, l, hd) -> None:
    if split:
        _need(out_first is not None, "attention: split needs out_first")
        ld0 = rows(out_first, split)
        fn = _lib.lib().fb_attention_split
        _lib.check(fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), out_first.data_ptr(), ld0, out.data_ptr(), ld1, split, b, h,
                      l, hd, ctypes.c_float(1.0 / math.sqrt(hd)), _stream()), "fb_attention_split")
    else:
        _lib.check(_lib.lib().fb_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), ld1, b, h, l, hd,
                                           ctypes.c_float(1.0 / math.sqrt(hd)), _stream()), "fb_attention")


# ------------------------------------------------------------------------------------------ linear


def make_linear(a: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None, rows_per_batch: int) -> _lib.FbLinear:
    """An fb_linear for y = a w^T + bias with a [M, K] (row stride allowed) and w [N, K] bf16."""
    _cuda(a, w, bias)
    _need(a.dtype == BF16 and w.dtype == BF16, "linear: bf16 activations and weight required")
    _need(a.dim() == 2 and w.dim() == 2 and a.stride(1) == 1 and w.stride(1) == 1, "linear: row-major 2-D operands")
    _need(a.shape[1] == w.shape[1], f"linear: K mismatch {tuple(a.shape)} x {tuple(w.shape)}")
    p = _lib.FbLinear()
    p.a, p.lda = a.data_ptr(), a.stride(0)
    p.w, p.ldw = w.data_ptr(), w.stride(0)
    if bias is not None:
        _need(bias.dtype == BF16 and bias.is_contiguous() and bias.numel() == w.shape[0], "linear: bf16 bias [N]")
        p.bias = bias.data_ptr()
    p.m, p.n, p.k = a.shape[0], w.shape[0], a.shape[1]
    p.rows_per_batch = max(int(rows_per_batch), 1)
    return p


def run_linears(problems: list[_lib.FbLinear], epilogue: int) -> None:
    arr = (_lib.FbLinear * len(problems))(*problems)
    flops = sum(2.0 * p.m * p.n * p.k for p in problems)
    nbytes = sum(2.0 * (p.m * p.k + p.n * p.k + p.m * p.n) for p in problems)
    with _prof.region("gemm", flops, nbytes):
        _lib.check(_lib.lib().fb_linear_grouped(ctypes.addressof(arr), len(problems), epilogue, _stream()),
                   "fb_linear_grouped")
    _count()


def make_linear_nf4(a: torch.Tensor, packed: torch.Tensor, absmax: torch.Tensor, code: torch.Tensor, blocksize: int,
                    n: int, bias: torch.Tensor | None, rows_per_batch: int) -> _lib.FbLinear:
    """An fb_linear for y = a W^T + bias with W [n, K] stored as NF4 (packed uint8, fp32 absmax, code)."""
    _cuda(a, packed, absmax, code, bias)
    _need(a.dtype == BF16 and a.dim() == 2 and a.stride(1) == 1, "linear_nf4: bf16 row-major activations")
    _need(packed.dtype == torch.uint8 and packed.is_contiguous() and packed.numel() * 2 == n * a.shape[1],
          "linear_nf4: packed must hold n * K / 2 bytes")
    _need(absmax.dtype == F32 and absmax.is_contiguous() and absmax.numel() * blocksize == n * a.shape[1],
          "linear_nf4: absmax size does not match the blocksize")
    _need(code.dtype == F32 and code.numel() == 16 and code.is_contiguous(), "linear_nf4: 16-entry fp32 code table")
    p = _lib.FbLinear()
    p.a, p.lda = a.data_ptr(), a.stride(0)
    p.w_nf4, p.absmax, p.code16, p.blocksize = packed.data_ptr(), absmax.data_ptr(), code.data_ptr(), int(blocksize)
    if bias is not None:
        _need(bias.dtype == BF16 and bias.is_contiguous() and bias.numel() == n, "linear_nf4: bf16 bias [n]")
        p.bias = bias.data_ptr()
    p.m, p.n, p.k = a.shape[0], int(n), a.shape[1]
    p.rows_per_batch = max(int(rows_per_batch), 1)
    return p


def make_linear_i8(a: torch.Tensor, q: torch.Tensor, scale: torch.Tensor, bias: torch.Tensor | None,
                   rows_per_batch: int) -> _lib.FbLinear:
    """An fb_linear for y = a W^T + bias with W [n, K] stored as int8_row (q int8 [n, K], fp32 scale [n]),
    decoded inside the GEMM's mainloop (selas/codecs.py:272-276)."""
    _cuda(a, q, scale, bias)
    _need(a.dtype == BF16 and a.dim() == 2 and a.stride(1) == 1, "linear_i8: bf16 row-major activations")
    n = q.shape[0]
    _need(q.dtype == torch.int8 and q.dim() == 2 and q.is_contiguous() and q.shape[1] == a.shape[1],
          "linear_i8: q must be int8 [n, K], row-major")
    _need(scale.dtype == F32 and scale.is_contiguous() and scale.numel() == n, "linear_i8: fp32 scale [n]")
    p = _lib.FbLinear()
    p.a, p.lda = a.data_ptr(), a.stride(0)
    p.w_i8, p.w_scale = q.data_ptr(), scale.data_ptr()
    if bias is not None:
        _need(bias.dtype == BF16 and bias.is_contiguous() and bias.numel() == n, "linear_i8: bf16 bias [n]")
        p.bias = bias.data_ptr()
    p.m, p.n, p.k = a.shape[0], int(n), a.shape[1]
    p.rows_per_batch = max(int(rows_per_batch), 1)
    return p


FP8_DTYPES = tuple(getattr(torch, n) for n in ("float8_e4m3fn", "float8_e5m2") if hasattr(torch, n))


def make_linear_f8(a: torch.Tensor, w8: torch.Tensor, bias: torch.Tensor | None, rows_per_batch: int) -> _lib.FbLinear:
    """An fb_linear for y = a W^T + bias with W [n, K] stored raw in fp8 (e4m3fn or e5m2), cast exactly to
    bf16 inside the GEMM's mainloop (selas casts fp8 sources at use: convert.py:178-180)."""
    _cuda(a, w8, bias)
    _need(a.dtype == BF16 and a.dim() == 2 and a.stride(1) == 1, "linear_f8: bf16 row-major activations")
    _need(w8.dtype in FP8_DTYPES and w8.dim() == 2 and w8.is_contiguous() and w8.shape[1] == a.shape[1],
          "linear_f8: w must be fp8 [n, K], row-major")
    n = w8.shape[0]
    p = _lib.FbLinear()
    p.a, p.lda = a.data_ptr(), a.stride(0)
    p.w_f8, p.w_f8_e5m2 = w8.data_ptr(), int(w8.dtype == getattr(torch, "float8_e5m2", None))
    if bias is not None:
        _need(bias.dtype == BF16 and bias.is_contiguous() and bias.numel() == n, "linear_f8: bf16 bias [n]")
        p.bias = bias.data_ptr()
    p.m, p.n, p.k = a.shape[0], int(n), a.shape[1]
    p.rows_per_batch = max(int(rows_per_batch), 1)
    return p


def run_linear_nf4(problem: _lib.FbLinear, epilogue: int, workspace: torch.Tensor) -> None:
    """``fb_linear_nf4``: decode into ``workspace`` (any dtype, used as raw bytes) and run the GEMM."""
    _cuda(workspace)
    _need(workspace.is_contiguous(), "linear_nf4: contiguous workspace")
    nbytes = workspace.numel() * workspace.element_size()
    with _prof.region("gemm_nf4", 2.0 * problem.m * problem.n * problem.k,
                      problem.m * problem.k * 2 + problem.n * problem.k * 0.5625 + problem.m * problem.n * 2):
        _lib.check(_lib.lib().fb_linear_nf4(ctypes.byref(problem), epilogue, workspace.data_ptr(), nbytes, _stream()),
                   "fb_linear_nf4")
    _count()


def run_linear_nf4_static(problem: _lib.FbLinear, epilogue: int) -> None:
    """``fb_linear_nf4_static``: the same Linear decoded into the library's fixed device array, for
    callers that cannot allocate a workspace. Its timeouts are read by ``_lib.raise_on_device_error``
    (through ``fb_linear_nf4_static_status``) once this has been called."""
    _lib.static_used = True
    _lib.check(_lib.load().fb_linear_nf4_static(ctypes.byref(problem), epilogue, _stream()), "fb_linear_nf4_static")
    _count()


def linear(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None, out_dtype: torch.dtype = BF16) -> torch.Tensor:
    """F.linear(x, w, bias) in bf16 (``UnitView.linear``, store.py:289-293); ``out_dtype=float32`` returns
    the bf16 result widened to fp32 (``.float()``)."""
    lead = x.shape[:-1]
    a = x.reshape(-1, x.shape[-1])
    if a.stride(1) != 1:
        a = a.contiguous()
    p = make_linear(a, w, bias, a.shape[0])
    out = torch.empty(a.shape[0], w.shape[0], dtype=out_dtype, device=x.device)
    p.out, p.ld_out = out.data_ptr(), out.stride(0)
    run_linears([p], _lib.FB_EPI_STORE_F32 if out_dtype == F32 else _lib.FB_EPI_STORE_BF16)
    return out.view(*lead, w.shape[0])


# ------------------------------------------------------------------------------------------ step cache

_F32_OR_BF16 = {F32: _lib.FB_F32, BF16: _lib.FB_BF16}
_probe_work: dict[int, torch.Tensor] = {}


def _flat4(t: torch.Tensor, what: str) -> None:
    _need(t.is_contiguous() and t.numel() % 4 == 0, f"{what}: contiguous with a multiple of 4 elements")


def probe_distance(x: torch.Tensor, x_in: torch.Tensor | None, ref: torch.Tensor | None,
                   resid: torch.Tensor | None) -> tuple[float, float] | None:
    """``fb_probe_distance``: r = x - x_in (or x) into ``resid``; with ``ref``, returns (sum|r - ref|,
    sum|ref|) in fp64 (one device->host read of two doubles)."""
    ts = [t for t in (x, x_in, ref, resid) if t is not None]
    _cuda(*ts)
    for t in ts:
        _need(t.dtype == F32 and t.numel() == x.numel(), "probe_distance: fp32 tensors of the same size")
        _flat4(t, "probe_distance")
    work = None
    if ref is not None:
        dev = x.device.index
        work = _probe_work.get(dev)
        if work is None:
            work = _probe_work[dev] = torch.empty(_lib.FB_PROBE_WORK_DOUBLES, dtype=torch.float64, device=x.device)
    _lib.check(_lib.lib().fb_probe_distance(x.data_ptr(), _ptr(x_in), _ptr(ref), _ptr(resid), x.numel(), _ptr(work),
                                            _stream()), "fb_probe_distance")
    _count()
    if ref is None:
        return None
    s = work[:2].tolist()
    return s[0], s[1]


def residual_predict(x: torch.Tensor | None, r1: torch.Tensor, r0: torch.Tensor | None, a: float,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """``fb_residual_predict``: out = x + (r1 + a (r1 - r0)) in fp32 (x None: the prediction alone;
    r0 None: r1). r1/r0 fp32 or bf16."""
    ts = [t for t in (x, r1, r0, out) if t is not None]
    _cuda(*ts)
    _need(r1.dtype in _F32_OR_BF16 and (r0 is None or r0.dtype == r1.dtype), "residual_predict: r1/r0 fp32 or bf16")
    _need(x is None or x.dtype == F32, "residual_predict: x must be fp32")
    for t in ts:
        _need(t.numel() == r1.numel(), "residual_predict: sizes differ")
        _flat4(t, "residual_predict")
    if out is None:
        out = torch.empty(r1.shape, dtype=F32, device=r1.device)
    _need(out.dtype == F32, "residual_predict: out must be fp32")
    _lib.check(_lib.lib().fb_residual_predict(_ptr(x), r1.data_ptr(), _ptr(r0), _F32_OR_BF16[r1.dtype], float(a),
                                              out.data_ptr(), r1.numel(), _stream()), "fb_residual_predict")
    _count()
    return out


def residual_diff(x: torch.Tensor, x0: torch.Tensor, dtype: torch.dtype = F32) -> torch.Tensor:
    """``fb_residual_diff``: (x - x0) as fp32 or bf16."""
    _cuda(x, x0)
    _need(x.dtype == F32 and x0.dtype == F32 and x.shape == x0.shape, "residual_diff: fp32 x and x0 of one shape")
    _need(dtype in _F32_OR_BF16, "residual_diff: dtype fp32 or bf16")
    _flat4(x, "residual_diff")
    _flat4(x0, "residual_diff")
    r = torch.empty(x.shape, dtype=dtype, device=x.device)
    _lib.check(_lib.lib().fb_residual_diff(x.data_ptr(), x0.data_ptr(), r.data_ptr(), _F32_OR_BF16[dtype], x.numel(),
                                           _stream()), "fb_residual_diff")
    _count()
    return r
