"""NF4 codec helpers on the device.

* ``NF4_CODE`` — the 16-level NF4 code book (the QLoRA / bitsandbytes table, as in selas/codecs.py:58-63).
* ``encode_device`` — NF4 encoding of a weight already on the GPU by the ``fb_nf4_encode`` kernel, for
  building quantised models in HBM (conversion time, not the hot path): blockwise absmax, nearest code
  with ties to the lower code, first element in the high nibble (selas/codecs.py:99-119).
* ``decode`` — selas's ``codecs.decode`` entry for the NF4 codec, on the NF4 kernel (bit-exact).
* ``encode_int8_row_device`` — int8_row encoding on the GPU by ``fb_int8_row_encode`` (conversion time):
  per-row absmax / 127 scale, round half to even, clamp to +-127 (selas/codecs.py:87-97). The block Linears decode int8_row
  inside the tcgen05 GEMM (fb_linear.w_i8); ``decode_int8_row`` is selas's decode formula
  (selas/codecs.py:272-276) for inspecting a weight outside that path.
"""

from __future__ import annotations

import torch

from . import _lib, ops
from ._lib import FluxB200Error

# input dtypes the encoder kernels read directly (others are widened to fp32 first)
_ENC_DTYPES = {torch.float32: _lib.FB_F32, torch.bfloat16: _lib.FB_BF16, torch.float16: _lib.FB_F16}

NF4_CODE = (
    -1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
    -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
    0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
    0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0,
)


@torch.no_grad()
def encode_device(w: torch.Tensor, blocksize: int = 64, code=NF4_CODE) -> tuple[torch.Tensor, torch.Tensor]:
    """(packed uint8 [n/2], absmax fp32 [n/blocksize]) of ``w`` (any shape, numel % blocksize == 0) by
    ``fb_nf4_encode`` (selas/codecs.py:99-119, bit-exact)."""
    if w.device.type != "cuda":
        raise FluxB200Error("encode_device needs a CUDA tensor")
    n = w.numel()
    if n % blocksize or blocksize % 2:
        raise ValueError(f"nf4 needs numel divisible by an even blocksize ({n} % {blocksize})")
    src = w.contiguous() if w.dtype in _ENC_DTYPES else w.float().contiguous()
    packed = torch.empty(n // 2, dtype=torch.uint8, device=w.device)
    absmax = torch.empty(n // blocksize, dtype=torch.float32, device=w.device)
    c = torch.tensor(code, dtype=torch.float32, device=w.device)
    _lib.check(_lib.lib().fb_nf4_encode(src.data_ptr(), _ENC_DTYPES[src.dtype], n, blocksize, c.data_ptr(),
                                        packed.data_ptr(), absmax.data_ptr(), ops._stream()), "fb_nf4_encode")
    ops._count()
    return packed, absmax


def decode(packed: torch.Tensor, absmax: torch.Tensor, meta: dict, shape, dtype: torch.dtype) -> torch.Tensor:
    """``codecs.decode("nf4", ...)`` (selas/codecs.py:278-279) on the NF4 kernel."""
    return ops.nf4_dequant(packed, absmax, int(meta["blocksize"]), meta["code"], tuple(shape), dtype)


@torch.no_grad()
def encode_int8_row_device(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(q int8 [N, K], scale fp32 [N]) of a 2-D weight by ``fb_int8_row_encode`` (selas/codecs.py:87-97,
    bit-exact)."""
    if w.device.type != "cuda":
        raise FluxB200Error("encode_int8_row_device needs a CUDA tensor")
    src = w.reshape(w.shape[0], -1)
    src = src.contiguous() if src.dtype in _ENC_DTYPES else src.float().contiguous()
    rows, cols = src.shape
    q = torch.empty(rows, cols, dtype=torch.int8, device=w.device)
    scale = torch.empty(rows, dtype=torch.float32, device=w.device)
    _lib.check(_lib.lib().fb_int8_row_encode(src.data_ptr(), _ENC_DTYPES[src.dtype], rows, cols, q.data_ptr(),
                                             scale.data_ptr(), ops._stream()), "fb_int8_row_encode")
    ops._count()
    return q, scale


@torch.no_grad()
def decode_int8_row(q: torch.Tensor, scale: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """``codecs.decode("int8_row", ...)`` (selas/codecs.py:272-276)."""
    return q.to(dtype) * scale.to(dtype).view(-1, *([1] * (q.dim() - 1)))
