"""NF4 codec helpers on the device.

* ``NF4_CODE`` — the 16-level NF4 code book (the QLoRA / bitsandbytes table, as in selas/codecs.py:58-63).
* ``encode_device`` — NF4 encoding of a weight already on the GPU, for building quantised models in
  HBM (conversion time, not the hot path): blockwise absmax, nearest code with ties to the lower code,
  first element in the high nibble (selas/codecs.py:99-119).
* ``decode`` — selas's ``codecs.decode`` entry for the NF4 codec, on the NF4 kernel (bit-exact).
* ``encode_int8_row_device`` — int8_row encoding on the GPU (conversion time): per-row absmax / 127
  scale, round half to even, clamp to +-127 (selas/codecs.py:87-97). The block Linears decode int8_row
  inside the tcgen05 GEMM (fb_linear.w_i8); ``decode_int8_row`` is selas's decode formula
  (selas/codecs.py:272-276) for inspecting a weight outside that path.
"""

from __future__ import annotations

import torch

from . import ops

NF4_CODE = (
    -1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
    -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
    0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
    0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0,
)


@torch.no_grad()
def encode_device(w: torch.Tensor, blocksize: int = 64, code=NF4_CODE) -> tuple[torch.Tensor, torch.Tensor]:
    """(packed uint8 [n/2], absmax fp32 [n/blocksize]) of ``w`` (any shape, numel % blocksize == 0)."""
    flat = w.float().reshape(-1)
    if flat.numel() % blocksize or blocksize % 2:
        raise ValueError(f"nf4 needs numel divisible by an even blocksize ({flat.numel()} % {blocksize})")
    blocks = flat.view(-1, blocksize)
    absmax = blocks.abs().amax(dim=1)
    safe = torch.where(absmax > 0, absmax, torch.ones_like(absmax))
    normed = (blocks / safe[:, None]).reshape(-1)
    c = torch.tensor(code, dtype=torch.float32, device=w.device)
    mids = (c[1:] + c[:-1]) / 2
    idx = torch.bucketize(normed, mids).to(torch.uint8)
    packed = (idx[0::2] << 4) | idx[1::2]
    return packed.contiguous(), absmax.contiguous()


def decode(packed: torch.Tensor, absmax: torch.Tensor, meta: dict, shape, dtype: torch.dtype) -> torch.Tensor:
    """``codecs.decode("nf4", ...)`` (selas/codecs.py:278-279) on the NF4 kernel."""
    return ops.nf4_dequant(packed, absmax, int(meta["blocksize"]), meta["code"], tuple(shape), dtype)


@torch.no_grad()
def encode_int8_row_device(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(q int8 [N, K], scale fp32 [N]) of a 2-D weight (selas/codecs.py:87-97)."""
    w = w.float().reshape(w.shape[0], -1)
    absmax = w.abs().amax(dim=1)
    scale = torch.where(absmax > 0, absmax / 127.0, torch.ones_like(absmax))
    q = torch.round(w / scale[:, None]).clamp_(-127, 127).to(torch.int8)
    return q.contiguous(), scale.contiguous()


@torch.no_grad()
def decode_int8_row(q: torch.Tensor, scale: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """``codecs.decode("int8_row", ...)`` (selas/codecs.py:272-276)."""
    return q.to(dtype) * scale.to(dtype).view(-1, *([1] * (q.dim() - 1)))
