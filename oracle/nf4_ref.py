"""NF4 codec restated in numpy — TEST INFRASTRUCTURE ONLY (the CPU checker for the CUDA NF4 paths).

Follows ``selas/codecs.py`` of tcox-coding/selas:

* code book ``NF4_CODE`` — ``selas/codecs.py:58-63``;
* encoder (nearest code, ties to the lower code, first element in the high nibble) — ``selas/codecs.py:99-119``;
* decoder ``value = fp32(code[nibble]) * fp32(absmax[block])``, one IEEE multiply, then a
  round-to-nearest-even cast to the output dtype — ``selas/codecs.py:178-199`` (torch path) and
  ``:211-221`` (Triton path); both agree bit for bit (``selas/codecs.py:242-253``).

Pinned by ``tests/test_oracle_golden.py`` against vectors written by the reference itself.
"""

from __future__ import annotations

import numpy as np

NF4_CODE = np.array(
    [-1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
     -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
     0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
     0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0],
    dtype=np.float32,
)


def encode(values: np.ndarray, blocksize: int = 64, code: np.ndarray = NF4_CODE) -> tuple[np.ndarray, np.ndarray]:
    """(packed uint8 [n/2], absmax fp32 [n/blocksize]) — selas/codecs.py:99-119."""
    flat = np.ascontiguousarray(values, dtype=np.float32).reshape(-1)
    n = flat.size
    if n % blocksize or blocksize % 2:
        raise ValueError(f"nf4 needs numel divisible by an even blocksize ({n} % {blocksize})")
    blocks = flat.reshape(-1, blocksize)
    absmax = np.abs(blocks).max(axis=1).astype(np.float32)
    safe = np.where(absmax > 0, absmax, np.float32(1.0)).astype(np.float32)
    normed = (blocks / safe[:, None]).astype(np.float32).reshape(-1)
    code = np.asarray(code, dtype=np.float32)
    mids = ((code[1:] + code[:-1]) / np.float32(2)).astype(np.float32)
    # index i such that mids[i-1] < x <= mids[i]  (ties go to the lower code)
    idx = np.searchsorted(mids, normed, side="left").astype(np.uint8)
    packed = ((idx[0::2] << 4) | idx[1::2]).astype(np.uint8)
    return packed, absmax


def decode_f32(packed: np.ndarray, absmax: np.ndarray, blocksize: int, code: np.ndarray = NF4_CODE) -> np.ndarray:
    """fp32 products code[nibble] * absmax[block], element order hi0, lo0, hi1, lo1, ..."""
    packed = np.asarray(packed, dtype=np.uint8).reshape(-1)
    code = np.asarray(code, dtype=np.float32)
    nib = np.empty(packed.size * 2, dtype=np.uint8)
    nib[0::2] = packed >> 4
    nib[1::2] = packed & 15
    scale = np.repeat(np.asarray(absmax, dtype=np.float32).reshape(-1), blocksize)
    if scale.size != nib.size:
        raise ValueError(f"absmax has {absmax.size} blocks for {nib.size} values at blocksize {blocksize}")
    return (code[nib] * scale).astype(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16, returned as uint16 bit patterns (NaN kept quiet)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint32)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    rounded = np.where(nan, ((u >> 16) | 0x40).astype(np.uint32), rounded)
    return rounded.astype(np.uint16)


def decode(packed: np.ndarray, absmax: np.ndarray, blocksize: int, out_dtype: str, code: np.ndarray = NF4_CODE) -> np.ndarray:
    """Decoded values in ``out_dtype`` ('float32' | 'float16' | 'bfloat16'); bf16 comes back as uint16 bits."""
    v = decode_f32(packed, absmax, blocksize, code)
    if out_dtype == "float32":
        return v
    if out_dtype == "float16":
        return v.astype(np.float16)
    if out_dtype == "bfloat16":
        return f32_to_bf16_bits(v)
    raise ValueError(f"unsupported output dtype {out_dtype!r}")


def decode_torch(packed, absmax, blocksize: int, shape, out_dtype, code=NF4_CODE):
    """The same decode in torch, on whatever device ``packed`` lives (selas/codecs.py:178-199, the torch
    path): value = fp32(code[nibble]) * fp32(absmax[block]), one IEEE multiply, then the cast to
    ``out_dtype`` (round to nearest even). Used by the GPU tests to give the fp32 checker the decoded
    weights of a whole NF4 model without a trip through numpy; pinned to ``decode`` on the CPU."""
    import torch

    p = packed.reshape(-1)
    table = torch.as_tensor(np.asarray(code, dtype=np.float32), device=p.device)
    nib = torch.stack(((p >> 4).long(), (p & 15).long()), dim=1).reshape(-1)
    vals = table[nib].reshape(-1, blocksize) * absmax.reshape(-1, 1).float()
    return vals.reshape(shape).to(out_dtype)
