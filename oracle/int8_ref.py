"""int8_row codec restated in numpy — TEST INFRASTRUCTURE ONLY (the CPU checker for the CUDA int8 path).

Follows ``selas/codecs.py`` of tcox-coding/selas:

* encoder — ``encode_int8_row`` (``selas/codecs.py:87-97``): per row of the [N, K] matrix, absmax over
  the row, scale = absmax / 127 (1 for an all-zero row), q = round(w / scale) (half to even) clamped to
  [-127, 127], all in fp32;
* decoder — ``decode`` for ``int8_row`` (``selas/codecs.py:272-276``): ``q.to(dtype) * scale.to(dtype)``;
  for bf16 that is bf16(fp32(q) * fp32(bf16(scale))), the product exact in fp32, one RNE cast.

Pinned by ``tests/test_oracle_golden.py`` against vectors written by the reference itself.
"""

from __future__ import annotations

import numpy as np


def encode(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """(q int8 [N, K], scale fp32 [N]) — selas/codecs.py:87-97."""
    w = np.ascontiguousarray(w, dtype=np.float32).reshape(w.shape[0], -1)
    absmax = np.abs(w).max(axis=1).astype(np.float32)
    scale = np.where(absmax > 0, (absmax / np.float32(127.0)).astype(np.float32), np.float32(1.0)).astype(np.float32)
    q = np.clip(np.rint((w / scale[:, None]).astype(np.float32)), -127, 127).astype(np.int8)
    return q, scale


def _bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16, as uint16 bit patterns (finite inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF).astype(np.uint16)


def _bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def decode_bf16(q: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """bf16 bit patterns [N, K] of the decoded weight — selas/codecs.py:272-276 with dtype bf16."""
    s = _bf16_to_f32(_bf16_bits(scale.astype(np.float32)))
    prod = (q.astype(np.float32) * s.reshape(-1, *([1] * (q.ndim - 1)))).astype(np.float32)
    return _bf16_bits(prod)
