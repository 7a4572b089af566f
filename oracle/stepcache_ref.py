"""Step-cache arithmetic restated in numpy — TEST INFRASTRUCTURE ONLY (the CPU checker for the CUDA
step-cache kernels, and the stand-in kernels of the CPU tests of ``selas_b200.stepcache``).

Follows ``selas/stepcache.py`` and ``selas/models/flux.py`` of tcox-coding/selas:

* the probe residual ``img - img_in`` (``selas/models/flux.py:548``) and the distance of
  ``StepCache.decide`` (``selas/stepcache.py:127-129``): ``mean|r - ref| / max(mean|ref|, 1e-12)``;
  elementwise values in fp32 (each op rounded once), sums in fp64;
* the prediction of ``_Hist.predict`` (``selas/stepcache.py:84-94``): ``r1 + a * (r1 - r0)`` with
  ``a = (sigma - s1) / (s1 - s0)`` rounded to fp32, each fp32 op rounded once, then the add of the
  predicted residual to the hidden state (``selas/models/flux.py:553, 559-561, 571``);
* the residual captures ``(x - x0).to(store_dtype)`` (``selas/stepcache.py:157``, ``flux.py:566, 576``).

The functions take and return CPU torch tensors with the signatures of ``selas_b200.ops.probe_distance``,
``residual_predict`` and ``residual_diff``, so a test can pass this module as the kernels of a StepCache.
Pinned by ``tests/test_oracle_golden.py`` against ``tests/golden/stepcache.npz``, written by the reference.
"""

from __future__ import annotations

import numpy as np
import torch


def _f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.float32).contiguous().numpy().reshape(-1)


def _bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (finite inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF).astype(np.uint16)


def probe_distance(x, x_in, ref, resid):
    """r = x - x_in (or x) into ``resid``; with ``ref``: (sum|r - ref|, sum|ref|) in fp64."""
    r = _f32(x)
    if x_in is not None:
        r = (r - _f32(x_in)).astype(np.float32)
    if resid is not None:
        resid.copy_(torch.from_numpy(r.reshape(resid.shape)))
    if ref is None:
        return None
    q = _f32(ref)
    return float(np.abs((r - q).astype(np.float32)).astype(np.float64).sum()), float(np.abs(q).astype(np.float64).sum())


def distance(sums: tuple[float, float], n: int) -> float:
    """The reference's distance from the two sums (selas/stepcache.py:129)."""
    return (sums[0] / n) / max(sums[1] / n, 1e-12)


def residual_predict(x, r1, r0, a, out=None):
    """x + (r1 + a (r1 - r0)) in fp32 (x None: the prediction; r0 None: r1)."""
    p = _f32(r1)
    if r0 is not None:
        af = np.float32(a)
        p = (p + (af * (p - _f32(r0)).astype(np.float32)).astype(np.float32)).astype(np.float32)
    if x is not None:
        p = (_f32(x) + p).astype(np.float32)
    res = torch.from_numpy(p.reshape(r1.shape).copy())
    if out is not None:
        out.copy_(res)
        return out
    return res


def residual_diff(x, x0, dtype=torch.float32):
    """(x - x0) as fp32 or bf16 (round to nearest even)."""
    d = (_f32(x) - _f32(x0)).astype(np.float32)
    if dtype == torch.bfloat16:
        return torch.from_numpy(_bf16_bits(d).view(np.int16).reshape(x.shape).copy()).view(torch.bfloat16)
    return torch.from_numpy(d.reshape(x.shape).copy())
