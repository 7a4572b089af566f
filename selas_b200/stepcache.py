"""Activation caching across denoising steps, with its arithmetic on the device (selas/stepcache.py).

The same policies, guards and decisions as selas's ``StepCache`` (``fbcache``: skip every block after
the probe and add the predicted tail residual; ``tiered``: recompute resident blocks and substitute
the predicted residuals of ``streamed`` ones; ``linear`` / ``reuse`` prediction; ``warmup``,
``tail_full``, ``max_consecutive``). What runs on the GPU are the three streams over the hidden state
(``csrc/stepcache.cu``):

* the probe residual and its distance to the reference residual in ONE pass (``decide_from``: the
  residual ``x - x_in`` is formed, stored for a possible full step, and reduced against the reference
  without a separate subtraction kernel); ``decide`` takes a residual as selas's does;
* the prediction and its add to the hidden state in one pass (``apply_tail`` / ``apply_block``:
  ``x + r1 + a (r1 - r0)`` without materialising the prediction); ``tail_residual`` /
  ``block_residual`` return the prediction as selas's do;
* the residual captures ``(x - x0).to(store_dtype)`` of ``put_block``.

The distance needs one device-to-host read of two fp64 sums per step, where selas reads one fp32 mean.
On a B200 every block is resident, so ``streamed`` is normally empty; residuals always stay in HBM
(``host_residuals`` is accepted for API compatibility: selas's pinned-RAM tier exists for GPUs whose
memory cannot hold them).

``kernels`` (default: the CUDA ops of ``selas_b200.ops``) supplies ``probe_distance``,
``residual_predict`` and ``residual_diff``; the CPU tests pass the oracle's restatements.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import NamedTuple

import torch

from ._lib import FluxB200Error

FULL, SKIP, HYBRID = "full", "skip", "hybrid"
POLICIES = ("none", "fbcache", "tiered")
_PREDICTORS = ("linear", "reuse")


@dataclass
class StepCacheConfig:
    """The knobs of selas's ``StepCacheConfig`` (selas/stepcache.py:49-72), same names and defaults:
    ``policy`` (none | fbcache | tiered), ``threshold`` on the probe distance, ``predict`` (linear
    extrapolation over the last two residuals, or reuse of the last), ``warmup`` / ``tail_full`` steps
    always computed at the start / end, and at most ``max_consecutive`` approximated steps in a row."""

    policy: str = "none"
    threshold: float = 0.08
    predict: str = "linear"
    warmup: int = 1
    tail_full: int = 1
    max_consecutive: int = 3

    def __post_init__(self):
        problems = []
        if self.policy not in POLICIES:
            problems.append(f"policy {self.policy!r} is not one of {POLICIES}")
        if self.predict not in _PREDICTORS:
            problems.append(f"predict {self.predict!r} is not one of {_PREDICTORS}")
        if problems:
            raise ValueError("StepCacheConfig: " + "; ".join(problems))

    @property
    def active(self) -> bool:
        return self.policy != "none"

    def describe(self) -> str:
        if not self.active:
            return "step cache: off, every step exact"
        return (f"step cache: {self.policy}, approximate when the probe moves < {self.threshold:g} "
                f"({self.predict} prediction); exact for the first {self.warmup} and last {self.tail_full} "
                f"step(s), at most {self.max_consecutive} approximated in a row")


class StepLog(NamedTuple):
    step: int
    decision: str
    distance: float | None


class _Residuals:
    """The newest ``depth`` (sigma, residual tensors) of one stream. A prediction for sigma is returned
    as coefficients, ``r1 + a (r1 - r0)`` (linear, two distinct sigmas) or ``r1`` (otherwise), so the
    kernel that applies it can fuse the arithmetic with the add to the hidden state."""

    def __init__(self, depth: int):
        self.depth = depth
        self.sigmas: list[float] = []
        self.tensors: list[tuple] = []

    def remember(self, sigma: float, tensors: tuple) -> None:
        self.sigmas = (self.sigmas + [sigma])[-self.depth:]
        self.tensors = (self.tensors + [tensors])[-self.depth:]

    def empty(self) -> bool:
        return not self.tensors

    def coefficients(self, sigma: float, mode: str):
        if self.empty():
            raise RuntimeError("step cache: nothing has been recorded to predict from")
        newest = self.tensors[-1]
        if mode == "linear" and len(self.tensors) == 2 and self.sigmas[0] != self.sigmas[1]:
            s_old, s_new = self.sigmas
            return newest, self.tensors[0], (sigma - s_new) / (s_new - s_old)
        return newest, None, 0.0


class StepCache:
    """Per-generation cache state with selas's ``StepCache`` interface (selas/stepcache.py:97-224):
    the same decisions on the same inputs, the residual arithmetic done by ``kernels``. ``streamed``
    names the non-resident units whose block residuals the tiered policy substitutes."""

    def __init__(self, cfg: StepCacheConfig, num_steps: int, streamed: set[str] | frozenset = frozenset(),
                 store_dtype: torch.dtype = torch.bfloat16, host_residuals: bool = False, kernels=None):
        if store_dtype not in (torch.float32, torch.bfloat16):
            raise FluxB200Error("StepCache: store_dtype must be float32 or bfloat16")
        if kernels is None:
            from . import ops as kernels
        self.k = kernels
        self.cfg = cfg
        self.num_steps = num_steps
        self.streamed = frozenset(streamed)
        self.store_dtype = store_dtype
        self.host = host_residuals  # accepted for API compatibility; residuals stay in HBM
        self._depth = 2 if cfg.predict == "linear" else 1
        self.ref_probe: torch.Tensor | None = None
        self.tail = _Residuals(self._depth)
        self.blocks: dict[str, _Residuals] = {}
        self.consecutive = 0
        self.log: list[StepLog] = []
        self.reasons: list[str] = []  # why each step was computed in full (or "approximated")

    @property
    def active(self) -> bool:
        return self.cfg.active

    # ------------------------------------------------------------------ decisions
    def _full_step_reason(self, step: int) -> str | None:
        """Why this step must run in full whatever the probe says, or None if it may be approximated."""
        cfg = self.cfg
        if step < cfg.warmup:
            return "warm-up"
        if step >= self.num_steps - cfg.tail_full:
            return "final steps"
        if self.ref_probe is None:
            return "no reference probe yet"
        if self.consecutive >= cfg.max_consecutive:
            return "approximation streak limit"
        return None

    def _settle(self, step: int, sums, candidate: torch.Tensor, n: int) -> tuple[str, float | None]:
        """Turn the device sums (sum |r - ref|, sum |ref|) into the distance and the step's decision; a
        full step makes ``candidate`` the new reference probe."""
        distance = None if sums is None else (sums[0] / n) / max(sums[1] / n, 1e-12)
        reason = self._full_step_reason(step)
        if reason is None and distance >= self.cfg.threshold:
            reason = "probe moved"
        if reason is None:
            decision = SKIP if self.cfg.policy == "fbcache" else HYBRID
            self.consecutive += 1
            self.reasons.append("approximated")
        else:
            decision = FULL
            self.ref_probe = candidate
            self.consecutive = 0
            self.reasons.append(reason)
        self.log.append(StepLog(step, decision, distance))
        return decision, distance

    def decide(self, step: int, sigma: float, probe_residual: torch.Tensor) -> tuple[str, float | None]:
        """The decision for ``step`` from the probe block's residual (selas/stepcache.py:114-138)."""
        r = probe_residual.detach().float().contiguous()
        sums = None if self.ref_probe is None else self.k.probe_distance(r, None, self.ref_probe, None)
        return self._settle(step, sums, r, r.numel())

    def decide_from(self, step: int, sigma: float, x: torch.Tensor, x_in: torch.Tensor) -> tuple[str, float | None]:
        """``decide(step, sigma, x - x_in)`` with the residual formed and reduced in the same pass."""
        x, x_in = x.contiguous(), x_in.contiguous()
        r = torch.empty(x.shape, dtype=torch.float32, device=x.device)
        sums = self.k.probe_distance(x, x_in, self.ref_probe, r)
        return self._settle(step, sums, r, r.numel())

    # ------------------------------------------------------------------ fbcache: the tail after the probe
    def put_tail(self, sigma: float, residual: torch.Tensor) -> None:
        self.tail.remember(sigma, (residual.detach().float().contiguous(),))

    def put_tail_from(self, sigma: float, x: torch.Tensor, x0: torch.Tensor) -> None:
        """``put_tail(sigma, x - x0)`` with the subtraction on the device kernel."""
        self.tail.remember(sigma, (self.k.residual_diff(x.contiguous(), x0.contiguous(), torch.float32),))

    def tail_residual(self, sigma: float) -> torch.Tensor:
        r1, r0, a = self.tail.coefficients(sigma, self.cfg.predict)
        return self.k.residual_predict(None, r1[0], None if r0 is None else r0[0], a)

    def apply_tail(self, x: torch.Tensor, sigma: float) -> torch.Tensor:
        """x + tail_residual(sigma) in one pass (selas/models/flux.py:553)."""
        r1, r0, a = self.tail.coefficients(sigma, self.cfg.predict)
        return self.k.residual_predict(x.contiguous(), r1[0], None if r0 is None else r0[0], a)

    # ------------------------------------------------------------------ tiered: streamed blocks
    def _tiered_stream(self, name: str) -> bool:
        return self.cfg.policy == "tiered" and name in self.streamed

    def records(self, name: str) -> bool:
        """Whether a full step stores this unit's block residuals."""
        return self._tiered_stream(name)

    def substitutes(self, name: str) -> bool:
        """Whether an approximated step replaces this unit by its predicted residuals."""
        if not self._tiered_stream(name):
            return False
        if name not in self.blocks:
            raise RuntimeError(f"step cache: unit {name} is streamed but no full step has recorded it")
        return True

    def _block_history(self, name: str) -> _Residuals:
        if name not in self.blocks:
            self.blocks[name] = _Residuals(self._depth)
        return self.blocks[name]

    def put_block(self, name: str, sigma: float, residuals: tuple) -> None:
        rs = tuple(r.detach().to(self.store_dtype).contiguous() for r in residuals)
        self._block_history(name).remember(sigma, rs)

    def put_block_from(self, name: str, sigma: float, pairs: tuple) -> None:
        """``put_block(name, sigma, tuple(x - x0 for x, x0 in pairs))`` with the difference and the cast
        to store_dtype in one pass each."""
        rs = tuple(self.k.residual_diff(x.contiguous(), x0.contiguous(), self.store_dtype) for x, x0 in pairs)
        self._block_history(name).remember(sigma, rs)

    def _per_tensor(self, name: str, sigma: float, xs):
        r1, r0, a = self.blocks[name].coefficients(sigma, self.cfg.predict)
        olds = r0 if r0 is not None else (None,) * len(r1)
        return tuple(self.k.residual_predict(x, t1, t0, a) for x, t1, t0 in zip(xs, r1, olds))

    def block_residual(self, name: str, sigma: float) -> tuple:
        n = len(self.blocks[name].tensors[-1])
        return self._per_tensor(name, sigma, (None,) * n)

    def apply_block(self, name: str, sigma: float, xs: tuple) -> tuple:
        """tuple(x + r for x, r in zip(xs, block_residual(name, sigma))), one pass per tensor."""
        return self._per_tensor(name, sigma, tuple(x.contiguous() for x in xs))

    def close(self) -> None:
        self.blocks.clear()
        self.tail = _Residuals(self._depth)

    # ------------------------------------------------------------------ reporting
    def summary(self) -> str:
        if not self.active:
            return "step cache off"
        approx = [e for e in self.log if e.decision != FULL]
        marks = " ".join(e.decision[0].upper() + ("" if e.distance is None else f"({e.distance:.3f})")
                         for e in self.log)
        return f"step cache {self.cfg.policy}: {len(approx)} of {len(self.log)} steps approximated: {marks}"
