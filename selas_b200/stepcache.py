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

from dataclasses import dataclass, field

import torch

from ._lib import FluxB200Error

FULL, SKIP, HYBRID = "full", "skip", "hybrid"
POLICIES = ("none", "fbcache", "tiered")


@dataclass
class StepCacheConfig:
    """selas/stepcache.py:49-72."""

    policy: str = "none"
    threshold: float = 0.08
    predict: str = "linear"  # linear | reuse
    warmup: int = 1
    tail_full: int = 1
    max_consecutive: int = 3

    def __post_init__(self):
        if self.policy not in POLICIES:
            raise ValueError(f"cache policy must be one of {POLICIES}")
        if self.predict not in ("reuse", "linear"):
            raise ValueError("cache prediction must be 'reuse' or 'linear'")

    @property
    def active(self) -> bool:
        return self.policy != "none"

    def describe(self) -> str:
        if not self.active:
            return "off (exact)"
        return (f"{self.policy} threshold={self.threshold} predict={self.predict} warmup={self.warmup} "
                f"tail_full={self.tail_full} max_consecutive={self.max_consecutive} (APPROXIMATE)")


@dataclass
class _Hist:
    """Newest-last history of (sigma, residual tensors) (selas/stepcache.py:75-94)."""

    items: list = field(default_factory=list)

    def push(self, sigma: float, tensors: tuple, keep: int) -> None:
        self.items.append((sigma, tensors))
        del self.items[:-keep]

    def plan(self, sigma: float, mode: str):
        """(r1 tensors, r0 tensors or None, a): the prediction is r1 + a (r1 - r0), or r1."""
        if not self.items:
            raise RuntimeError("no cached residual available")
        s1, r1 = self.items[-1]
        if mode == "linear" and len(self.items) >= 2:
            s0, r0 = self.items[-2]
            if s1 != s0:
                return r1, r0, (sigma - s1) / (s1 - s0)
        return r1, None, 0.0


class StepCache:
    """Per-generation cache state (selas/stepcache.py:97-219). ``streamed`` = names of non-resident units."""

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
        self.keep = 2 if cfg.predict == "linear" else 1
        self.host = host_residuals
        self.ref_probe: torch.Tensor | None = None
        self.tail = _Hist()
        self.blocks: dict[str, _Hist] = {}
        self.consecutive = 0
        self.log: list[tuple[int, str, float | None]] = []

    @property
    def active(self) -> bool:
        return self.cfg.active

    # ------------------------------------------------------------------ decisions
    def _decide(self, step: int, sums, candidate: torch.Tensor, n: int) -> tuple[str, float | None]:
        cfg = self.cfg
        d = None
        decision = FULL
        forced = (step < cfg.warmup or step >= self.num_steps - cfg.tail_full or self.ref_probe is None
                  or self.consecutive >= cfg.max_consecutive)
        if sums is not None:
            d = (sums[0] / n) / max(sums[1] / n, 1e-12)
        if not forced and d is not None and d < cfg.threshold:
            decision = SKIP if cfg.policy == "fbcache" else HYBRID
        if decision == FULL:
            self.ref_probe = candidate
            self.consecutive = 0
        else:
            self.consecutive += 1
        self.log.append((step, decision, d))
        return decision, d

    def decide(self, step: int, sigma: float, probe_residual: torch.Tensor) -> tuple[str, float | None]:
        """selas/stepcache.py:114-138 on a probe residual."""
        r = probe_residual.detach().float().contiguous()
        sums = None if self.ref_probe is None else self.k.probe_distance(r, None, self.ref_probe, None)
        return self._decide(step, sums, r, r.numel())

    def decide_from(self, step: int, sigma: float, x: torch.Tensor, x_in: torch.Tensor) -> tuple[str, float | None]:
        """``decide(step, sigma, x - x_in)`` with the residual formed and reduced in the same pass."""
        x, x_in = x.contiguous(), x_in.contiguous()
        r = torch.empty(x.shape, dtype=torch.float32, device=x.device)
        sums = self.k.probe_distance(x, x_in, self.ref_probe, r)
        return self._decide(step, sums, r, r.numel())

    # ------------------------------------------------------------------ fbcache
    def put_tail(self, sigma: float, residual: torch.Tensor) -> None:
        self.tail.push(sigma, (residual.detach().float().contiguous(),), self.keep)

    def put_tail_from(self, sigma: float, x: torch.Tensor, x0: torch.Tensor) -> None:
        """``put_tail(sigma, x - x0)`` with the subtraction on the device kernel."""
        self.tail.push(sigma, (self.k.residual_diff(x.contiguous(), x0.contiguous(), torch.float32),), self.keep)

    def tail_residual(self, sigma: float) -> torch.Tensor:
        r1, r0, a = self.tail.plan(sigma, self.cfg.predict)
        return self.k.residual_predict(None, r1[0], None if r0 is None else r0[0], a)

    def apply_tail(self, x: torch.Tensor, sigma: float) -> torch.Tensor:
        """x + tail_residual(sigma) in one pass (selas/models/flux.py:553)."""
        r1, r0, a = self.tail.plan(sigma, self.cfg.predict)
        return self.k.residual_predict(x.contiguous(), r1[0], None if r0 is None else r0[0], a)

    # ------------------------------------------------------------------ tiered
    def records(self, name: str) -> bool:
        return self.cfg.policy == "tiered" and name in self.streamed

    def substitutes(self, name: str) -> bool:
        if self.cfg.policy != "tiered" or name not in self.streamed:
            return False
        if name not in self.blocks:
            raise RuntimeError(f"tiered cache has no residual for streamed unit {name}")
        return True

    def put_block(self, name: str, sigma: float, residuals: tuple) -> None:
        rs = tuple(r.detach().to(self.store_dtype).contiguous() for r in residuals)
        self.blocks.setdefault(name, _Hist()).push(sigma, rs, self.keep)

    def put_block_from(self, name: str, sigma: float, pairs: tuple) -> None:
        """``put_block(name, sigma, tuple(x - x0 for x, x0 in pairs))`` with the difference and the cast
        to store_dtype in one pass each."""
        rs = tuple(self.k.residual_diff(x.contiguous(), x0.contiguous(), self.store_dtype) for x, x0 in pairs)
        self.blocks.setdefault(name, _Hist()).push(sigma, rs, self.keep)

    def block_residual(self, name: str, sigma: float) -> tuple:
        r1, r0, a = self.blocks[name].plan(sigma, self.cfg.predict)
        return tuple(self.k.residual_predict(None, t1, None if r0 is None else t0, a)
                     for t1, t0 in zip(r1, r0 if r0 is not None else r1))

    def apply_block(self, name: str, sigma: float, xs: tuple) -> tuple:
        """tuple(x + r for x, r in zip(xs, block_residual(name, sigma))), one pass per tensor."""
        r1, r0, a = self.blocks[name].plan(sigma, self.cfg.predict)
        return tuple(self.k.residual_predict(x.contiguous(), t1, None if r0 is None else t0, a)
                     for x, t1, t0 in zip(xs, r1, r0 if r0 is not None else r1))

    def close(self) -> None:
        self.blocks.clear()
        self.tail = _Hist()

    # ------------------------------------------------------------------ reporting
    def summary(self) -> str:
        if not self.active:
            return "step cache off"
        n = len(self.log)
        approx = sum(1 for _, dec, _ in self.log if dec != FULL)
        dists = " ".join(f"{dec[0]}{'' if d is None else f'{d:.3f}'}" for _, dec, d in self.log)
        return f"step cache: {approx}/{n} steps approximated ({self.cfg.policy}); per-step: {dists}"
