"""A FLUX transformer held resident in HBM and stepped on the B200 blocks.

* ``FluxArch`` — the architecture fields of ``selas.models.flux.FluxConfig`` (flux.py:44-73).
* ``ResidentUnit`` — a unit's tensors on the device behind selas's ``UnitView`` interface
  (``get`` / ``has`` / ``codec`` / ``parts`` / ``spec``; store.py:242-293), raw bf16 or NF4.
* ``random_model`` — random-init weights N(0, std) generated on the device (the benchmark model).
* ``FluxStepper`` — the caller side of the hot path, mirroring ``FluxRunner.prepare`` / ``step``
  (flux.py:411-465, :527-582, without the step cache) and the Euler update (pipeline.py:489). Its
  prologue (time/guidance/vector embeddings, per-step modulations, txt_in, RoPE tables) runs once per
  batch, outside the step; the Linears there also run on the tcgen05 GEMM.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from . import codec as nf4codec
from . import flux as B
from . import ops
from ._lib import FluxB200Error

BF16, F32 = torch.bfloat16, torch.float32


@dataclass(frozen=True)
class FluxArch:
    hidden: int = 3072
    heads: int = 24
    mlp_hidden: int = 12288
    depth_double: int = 19
    depth_single: int = 38
    in_channels: int = 64
    context_dim: int = 4096
    vec_dim: int = 768
    axes_dim: tuple = (16, 56, 56)
    theta: float = 10000.0
    guidance_embed: bool = True

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads


# ------------------------------------------------------------------------------------------ units


@dataclass
class TensorSpec:
    codec: str
    shape: tuple
    meta: dict = field(default_factory=dict)


@dataclass
class UnitSpec:
    tensors: dict


class ResidentUnit:
    """One unit's tensors on the device with the methods of selas's UnitView that the blocks use."""

    def __init__(self, raw: dict[str, torch.Tensor], nf4: dict[str, dict] | None = None,
                 int8: dict[str, dict] | None = None):
        self._raw = raw
        self._nf4 = nf4 or {}
        self._i8 = int8 or {}  # name -> {"q": int8 [N, K], "scale": fp32 [N]}
        specs = {n: TensorSpec("raw", tuple(t.shape)) for n, t in raw.items()}
        for n, e in self._nf4.items():
            specs[n] = TensorSpec("nf4", tuple(e["shape"]), {"blocksize": e["blocksize"], "code": list(e["code"])})
        for n, e in self._i8.items():
            specs[n] = TensorSpec("int8_row", tuple(e["q"].shape))
        self.spec = UnitSpec(specs)

    def has(self, name: str) -> bool:
        return name in self.spec.tensors

    def codec(self, name: str) -> str:
        return self.spec.tensors[name].codec

    def parts(self, name: str) -> dict[str, torch.Tensor]:
        if name in self._nf4:
            e = self._nf4[name]
            return {"packed": e["packed"], "absmax": e["absmax"]}
        if name in self._i8:
            e = self._i8[name]
            return {"q": e["q"], "scale": e["scale"]}
        return {"data": self._raw[name]}

    def get(self, name: str, dtype: torch.dtype | None = None) -> torch.Tensor:
        if name in self._nf4:
            e = self._nf4[name]
            return ops.nf4_dequant(e["packed"], e["absmax"], e["blocksize"], e["code"], e["shape"], dtype or BF16)
        if name in self._i8:
            e = self._i8[name]
            return nf4codec.decode_int8_row(e["q"], e["scale"], dtype or BF16)
        t = self._raw[name]
        return t if dtype is None or t.dtype == dtype else t.to(dtype)

    def linear(self, x: torch.Tensor, prefix: str, dtype: torch.dtype | None = None) -> torch.Tensor:
        wt = B.weight(self, prefix + ".weight")
        return ops.linear(x.to(BF16), wt, B.bias(self, prefix))

    def nbytes(self) -> int:
        n = sum(t.numel() * t.element_size() for t in self._raw.values())
        for e in self._nf4.values():
            n += e["packed"].numel() + e["absmax"].numel() * 4
        for e in self._i8.values():
            n += e["q"].numel() + e["scale"].numel() * 4
        return n


def _lin_shapes(a: FluxArch, kind: str) -> dict[str, tuple[int, int]]:
    d, m = a.hidden, a.mlp_hidden
    if kind == "double":
        out = {}
        for s in ("img", "txt"):
            out.update({f"{s}_attn.qkv": (3 * d, d), f"{s}_attn.proj": (d, d), f"{s}_mlp.0": (m, d), f"{s}_mlp.2": (d, m)})
        return out
    if kind == "single":
        return {"linear1": (3 * d + m, d), "linear2": (d, d + m)}
    if kind == "double_mod":
        return {"img_mod.lin": (6 * d, d), "txt_mod.lin": (6 * d, d)}
    if kind == "single_mod":
        return {"modulation.lin": (3 * d, d)}
    out = {"img_in": (d, a.in_channels), "txt_in": (d, a.context_dim), "time_in.in_layer": (d, 256),
           "time_in.out_layer": (d, d), "vector_in.in_layer": (d, a.vec_dim), "vector_in.out_layer": (d, d),
           "final_layer.linear": (a.in_channels, d), "final_layer.adaLN_modulation.1": (2 * d, d)}
    if a.guidance_embed:
        out.update({"guidance_in.in_layer": (d, 256), "guidance_in.out_layer": (d, d)})
    return out


def _norm_names(kind: str) -> list[str]:
    if kind == "double":
        return [f"{s}_attn.norm.{q}_norm.scale" for s in ("img", "txt") for q in ("query", "key")]
    if kind == "single":
        return ["norm.query_norm.scale", "norm.key_norm.scale"]
    return []


def random_unit(a: FluxArch, kind: str, gen: torch.Generator, device, std: float = 0.02, quant: str = "none",
                blocksize: int = 64) -> ResidentUnit:
    """Random-init unit: Linear weights and biases N(0, std) in bf16, QK-norm scales N(1, 0.1) fp32.
    With ``quant="nf4"`` (or ``"int8"``) the 2-D block weights are NF4- (int8_row-) encoded on the device,
    as selas's converter does for --quant nf4 / int8 (convert.py:170-185); ``"fp8"`` / ``"fp8_e5m2"`` store
    them raw in fp8, as an fp8 source converted without --quant (convert.py:178-180). Biases stay bf16."""
    raw, nf4, i8 = {}, {}, {}
    for name, (n, k) in _lin_shapes(a, kind).items():
        w = torch.randn(n, k, generator=gen, device=device, dtype=F32).mul_(std)
        if quant == "nf4" and kind in ("double", "single"):
            packed, absmax = nf4codec.encode_device(w, blocksize)
            nf4[name + ".weight"] = {"packed": packed, "absmax": absmax, "blocksize": blocksize,
                                     "code": nf4codec.NF4_CODE, "shape": (n, k)}
        elif quant == "int8" and kind in ("double", "single"):
            q, scale = nf4codec.encode_int8_row_device(w)
            i8[name + ".weight"] = {"q": q, "scale": scale}
        elif quant in ("fp8", "fp8_e5m2") and kind in ("double", "single"):
            raw[name + ".weight"] = w.to(torch.float8_e5m2 if quant == "fp8_e5m2" else torch.float8_e4m3fn)
        else:
            raw[name + ".weight"] = w.to(BF16)
        del w
        raw[name + ".bias"] = torch.randn(n, generator=gen, device=device, dtype=F32).mul_(std).to(BF16)
    for name in _norm_names(kind):
        raw[name] = torch.randn(a.head_dim, generator=gen, device=device, dtype=F32).mul_(0.1).add_(1.0)
    return ResidentUnit(raw, nf4, i8)


def random_model(a: FluxArch, device, seed: int = 0, std: float = 0.02, quant: str = "none",
                 with_mod_units: bool = True) -> dict[str, ResidentUnit]:
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    units = {"globals": random_unit(a, "globals", gen, device, std)}
    for i in range(a.depth_double):
        units[f"double.{i}"] = random_unit(a, "double", gen, device, std, quant)
        if with_mod_units:
            units[f"double.{i}.mod"] = random_unit(a, "double_mod", gen, device, std)
    for i in range(a.depth_single):
        units[f"single.{i}"] = random_unit(a, "single", gen, device, std, quant)
        if with_mod_units:
            units[f"single.{i}.mod"] = random_unit(a, "single_mod", gen, device, std)
    return units


# ------------------------------------------------------------------------------------------ prologue


def timestep_embedding(t: torch.Tensor, dim: int = 256, max_period: float = 10000.0, time_factor: float = 1000.0):
    """Sinusoidal [cos | sin] embedding (flux.py:95-103)."""
    t = time_factor * t.float()
    half = dim // 2
    freqs = torch.exp(-math.log(max_period) * torch.arange(half, dtype=F32, device=t.device) / half)
    args = t[:, None] * freqs[None]
    emb = torch.cat([torch.cos(args), torch.sin(args)], dim=-1)
    if dim % 2:
        emb = torch.cat([emb, torch.zeros_like(emb[:, :1])], dim=-1)
    return emb


def rope_tables(ids: torch.Tensor, axes_dim, theta: float):
    """cos/sin [L, head_dim/2] fp32 from position ids, angles in fp64 (flux.py:106-114)."""
    cols = []
    for i, dim in enumerate(axes_dim):
        omega = theta ** (-(torch.arange(0, dim, 2, dtype=torch.float64, device=ids.device) / dim))
        cols.append(ids[:, i].double()[:, None] * omega[None])
    ang = torch.cat(cols, dim=-1)
    return ang.cos().float().contiguous(), ang.sin().float().contiguous()


@dataclass
class Conditioning:
    sigmas: list
    mods: dict  # unit -> [S, B, k*D] bf16
    final_mod: torch.Tensor  # [S, B, 2D]
    txt: torch.Tensor  # [B, Lt, D] fp32
    cos: torch.Tensor
    sin: torch.Tensor
    l_txt: int


class FluxStepper:
    """Prologue + denoise step of the FLUX transformer on the B200 kernels (no CPU path)."""

    def __init__(self, units: dict[str, ResidentUnit], arch: FluxArch):
        self.u = units
        self.a = arch
        self.g = units["globals"]

    def _mlp_embed(self, prefix: str, x: torch.Tensor) -> torch.Tensor:
        return self.g.linear(F.silu(self.g.linear(x, prefix + ".in_layer")), prefix + ".out_layer")

    @torch.no_grad()
    def svec(self, sigmas, guidance: float, pooled: torch.Tensor) -> torch.Tensor:
        """silu(vec) [S, 1, D] for one image (flux.py:411-425)."""
        dev = pooled.device
        t = torch.tensor(list(sigmas[:-1]), dtype=F32, device=dev)
        vec = self._mlp_embed("time_in", timestep_embedding(t, 256).to(BF16)).float()[:, None, :]
        if self.a.guidance_embed:
            gv = torch.full((1,), float(guidance), dtype=F32, device=dev)
            vec = vec + self._mlp_embed("guidance_in", timestep_embedding(gv, 256).to(BF16)).float()[None]
        vec = vec + self._mlp_embed("vector_in", pooled.to(BF16)).float()[None]
        return F.silu(vec).to(BF16)

    @torch.no_grad()
    def prepare(self, sigmas, guidance: float, pooled, txt, img_ids, txt_ids, mods: dict | None = None) -> Conditioning:
        """Per-batch conditioning (flux.py:448-465)."""
        a = self.a
        svecs = [self.svec(sigmas, guidance, pooled[i:i + 1]) for i in range(pooled.shape[0])]
        if mods is None:
            mods = {}
            for i in range(a.depth_double):
                u = self.u[f"double.{i}.mod"]
                mods[f"double.{i}"] = torch.cat([torch.cat((u.linear(sv, "img_mod.lin"), u.linear(sv, "txt_mod.lin")), -1)
                                                 for sv in svecs], dim=1)
            for i in range(a.depth_single):
                u = self.u[f"single.{i}.mod"]
                mods[f"single.{i}"] = torch.cat([u.linear(sv, "modulation.lin") for sv in svecs], dim=1)
        final_mod = torch.cat([self.g.linear(sv, "final_layer.adaLN_modulation.1") for sv in svecs], dim=1)
        txt_h = self.g.linear(txt.to(BF16), "txt_in").float()
        cos, sin = rope_tables(torch.cat((txt_ids, img_ids), 0).to(pooled.device), a.axes_dim, a.theta)
        return Conditioning(list(sigmas), mods, final_mod, txt_h, cos, sin, txt.shape[1])

    @torch.no_grad()
    def step(self, s: int, latents: torch.Tensor, cond: Conditioning, sp=None, cache=None) -> torch.Tensor:
        """Velocity for step s; latents [B, Li, in_channels] fp32 (flux.py:527-582). With ``sp`` (a
        ``selas_b200.sp.Ulysses``), latents and ``cond`` are this rank's tokens (``sp.localize``) and the
        result is the velocity of those tokens. With ``cache`` (a ``selas_b200.stepcache.StepCache``),
        the first double block is the probe and the cache decides whether the rest of the step runs
        (full), is replaced by the predicted tail residual (skip) or substitutes the predicted residuals
        of its streamed blocks (hybrid); ``self.last_info`` holds (decision, distance)."""
        from .stepcache import FULL, HYBRID, SKIP

        a = self.a
        caching = cache is not None and cache.active
        if caching and sp is not None:
            raise FluxB200Error("step caching with sequence parallelism is not supported")
        sigma = cond.sigmas[s]
        img = ops.linear(latents.to(BF16), B.weight(self.g, "img_in.weight"), B.bias(self.g, "img_in"), out_dtype=F32)
        txt = cond.txt
        names = [f"double.{i}" for i in range(a.depth_double)]
        img_in = img
        img, txt = self._double(names[0], img, txt, cond, s, sp)
        decision, dist = FULL, None
        if caching:
            decision, dist = cache.decide_from(s, sigma, img, img_in)
        del img_in
        self.last_info = (decision, dist)
        if decision == SKIP:
            img = cache.apply_tail(img, sigma)
        else:
            img_probe = img
            hybrid = decision == HYBRID
            for name in names[1:]:
                if hybrid and cache.substitutes(name):
                    img, txt = cache.apply_block(name, sigma, (img, txt))
                    continue
                i0, t0 = img, txt
                img, txt = self._double(name, img, txt, cond, s, sp)
                if decision == FULL and caching and cache.records(name):
                    cache.put_block_from(name, sigma, ((img, i0), (txt, t0)))
            x = torch.cat((txt, img), dim=1)
            del txt, img
            for i in range(a.depth_single):
                name = f"single.{i}"
                if hybrid and cache.substitutes(name):
                    x = cache.apply_block(name, sigma, (x,))[0]
                    continue
                x0 = x
                x = B.single_block(self.u[name], x, cond.mods[name][s], cond.cos, cond.sin, a, BF16, False, sp=sp)
                if decision == FULL and caching and cache.records(name):
                    cache.put_block_from(name, sigma, ((x, x0),))
            img = x[:, cond.l_txt:]
            del x
            if decision == FULL and caching:
                cache.put_tail_from(sigma, img, img_probe)
        return B.final_layer(self.g, img, cond.final_mod[s], BF16)

    def _double(self, name, img, txt, cond, s, sp):
        return B.double_block(self.u[name], img, txt, cond.mods[name][s], cond.cos, cond.sin, self.a, BF16, False, sp=sp)

    @torch.no_grad()
    def denoise(self, x: torch.Tensor, cond: Conditioning, sp=None, cache=None) -> torch.Tensor:
        """Euler flow-matching loop (pipeline.py:483-489); with ``sp``, over this rank's tokens; with
        ``cache``, steps approximated by the step cache."""
        sig = cond.sigmas
        for s in range(len(sig) - 1):
            x = x + (sig[s + 1] - sig[s]) * self.step(s, x, cond, sp, cache)
        return x
