"""Deterministic synthetic FLUX weights and inputs — TEST INFRASTRUCTURE ONLY.

Random-init weights in the reference's own key layout (BFL names inside a unit, as
``selas/convert.py:144-167`` lays them out): every Linear weight and bias is N(0, std), the QK-RMSNorm
scales are N(1, 0.1) (the choice of ``tests/conftest.py:50-52`` in the reference, so q/k are not
squashed). Each tensor draws from its own numpy stream keyed by (seed, unit, name), so a tensor's
values do not depend on which other tensors were generated. Values are rounded to bfloat16 and kept
as fp32 when ``bf16_exact`` is set, so an fp32 run and a bf16 run see the same weights.
"""

from __future__ import annotations

import zlib
from dataclasses import dataclass

import numpy as np
import torch


@dataclass(frozen=True)
class Arch:
    """FLUX architecture sizes (the fields of ``FluxConfig``, ``selas/models/flux.py:44-56``)."""

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


def _stream(seed: int, key: str) -> np.random.Generator:
    return np.random.default_rng(np.random.SeedSequence([int(seed), zlib.crc32(key.encode())]))


def normal(seed: int, key: str, shape, std: float = 1.0, mean: float = 0.0) -> torch.Tensor:
    a = _stream(seed, key).standard_normal(size=tuple(shape), dtype=np.float32)
    if std != 1.0:
        a *= np.float32(std)
    if mean != 0.0:
        a += np.float32(mean)
    return torch.from_numpy(a)


def _bf16_exact(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).float()


def _lin(out: dict, seed: int, unit: str, name: str, n_in: int, n_out: int, std: float, exact: bool) -> None:
    w = normal(seed, f"{unit}/{name}.weight", (n_out, n_in), std)
    b = normal(seed, f"{unit}/{name}.bias", (n_out,), std)
    out[name + ".weight"] = _bf16_exact(w) if exact else w
    out[name + ".bias"] = _bf16_exact(b) if exact else b


def _norms(out: dict, seed: int, unit: str, prefix: str, hd: int) -> None:
    for q in ("query", "key"):
        name = f"{prefix}.{q}_norm.scale"
        out[name] = normal(seed, f"{unit}/{name}", (hd,), 0.1, 1.0)


def double_unit(a: Arch, seed: int, index: int, std: float = 0.02, bf16_exact: bool = True) -> dict:
    unit, d, m, out = f"double.{index}", a.hidden, a.mlp_hidden, {}
    for s in ("img", "txt"):
        _lin(out, seed, unit, f"{s}_attn.qkv", d, 3 * d, std, bf16_exact)
        _lin(out, seed, unit, f"{s}_attn.proj", d, d, std, bf16_exact)
        _lin(out, seed, unit, f"{s}_mlp.0", d, m, std, bf16_exact)
        _lin(out, seed, unit, f"{s}_mlp.2", m, d, std, bf16_exact)
        _norms(out, seed, unit, f"{s}_attn.norm", a.head_dim)
    return out


def single_unit(a: Arch, seed: int, index: int, std: float = 0.02, bf16_exact: bool = True) -> dict:
    unit, d, m, out = f"single.{index}", a.hidden, a.mlp_hidden, {}
    _lin(out, seed, unit, "linear1", d, 3 * d + m, std, bf16_exact)
    _lin(out, seed, unit, "linear2", d + m, d, std, bf16_exact)
    _norms(out, seed, unit, "norm", a.head_dim)
    return out


def mod_unit(a: Arch, seed: int, kind: str, index: int, std: float = 0.02, bf16_exact: bool = True) -> dict:
    d, out = a.hidden, {}
    unit = f"{kind}.{index}.mod"
    if kind == "double":
        _lin(out, seed, unit, "img_mod.lin", d, 6 * d, std, bf16_exact)
        _lin(out, seed, unit, "txt_mod.lin", d, 6 * d, std, bf16_exact)
    else:
        _lin(out, seed, unit, "modulation.lin", d, 3 * d, std, bf16_exact)
    return out


def globals_unit(a: Arch, seed: int, std: float = 0.02, bf16_exact: bool = True) -> dict:
    d, out, unit = a.hidden, {}, "globals"
    _lin(out, seed, unit, "img_in", a.in_channels, d, std, bf16_exact)
    _lin(out, seed, unit, "txt_in", a.context_dim, d, std, bf16_exact)
    _lin(out, seed, unit, "time_in.in_layer", 256, d, std, bf16_exact)
    _lin(out, seed, unit, "time_in.out_layer", d, d, std, bf16_exact)
    _lin(out, seed, unit, "vector_in.in_layer", a.vec_dim, d, std, bf16_exact)
    _lin(out, seed, unit, "vector_in.out_layer", d, d, std, bf16_exact)
    if a.guidance_embed:
        _lin(out, seed, unit, "guidance_in.in_layer", 256, d, std, bf16_exact)
        _lin(out, seed, unit, "guidance_in.out_layer", d, d, std, bf16_exact)
    _lin(out, seed, unit, "final_layer.linear", d, a.in_channels, std, bf16_exact)
    _lin(out, seed, unit, "final_layer.adaLN_modulation.1", d, 2 * d, std, bf16_exact)
    return out


def all_units(a: Arch, seed: int, std: float = 0.02, bf16_exact: bool = True) -> dict[str, dict]:
    units = {"globals": globals_unit(a, seed, std, bf16_exact)}
    for i in range(a.depth_double):
        units[f"double.{i}"] = double_unit(a, seed, i, std, bf16_exact)
        units[f"double.{i}.mod"] = mod_unit(a, seed, "double", i, std, bf16_exact)
    for i in range(a.depth_single):
        units[f"single.{i}"] = single_unit(a, seed, i, std, bf16_exact)
        units[f"single.{i}.mod"] = mod_unit(a, seed, "single", i, std, bf16_exact)
    return units


def block_inputs(a: Arch, seed: int, l_img: int, l_txt: int, batch: int = 1, mod_std: float = 1.0):
    """Seeded block inputs: img [B,Li,D], txt [B,Lt,D] fp32 N(0,1); double/single mods N(0, mod_std),
    rounded to bf16 (the compute dtype they arrive in)."""
    d = a.hidden
    img = normal(seed, "in/img", (batch, l_img, d))
    txt = normal(seed, "in/txt", (batch, l_txt, d))
    dmod = _bf16_exact(normal(seed, "in/dmod", (batch, 12 * d), mod_std))
    smod = _bf16_exact(normal(seed, "in/smod", (batch, 3 * d), mod_std))
    fmod = _bf16_exact(normal(seed, "in/fmod", (batch, 2 * d), mod_std))
    return img, txt, dmod, smod, fmod
