"""FLUX autoencoder decoder restated with torch CPU ops — TEST INFRASTRUCTURE ONLY (the checker of
``selas_b200.vae`` and its kernels).

Follows ``selas/models/vae.py`` of tcox-coding/selas (``VaeDecoder.decode``, vae.py:78-96, and its
helpers ``_conv`` :51-52, ``_gn`` :54-55, ``_resnet`` :57-64, ``_attn`` :66-76) on a dict of the
``decoder`` unit's tensors, in fp32 (selas's dtype) or fp64 (a tighter reference for the tests).
``tf32`` rounds the operands of every product to tf32 first, as the B200 kernels feed the tensor
cores: round to nearest (ties away) for the values the kernels round before storing (weights, the
GroupNorm / upsampling outputs, q/k/v, P, O), truncation for the one input read unrounded (the
residual stream into a 1x1 ``nin_shortcut``, whose low mantissa bits the tensor core ignores).
Pinned by ``tests/test_oracle_golden.py`` against ``tests/golden/vae_mini.pt``, written by the
reference's own ``VaeDecoder``.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def tf32_round(t: torch.Tensor) -> torch.Tensor:
    """fp32 -> tf32 values (nearest, ties away from zero) in an fp32 tensor (finite inputs)."""
    u = t.to(torch.float32).contiguous().view(torch.int32)
    return ((u + 0x1000) & ~0x1FFF).view(torch.float32)


def tf32_trunc(t: torch.Tensor) -> torch.Tensor:
    """fp32 -> tf32 by dropping the low 13 mantissa bits (what the tensor core reads from an fp32 value)."""
    u = t.to(torch.float32).contiguous().view(torch.int32)
    return (u & ~0x1FFF).view(torch.float32)


class Decoder:
    def __init__(self, w: dict, ch_mult=(1, 2, 4, 4), num_res_blocks=2, scale_factor=0.3611, shift_factor=0.1159,
                 dtype=torch.float32, tf32: bool = False):
        self.w, self.ch_mult, self.nrb = w, tuple(ch_mult), num_res_blocks
        self.scale, self.shift, self.dt, self.tf32 = scale_factor, shift_factor, dtype, tf32

    def _g(self, name):
        return self.w[name].to(self.dt)

    def _op(self, t):
        return tf32_round(t).to(self.dt) if self.tf32 else t

    def conv(self, x, p, padding=1):
        b = self._g(p + ".bias") if p + ".bias" in self.w else None
        xin = tf32_trunc(x).to(self.dt) if self.tf32 and p.endswith("nin_shortcut") else self._op(x)
        return F.conv2d(xin, self._op(self._g(p + ".weight")), b, padding=padding)

    def gn(self, x, p):
        return F.group_norm(x, 32, self._g(p + ".weight"), self._g(p + ".bias"), eps=1e-6)

    def resnet(self, x, p):
        h = F.silu(self.gn(x, p + ".norm1"))
        h = self.conv(h, p + ".conv1")
        h = F.silu(self.gn(h, p + ".norm2"))
        h = self.conv(h, p + ".conv2")
        if p + ".nin_shortcut.weight" in self.w:
            x = self.conv(x, p + ".nin_shortcut", padding=0)
        return x + h

    def attn(self, x, p):
        b, c, hh, ww = x.shape
        h = self.gn(x, p + ".norm")
        q, k, v = (self.conv(h, f"{p}.{n}", padding=0).reshape(b, c, hh * ww).transpose(1, 2) for n in "qkv")
        s = torch.matmul(self._op(q), self._op(k).transpose(1, 2)) / (c ** 0.5)
        a = torch.matmul(self._op(torch.softmax(s, dim=-1)), self._op(v))  # [b, L, c]
        a = a.transpose(1, 2).reshape(b, c, hh, ww)
        return x + self.conv(a, p + ".proj_out", padding=0)

    @torch.no_grad()
    def decode(self, z: torch.Tensor) -> torch.Tensor:
        h = self.conv((z.to(torch.float32) / self.scale + self.shift).to(self.dt), "conv_in")
        h = self.resnet(h, "mid.block_1")
        h = self.attn(h, "mid.attn_1")
        h = self.resnet(h, "mid.block_2")
        for lvl in reversed(range(len(self.ch_mult))):
            for i in range(self.nrb + 1):
                h = self.resnet(h, f"up.{lvl}.block.{i}")
            if lvl != 0:
                h = F.interpolate(h, scale_factor=2.0, mode="nearest")
                h = self.conv(h, f"up.{lvl}.upsample.conv")
        h = F.silu(self.gn(h, "norm_out"))
        h = self.conv(h, "conv_out")
        return h.to(torch.float32).clamp_(-1, 1)


def random_decoder_weights(ch=128, ch_mult=(1, 2, 4, 4), num_res_blocks=2, z_channels=16, out_ch=3, seed=0) -> dict:
    """Random weights in the decoder unit's LDM key layout, scaled so activations stay O(1) through the
    network (He-like conv init, GroupNorm affine near identity)."""
    g = torch.Generator().manual_seed(seed)
    w = {}

    def conv(p, co, ci, k):
        w[p + ".weight"] = torch.randn(co, ci, k, k, generator=g) * (1.0 / (ci * k * k)) ** 0.5
        w[p + ".bias"] = torch.randn(co, generator=g) * 0.02

    def norm(p, c):
        w[p + ".weight"] = 1.0 + 0.1 * torch.randn(c, generator=g)
        w[p + ".bias"] = 0.1 * torch.randn(c, generator=g)

    def resnet(p, ci, co):
        norm(p + ".norm1", ci)
        conv(p + ".conv1", co, ci, 3)
        norm(p + ".norm2", co)
        conv(p + ".conv2", co, co, 3)
        if ci != co:
            conv(p + ".nin_shortcut", co, ci, 1)

    block_in = ch * ch_mult[-1]
    conv("conv_in", block_in, z_channels, 3)
    resnet("mid.block_1", block_in, block_in)
    norm("mid.attn_1.norm", block_in)
    for n in ("q", "k", "v", "proj_out"):
        conv(f"mid.attn_1.{n}", block_in, block_in, 1)
    resnet("mid.block_2", block_in, block_in)
    for lvl in reversed(range(len(ch_mult))):
        block_out = ch * ch_mult[lvl]
        for i in range(num_res_blocks + 1):
            resnet(f"up.{lvl}.block.{i}", block_in, block_out)
            block_in = block_out
        if lvl != 0:
            conv(f"up.{lvl}.upsample.conv", block_in, block_in, 3)
    norm("norm_out", block_in)
    conv("conv_out", out_ch, block_in, 3)
    return w
