"""FLUX autoencoder decoder on the B200 kernels (selas/models/vae.py): the step after denoising.

The same API as selas's ``VaeConfig`` / ``VaeDecoder`` (``decode``, ``decode_tiled``) over the same
weights (the ``decoder`` unit of the LDM key layout), run by the kernels of ``csrc/vae.cu``:

* activations NHWC fp32 in HBM; every convolution (3x3 and 1x1) is the tcgen05 implicit-GEMM kernel
  ``fb_vae_conv`` in tf32 (the arithmetic torch uses for fp32 convolutions on tensor-core GPUs), with
  the bias, the ResNet residual add, the tf32 rounding of outputs that feed another product, and the
  final clamp + NCHW store in its epilogue;
* GroupNorm (+ SiLU) with fp64 statistics (``fb_vae_group_norm``), nearest 2x upsampling, the latent
  scaling (``fb_vae_latent_prep``);
* the mid-block attention (one head of 512 channels over the h*w latent pixels) as three products on
  the same conv kernel — a fused q/k/v 1x1 conv, S = Q K^T, O = P V — around a row softmax.

Weights are converted once at construction: conv kernels permuted from [Cout, Cin, k, k] to the
tap-major [k*k, Cout, Cin] (Cin padded to a multiple of 32 with zeros) and rounded to tf32, q/k/v fused
into one [3C, C] matrix. ``decode_tiled`` follows selas's tiling and linear blend (vae.py:98-131); its blend is
elementwise torch on the device.
"""

from __future__ import annotations

import math
from dataclasses import asdict, dataclass

import torch

from . import _lib
from . import profile as _prof
from ._lib import FluxB200Error
from .ops import _count, _need, _stream

F32 = torch.float32


@dataclass
class VaeConfig:
    """selas/models/vae.py:20-40."""

    ch: int = 128
    ch_mult: tuple[int, ...] = (1, 2, 4, 4)
    num_res_blocks: int = 2
    z_channels: int = 16
    out_ch: int = 3
    scale_factor: float = 0.3611
    shift_factor: float = 0.1159

    @classmethod
    def from_dict(cls, d: dict) -> "VaeConfig":
        kw = {k: v for k, v in d.items() if k in cls.__dataclass_fields__}
        if "ch_mult" in kw:
            kw["ch_mult"] = tuple(kw["ch_mult"])
        return cls(**kw)

    def to_dict(self) -> dict:
        d = asdict(self)
        d["ch_mult"] = list(self.ch_mult)
        return d


def _tf32(t: torch.Tensor) -> torch.Tensor:
    """Round fp32 to tf32 (nearest, ties away from zero; the kernels' cvt.rna), in an fp32 container."""
    u = t.contiguous().view(torch.int32)
    return ((u + 0x1000) & ~0x1FFF).view(F32)


def _rows(t: torch.Tensor, cin_pad: int | None = None) -> torch.Tensor:
    """torch conv weight [Cout, Cin, k, k] -> tap-major [k*k, Cout, Cin_pad] fp32 (tf32-rounded)."""
    co, ci, kh, kw = t.shape
    w = t.to(F32).permute(2, 3, 0, 1)
    cp = cin_pad or ci
    if cp != ci:
        w = torch.nn.functional.pad(w, (0, cp - ci))
    return _tf32(w.reshape(kh * kw, co, cp).contiguous())


def _pad32(c: int) -> int:
    return (c + 31) // 32 * 32


class _Weights:
    """The decoder unit's tensors, looked up by name (a dict, or selas's UnitView-like get/has)."""

    def __init__(self, src, device):
        if hasattr(src, "view") and callable(getattr(src, "view")) and not isinstance(src, dict):
            src = src.view("decoder")
        self.src, self.device = src, device

    def has(self, name: str) -> bool:
        return name in self.src if isinstance(self.src, dict) else self.src.has(name)

    def get(self, name: str) -> torch.Tensor:
        t = self.src[name] if isinstance(self.src, dict) else self.src.get(name, F32)
        return t.to(self.device, F32).contiguous()


class VaeDecoder:
    """selas/models/vae.py:42-131 on the B200 kernels. ``store``: a dict of the ``decoder`` unit's
    tensors (LDM key layout), or a store whose ``view("decoder")`` has ``get(name, dtype)`` / ``has``."""

    def __init__(self, store, cfg: VaeConfig, dtype: torch.dtype = F32, device=None):
        if dtype != F32:
            raise FluxB200Error("the B200 VAE decoder computes in fp32 (tf32 tensor-core products)")
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.cfg, self.device = cfg, torch.device(device)
        if self.device.type != "cuda":
            raise FluxB200Error("VaeDecoder needs a CUDA device")
        _lib.lib()
        w = _Weights(store, self.device)
        self.p: dict[str, torch.Tensor] = {}
        self.convs: dict[str, tuple[torch.Tensor, torch.Tensor | None, int, int, int]] = {}
        self._conv("conv_in", w, cin_pad=_pad32(cfg.z_channels))
        self._resnet("mid.block_1", w)
        self._attn("mid.attn_1", w)
        self._resnet("mid.block_2", w)
        for lvl in reversed(range(len(cfg.ch_mult))):
            for i in range(cfg.num_res_blocks + 1):
                self._resnet(f"up.{lvl}.block.{i}", w)
            if lvl != 0:
                self._conv(f"up.{lvl}.upsample.conv", w)
        self._norm("norm_out", w)
        self._conv("conv_out", w)
        # norm_out + conv_out run as one kernel when the shapes are FLUX's (128 -> 3 channels, 3x3)
        _, _, co, ci, k = self.convs["conv_out"]
        self._fused_out = (co, ci, k) == (3, 128, 3)
        self._work: dict[int, torch.Tensor] = {}

    # ------------------------------------------------------------------ weight conversion
    def _conv(self, p: str, w: _Weights, cin_pad: int | None = None) -> None:
        wt = w.get(p + ".weight")
        co, ci, k, _ = wt.shape
        cp = cin_pad or ci
        if cp % 32:
            raise FluxB200Error(f"{p}: {ci} input channels; the conv kernel needs a multiple of 32")
        b = w.get(p + ".bias") if w.has(p + ".bias") else None
        self.convs[p] = (_rows(wt, cp), b, co, cp, k)

    def _norm(self, p: str, w: _Weights) -> None:
        self.p[p + ".weight"] = w.get(p + ".weight")
        self.p[p + ".bias"] = w.get(p + ".bias")

    def _resnet(self, p: str, w: _Weights) -> None:
        self._norm(p + ".norm1", w)
        self._conv(p + ".conv1", w)
        self._norm(p + ".norm2", w)
        self._conv(p + ".conv2", w)
        if w.has(p + ".nin_shortcut.weight"):
            self._conv(p + ".nin_shortcut", w)

    def _attn(self, p: str, w: _Weights) -> None:
        self._norm(p + ".norm", w)
        qkv = torch.cat([w.get(f"{p}.{n}.weight") for n in ("q", "k", "v")], 0)
        bias = torch.cat([w.get(f"{p}.{n}.bias") for n in ("q", "k", "v")], 0)
        self.convs[p + ".qkv"] = (_rows(qkv), bias, qkv.shape[0], qkv.shape[1], 1)
        self._conv(p + ".proj_out", w)

    # ------------------------------------------------------------------ kernel calls
    def _run_conv(self, x: torch.Tensor, p: str, resid: torch.Tensor | None = None, flags: int = 0) -> torch.Tensor:
        wt, b, co, cin, k = self.convs[p]  # wt: [k*k, co, cin]
        bsz, h, wd, c = x.shape
        _need(c == cin, f"{p}: input has {c} channels, the weights {cin}")
        if flags & _lib.FB_VAE_OUT_NCHW_CLAMP:
            out = torch.empty(bsz, co, h, wd, dtype=F32, device=x.device)
        else:
            out = torch.empty(bsz, h, wd, co, dtype=F32, device=x.device)
        conv_raw(x, c, wt, co, k, b, resid, out, co, flags, bsz, h, wd)
        return out

    def _gn(self, x: torch.Tensor, p: str, silu: bool, round_tf32: bool = True) -> torch.Tensor:
        bsz, h, wd, c = x.shape
        out = torch.empty_like(x)
        work = self._work.get(bsz)
        if work is None:
            n = _lib.lib().fb_vae_group_norm_work_doubles(bsz)
            work = self._work[bsz] = torch.empty(n, dtype=torch.float64, device=x.device)
        with _prof.region("vae_gn", 0.0, 3.0 * x.numel() * 4):
            _lib.check(_lib.lib().fb_vae_group_norm(x.data_ptr(), c, bsz, h * wd, c, self.p[p + ".weight"].data_ptr(),
                                                    self.p[p + ".bias"].data_ptr(), 1e-6, int(silu), int(round_tf32),
                                                    out.data_ptr(), c, work.data_ptr(), _stream()),
                       "fb_vae_group_norm")
        _count()
        return out

    def _resnet_fwd(self, x: torch.Tensor, p: str) -> torch.Tensor:
        """selas/models/vae.py:57-64."""
        h = self._gn(x, p + ".norm1", True)
        h = self._run_conv(h, p + ".conv1")
        h = self._gn(h, p + ".norm2", True)
        s = self._run_conv(x, p + ".nin_shortcut") if p + ".nin_shortcut" in self.convs else x
        return self._run_conv(h, p + ".conv2", resid=s)

    def _attn_fwd(self, x: torch.Tensor, p: str) -> torch.Tensor:
        """selas/models/vae.py:66-76: one head over the h*w pixels, softmax(Q K^T / sqrt(C)) V."""
        bsz, h, wd, c = x.shape
        L = h * wd
        lp = _pad32(L)  # P's row stride: the P V product reads L as its K dimension, in steps of 32
        t = self._gn(x, p + ".norm", False)
        qkv = self._run_conv(t, p + ".qkv", flags=_lib.FB_VAE_ROUND_OUT)  # [B, h, w, 3C]
        o = torch.empty(bsz, h, wd, c, dtype=F32, device=x.device)
        pad = torch.zeros if lp != L else torch.empty  # padding columns L.. must read as zero
        s = pad(L, lp, dtype=F32, device=x.device)
        vt = pad(c, lp, dtype=F32, device=x.device)
        for b in range(bsz):
            base = qkv[b]
            # S = Q K^T: Q [L, C] and K [L, C] are column slices (pixel stride 3C) of the fused output
            conv_raw(base, 3 * c, base[..., c:2 * c], L, 1, None, None, s, lp, 0, 1, h, wd, cin=c, ld_w=3 * c)
            with _prof.region("vae_softmax", 0.0, 2.0 * L * L * 4):
                _lib.check(_lib.lib().fb_vae_softmax_rows(s.data_ptr(), L, L, lp, 1.0 / math.sqrt(c), 1, _stream()),
                           "fb_vae_softmax_rows")
            _count()
            _lib.check(_lib.lib().fb_vae_transpose(base[..., 2 * c:].data_ptr(), L, c, 3 * c, vt.data_ptr(), lp,
                                                   _stream()), "fb_vae_transpose")
            _count()
            # O = P V: P [L, lp] read as an image of lp channels, V^T [C, lp] as the weights
            conv_raw(s, lp, vt, c, 1, None, None, o[b], c, _lib.FB_VAE_ROUND_OUT, 1, h, wd, cin=lp, ld_w=lp)
        return self._run_conv(o, p + ".proj_out", resid=x)

    # ------------------------------------------------------------------ public API
    @torch.no_grad()
    def decode(self, z: torch.Tensor) -> torch.Tensor:
        """z [B, 16, h, w] (sampler latents) -> image [B, 3, 8h, 8w] in [-1, 1] fp32 (vae.py:78-96)."""
        cfg = self.cfg
        z = z.to(self.device, F32).contiguous()
        bsz, zc, h, wd = z.shape
        _need(zc == cfg.z_channels, f"latents have {zc} channels, the decoder {cfg.z_channels}")
        cp = _pad32(zc)
        x = torch.empty(bsz, h, wd, cp, dtype=F32, device=self.device)
        _lib.check(_lib.lib().fb_vae_latent_prep(z.data_ptr(), bsz, zc, h, wd, cp, cfg.scale_factor, cfg.shift_factor,
                                                 x.data_ptr(), _stream()), "fb_vae_latent_prep")
        _count()
        x = self._run_conv(x, "conv_in")
        x = self._resnet_fwd(x, "mid.block_1")
        x = self._attn_fwd(x, "mid.attn_1")
        x = self._resnet_fwd(x, "mid.block_2")
        for lvl in reversed(range(len(cfg.ch_mult))):
            for i in range(cfg.num_res_blocks + 1):
                x = self._resnet_fwd(x, f"up.{lvl}.block.{i}")
            if lvl != 0:
                b_, h_, w_, c_ = x.shape
                up = torch.empty(b_, 2 * h_, 2 * w_, c_, dtype=F32, device=self.device)
                with _prof.region("vae_upsample", 0.0, 5.0 * x.numel() * 4):
                    _lib.check(_lib.lib().fb_vae_upsample2(x.data_ptr(), b_, h_, w_, c_, 1, up.data_ptr(), _stream()),
                               "fb_vae_upsample2")
                _count()
                x = self._run_conv(up, f"up.{lvl}.upsample.conv")
        if not self._fused_out:
            x = self._gn(x, "norm_out", True)
            return self._run_conv(x, "conv_out", flags=_lib.FB_VAE_OUT_NCHW_CLAMP)
        return self._norm_out_conv(x)

    def _norm_out_conv(self, x: torch.Tensor) -> torch.Tensor:
        """norm_out (GroupNorm + SiLU) and conv_out (selas/models/vae.py:94-95) as one kernel."""
        bsz, h, wd, c = x.shape
        x = x.contiguous()
        out = torch.empty(bsz, 3, h, wd, dtype=F32, device=x.device)
        work = self._work.get(bsz)
        if work is None:
            n = _lib.lib().fb_vae_group_norm_work_doubles(bsz)
            work = self._work[bsz] = torch.empty(n, dtype=torch.float64, device=x.device)
        wt, b, _, _, _ = self.convs["conv_out"]
        flops = 2.0 * bsz * h * wd * 3 * 9 * c
        with _prof.region("vae_conv", flops, 4.0 * bsz * h * wd * (c + 3)):
            _lib.check(_lib.lib().fb_vae_norm_out_conv(x.data_ptr(), bsz, h, wd, c, self.p["norm_out.weight"].data_ptr(),
                                                       self.p["norm_out.bias"].data_ptr(), 1e-6, wt.data_ptr(),
                                                       None if b is None else b.data_ptr(), 3, out.data_ptr(),
                                                       work.data_ptr(), _stream()), "fb_vae_norm_out_conv")
        _count()
        return out

    @torch.no_grad()
    def decode_tiled(self, z: torch.Tensor, tile: int = 64, overlap: int = 16) -> torch.Tensor:
        """Decode overlapping ``tile`` x ``tile`` latent tiles and blend them (vae.py:98-131)."""
        b, _, h, w = z.shape
        if h <= tile and w <= tile:
            return self.decode(z)
        up = 2 ** (len(self.cfg.ch_mult) - 1)
        stride = tile - overlap
        dev = self.device
        out = torch.zeros(b, 3, h * up, w * up, dtype=F32, device=dev)
        weight = torch.zeros(1, 1, h * up, w * up, dtype=F32, device=dev)
        ys = list(range(0, max(h - tile, 0) + 1, stride))
        xs = list(range(0, max(w - tile, 0) + 1, stride))
        if ys[-1] + tile < h:
            ys.append(h - tile)
        if xs[-1] + tile < w:
            xs.append(w - tile)
        ramp = overlap * up
        for y in ys:
            for x in xs:
                th, tw = min(tile, h - y), min(tile, w - x)
                dec = self.decode(z[:, :, y:y + th, x:x + tw])
                mask = torch.ones(1, 1, th * up, tw * up, device=dev)
                if ramp:
                    r = torch.linspace(0, 1, ramp + 2, device=dev)[1:-1]
                    if y > 0:
                        mask[:, :, :ramp, :] *= r.view(1, 1, -1, 1)
                    if y + th < h:
                        mask[:, :, -ramp:, :] *= r.flip(0).view(1, 1, -1, 1)
                    if x > 0:
                        mask[:, :, :, :ramp] *= r.view(1, 1, 1, -1)
                    if x + tw < w:
                        mask[:, :, :, -ramp:] *= r.flip(0).view(1, 1, 1, -1)
                out[:, :, y * up:(y + th) * up, x * up:(x + tw) * up] += dec * mask
                weight[:, :, y * up:(y + th) * up, x * up:(x + tw) * up] += mask
        return (out / weight.clamp_min(1e-6)).clamp_(-1, 1)


def random_weights(cfg: VaeConfig, device, seed: int = 0) -> dict:
    """Random decoder weights in the LDM key layout for ``cfg`` (benchmarks; there is no checkpoint):
    He-scaled convs, GroupNorm affine near identity, so activations stay O(1) through the network."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    w: dict[str, torch.Tensor] = {}

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

    cin = cfg.ch * cfg.ch_mult[-1]
    conv("conv_in", cin, cfg.z_channels, 3)
    resnet("mid.block_1", cin, cin)
    norm("mid.attn_1.norm", cin)
    for n in ("q", "k", "v", "proj_out"):
        conv(f"mid.attn_1.{n}", cin, cin, 1)
    resnet("mid.block_2", cin, cin)
    for lvl in reversed(range(len(cfg.ch_mult))):
        cout = cfg.ch * cfg.ch_mult[lvl]
        for i in range(cfg.num_res_blocks + 1):
            resnet(f"up.{lvl}.block.{i}", cin, cout)
            cin = cout
        if lvl != 0:
            conv(f"up.{lvl}.upsample.conv", cin, cin, 3)
    norm("norm_out", cin)
    conv("conv_out", cfg.out_ch, cin, 3)
    return {k: v.to(device) for k, v in w.items()}


def conv_raw(x: torch.Tensor, ld_in: int, wt: torch.Tensor, cout: int, k: int, bias, resid, out: torch.Tensor,
             ld_out: int, flags: int, bsz: int, h: int, wd: int, cin: int | None = None, ld_w: int | None = None) -> None:
    """``fb_vae_conv`` on raw views: x [bsz, h, wd, *] with pixel stride ld_in, tap-major weights
    [k*k, cout, cin] with row stride ld_w, output pixel stride ld_out (NHWC) or NCHW with
    FB_VAE_OUT_NCHW_CLAMP."""
    cin = cin if cin is not None else wt.shape[-1]
    ld_w = ld_w if ld_w is not None else wt.shape[-1]
    flops = 2.0 * bsz * h * wd * cout * k * k * cin
    with _prof.region("vae_conv", flops, 4.0 * (bsz * h * wd * (cin + cout))):
        _lib.check(_lib.lib().fb_vae_conv(x.data_ptr(), ld_in, bsz, h, wd, cin, wt.data_ptr(), ld_w, cout, k,
                                          None if bias is None else bias.data_ptr(),
                                          None if resid is None else resid.data_ptr(),
                                          0 if resid is None else resid.shape[-1], out.data_ptr(), ld_out, flags,
                                          _stream()), "fb_vae_conv")
    _count()


__all__ = ["VaeConfig", "VaeDecoder", "conv_raw", "random_weights"]
