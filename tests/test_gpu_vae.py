"""The FLUX VAE decoder on a B200 (csrc/vae.cu through the C-ABI), against the oracle.

Kernel level: the tf32 implicit-GEMM conv (3x3 / 1x1, ragged image sizes, every BN variant and the
strip kernel of rows >= 128 pixels, bias, residual, tf32-rounded and NCHW-clamped outputs) against an fp64 conv of the same tf32 operands, so
that only the fp32 accumulation order separates the two; GroupNorm (+ SiLU) against fp64
F.group_norm; upsampling and the latent preparation bit for bit; the row softmax.

Decoder level: ``VaeDecoder.decode`` / ``decode_tiled`` on the mini decoder of
tests/golden/vae_mini.pt (written by selas's own VaeDecoder, fp32) and a full FLUX-shaped decoder
(ch 128, ch_mult (1, 2, 4, 4), two ResNets + 1 per level) against the fp64 oracle with the kernels'
tf32 operand rounding. Tolerances: the fp32 reference differs from the tf32 path by the tf32 rounding
of the products (2^-11 relative per operand), which is the difference torch's own fp32 convolutions
on tensor-core GPUs show; the tf32-operand fp64 oracle is held to a tolerance ten times tighter.
"""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from oracle import vae_ref as VR

from .conftest import GOLDEN, cuda_ok

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a B200")]

DEV = "cuda"
F64 = torch.float64


@pytest.fixture(scope="module", autouse=True)
def _lib_ready():
    from selas_b200 import _lib

    _lib.lib()
    yield
    torch.cuda.synchronize()
    assert _lib.device_status() == 0


def _rand(*shape, seed=0, scale=1.0):
    return torch.randn(*shape, generator=torch.Generator().manual_seed(seed)) * scale


@pytest.mark.parametrize("b,h,w,cin,cout,k", [
    (1, 8, 16, 32, 256, 3),     # one full tile, BN 256
    (2, 13, 7, 64, 128, 3),     # ragged tiles (tw 8), batch 2, BN 128
    (1, 20, 37, 128, 3, 3),     # conv_out-like: 3 outputs, BN 16, partial N tile
    (1, 9, 40, 96, 48, 1),      # 1x1, BN 64 with a partial N tile
    (1, 16, 16, 512, 512, 3),   # two N tiles of 256, 144 K steps
    (1, 4, 2, 32, 200, 1),      # tiny image (tw 2, th 64)
    (1, 5, 128, 64, 128, 3),    # strip kernel: odd height (the last tile's second row masked)
    (2, 4, 200, 32, 256, 3),    # strip kernel: ragged width, batch 2, two N blocks
    (1, 2, 384, 128, 128, 3),   # strip kernel: three strips per row
])
@pytest.mark.parametrize("mode", ["plain", "resid_round", "nchw"])
def test_conv_matches_fp64_tf32(b, h, w, cin, cout, k, mode):
    from selas_b200 import _lib
    from selas_b200.vae import _rows, conv_raw

    if mode == "nchw" and cout > 16:
        pytest.skip("the NCHW clamp output is the 3-channel last conv")
    x = VR.tf32_round(_rand(b, h, w, cin, seed=1))
    wt = _rand(cout, cin, k, k, seed=2, scale=(1.0 / (cin * k * k)) ** 0.5)
    bias = _rand(cout, seed=3, scale=0.1)
    resid = _rand(b, h, w, cout, seed=4) if mode == "resid_round" else None
    ref = F.conv2d(x.permute(0, 3, 1, 2).to(F64), VR.tf32_round(wt).to(F64), bias.to(F64), padding=k // 2)
    flags = 0
    if mode == "resid_round":
        ref = ref + resid.permute(0, 3, 1, 2).to(F64)
        flags = _lib.FB_VAE_ROUND_OUT
    if mode == "nchw":
        ref = ref.clamp(-1, 1)
        flags = _lib.FB_VAE_OUT_NCHW_CLAMP
        out = torch.full((b, cout, h, w), 7.0, device=DEV)
    else:
        ref = ref.permute(0, 2, 3, 1)
        out = torch.full((b, h, w, cout), 7.0, device=DEV)
    wr = _rows(wt.to(DEV))
    r_dev = None if resid is None else resid.to(DEV).contiguous()
    conv_raw(x.to(DEV), cin, wr, cout, k, bias.to(DEV), r_dev, out, cout, flags, b, h, w)
    torch.cuda.synchronize()
    got = out.cpu().to(F64)
    scale = ref.abs().max().item() + 1e-6
    if mode == "resid_round":  # each output carries its own tf32 rounding (2^-11 relative) on top
        assert ((got - ref).abs() <= 6e-4 * ref.abs() + 2e-5 * scale).all()
        assert torch.equal(VR.tf32_round(out.cpu()), out.cpu())  # outputs are tf32 values
    else:
        err = (got - ref).abs().max().item() / scale
        assert err < 2e-5, err


def test_conv_as_strided_gemm():
    """S = Q K^T with Q and K column slices of one [L, 3C] matrix (the mid-block attention's use)."""
    from selas_b200.vae import conv_raw

    h, w, c = 6, 16, 64
    L = h * w
    qkv = VR.tf32_round(_rand(h, w, 3 * c, seed=5))
    s = torch.zeros(L, 128, device=DEV)
    base = qkv.to(DEV)
    conv_raw(base, 3 * c, base[..., c:2 * c], L, 1, None, None, s, 128, 0, 1, h, w, cin=c, ld_w=3 * c)
    torch.cuda.synchronize()
    q = qkv.reshape(L, 3 * c)[:, :c].to(F64)
    k = qkv.reshape(L, 3 * c)[:, c:2 * c].to(F64)
    ref = q @ k.T
    assert ((s.cpu()[:, :L].to(F64) - ref).abs().max() / ref.abs().max()).item() < 2e-5
    assert not s.cpu()[:, L:].any()


@pytest.mark.parametrize("c,b,h,w", [(128, 1, 16, 24), (256, 2, 7, 9), (512, 1, 32, 32)])
@pytest.mark.parametrize("silu", [False, True])
def test_group_norm(c, b, h, w, silu):
    from selas_b200 import _lib, ops

    x = _rand(b, h, w, c, seed=6, scale=3.0) + 0.5
    gamma, beta = 1 + 0.1 * _rand(c, seed=7), 0.1 * _rand(c, seed=8)
    xd, gd, bd = x.to(DEV), gamma.to(DEV), beta.to(DEV)  # held until the kernel has run
    out = torch.full_like(xd, 7.0)
    work = torch.empty(_lib.lib().fb_vae_group_norm_work_doubles(b), dtype=F64, device=DEV)
    _lib.check(_lib.lib().fb_vae_group_norm(xd.data_ptr(), c, b, h * w, c, gd.data_ptr(), bd.data_ptr(), 1e-6,
                                            int(silu), 0, out.data_ptr(), c, work.data_ptr(), ops._stream()), "gn")
    torch.cuda.synchronize()
    ref = F.group_norm(x.permute(0, 3, 1, 2).to(F64), 32, gamma.to(F64), beta.to(F64), eps=1e-6)
    if silu:
        ref = F.silu(ref)
    got = out.cpu().permute(0, 3, 1, 2).to(F64)
    assert (got - ref).abs().max().item() < 1e-5


@pytest.mark.parametrize("b,h,w", [(1, 20, 37), (2, 9, 64), (1, 64, 96)])
def test_norm_out_conv_matches_the_two_kernel_path(b, h, w):
    """fb_vae_norm_out_conv (GroupNorm + SiLU + the 3x3 conv to 3 channels, clamped, NCHW) against
    fb_vae_group_norm followed by the tensor-core conv, and both against an fp64 conv of the same
    tf32 inputs: the fused kernel sums in another order, nothing else."""
    from selas_b200 import _lib, ops
    from selas_b200.vae import _rows, conv_raw

    c = 128
    x = _rand(b, h, w, c, seed=21, scale=3.0) + 0.5
    gamma, beta = 1 + 0.1 * _rand(c, seed=22), 0.1 * _rand(c, seed=23)
    wt = _rand(3, c, 3, 3, seed=24, scale=(1.0 / (9 * c)) ** 0.5)
    bias = _rand(3, seed=25, scale=0.1)
    xd, gd, bd = x.to(DEV), gamma.to(DEV), beta.to(DEV)
    wr = _rows(wt.to(DEV))  # [9, 3, 128] tf32
    bias_d = bias.to(DEV)
    work = torch.empty(_lib.lib().fb_vae_group_norm_work_doubles(b), dtype=F64, device=DEV)
    fused = torch.full((b, 3, h, w), 7.0, device=DEV)
    _lib.check(_lib.lib().fb_vae_norm_out_conv(xd.data_ptr(), b, h, w, c, gd.data_ptr(), bd.data_ptr(), 1e-6,
                                               wr.data_ptr(), bias_d.data_ptr(), 3, fused.data_ptr(),
                                               work.data_ptr(), ops._stream()), "norm_out_conv")
    t = torch.empty_like(xd)
    _lib.check(_lib.lib().fb_vae_group_norm(xd.data_ptr(), c, b, h * w, c, gd.data_ptr(), bd.data_ptr(), 1e-6, 1, 1,
                                            t.data_ptr(), c, work.data_ptr(), ops._stream()), "gn")
    two = torch.full((b, 3, h, w), 7.0, device=DEV)
    conv_raw(t, c, wr, 3, 3, bias_d, None, two, 3, _lib.FB_VAE_OUT_NCHW_CLAMP, b, h, w)
    torch.cuda.synchronize()
    ref = F.conv2d(t.cpu().permute(0, 3, 1, 2).to(F64), VR.tf32_round(wt).to(F64), bias.to(F64), padding=1).clamp(-1, 1)
    scale = ref.abs().max().item() + 1e-6
    for got in (fused, two):
        err = (got.cpu().to(F64) - ref).abs().max().item() / scale
        assert err < 2e-5, err


def test_upsample_and_latent_prep_bit_exact():
    from selas_b200 import _lib, ops

    x = _rand(2, 5, 7, 64, seed=8)
    xd = x.to(DEV)
    out = torch.empty(2, 10, 14, 64, device=DEV)
    _lib.check(_lib.lib().fb_vae_upsample2(xd.data_ptr(), 2, 5, 7, 64, 0, out.data_ptr(), ops._stream()), "up")
    ref = F.interpolate(x.permute(0, 3, 1, 2), scale_factor=2.0, mode="nearest").permute(0, 2, 3, 1)
    assert torch.equal(out.cpu(), ref)
    z = _rand(2, 16, 6, 10, seed=9)
    zd = z.to(DEV)
    zp = torch.full((2, 6, 10, 32), 7.0, device=DEV)
    _lib.check(_lib.lib().fb_vae_latent_prep(zd.data_ptr(), 2, 16, 6, 10, 32, 0.3611, 0.1159, zp.data_ptr(),
                                             ops._stream()), "prep")
    ref = torch.zeros(2, 6, 10, 32)
    ref[..., :16] = VR.tf32_round(z / torch.tensor(0.3611, dtype=torch.float32) + 0.1159).permute(0, 2, 3, 1)
    assert torch.equal(zp.cpu(), ref)


@pytest.mark.parametrize("n", [96, 16384, 1001])
def test_softmax_rows(n):
    from selas_b200 import _lib, ops

    rows, ld = 5, (n + 31) // 32 * 32
    s = torch.zeros(rows, ld)
    s[:, :n] = _rand(rows, n, seed=10, scale=30.0)
    d = s.to(DEV)
    _lib.check(_lib.lib().fb_vae_softmax_rows(d.data_ptr(), rows, n, ld, 0.05, 0, ops._stream()), "softmax")
    ref = torch.softmax(s[:, :n].to(F64) * 0.05, dim=-1)
    got = d.cpu()
    assert (got[:, :n].to(F64) - ref).abs().max().item() < 2e-6
    assert not got[:, n:].any()


def _mini():
    g = torch.load(GOLDEN / "vae_mini.pt")
    cfg = dict(g["config"])
    seed = cfg.pop("seed")
    return g, cfg, VR.random_decoder_weights(seed=seed, **cfg)


def _check_decode(out, w, z, ch_mult, nrb):
    """The kernels' image against the fp64 decoder: no further from it than the oracle with the same tf32
    operands and fp32 arithmetic (what a tensor-core GPU computes for selas's fp32 decoder) is, up to
    run-to-run rounding noise; and, as 8-bit pixels (selas/pipeline.py:572), at most one level apart."""
    d64 = VR.Decoder(w, ch_mult, nrb, dtype=F64).decode(z)
    t32 = VR.Decoder(w, ch_mult, nrb, dtype=torch.float32, tf32=True).decode(z).to(F64)
    spread = (t32 - d64).abs()
    err = (out.to(F64) - d64).abs()
    assert err.mean().item() <= 1.5 * spread.mean().item() + 1e-6, (err.mean().item(), spread.mean().item())
    assert err.max().item() <= 3.0 * spread.max().item() + 1e-5, (err.max().item(), spread.max().item())
    px = ((out + 1) * 127.5).round().clamp(0, 255)
    rpx = ((d64.float() + 1) * 127.5).round().clamp(0, 255)
    assert (px - rpx).abs().max().item() <= 1
    return err


def test_decode_mini_matches_reference():
    from selas_b200.vae import VaeConfig, VaeDecoder

    g, cfg, w = _mini()
    dec = VaeDecoder(w, VaeConfig(**cfg))
    out = dec.decode(g["z"].to(DEV)).cpu()
    assert out.shape == g["out"].shape
    _check_decode(out, w, g["z"], cfg["ch_mult"], cfg["num_res_blocks"])
    # selas's own fp32 output (the golden file): within the tf32 spread too
    assert (out - g["out"]).abs().mean().item() < 1e-3
    tiled = dec.decode_tiled(g["z"].to(DEV), tile=6, overlap=2).cpu()
    et = (tiled - g["out_tiled"]).abs()
    assert et.max().item() < 1e-2 and et.mean().item() < 1e-3, (et.max().item(), et.mean().item())
    # deterministic: the same image twice
    assert torch.equal(dec.decode(g["z"].to(DEV)).cpu(), out)


def test_decode_flux_shaped_decoder():
    """ch 128, ch_mult (1, 2, 4, 4), 2 ResNets + 1 per level (FLUX's decoder), 16 x 16 latent -> 128^2."""
    from selas_b200.vae import VaeConfig, VaeDecoder

    w = VR.random_decoder_weights(seed=11)
    z = _rand(1, 16, 16, 16, seed=12)
    out = VaeDecoder(w, VaeConfig()).decode(z.to(DEV)).cpu()
    assert out.shape == (1, 3, 128, 128)
    _check_decode(out, w, z, (1, 2, 4, 4), 2)
