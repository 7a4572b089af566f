"""Block-level parity on a B200: selas_b200's double_block / single_block / final_layer against the
reference's own outputs (golden vectors written by selas) and against the CPU oracle.

Tolerance (bf16 compute, fp32 residual stream): the B200 output is compared with the fp32 result on
the same inputs, and must be no further from it than the reference's own bf16 eager path is:
  rel-L2(B200, fp32) <= 1.5 x rel-L2(reference bf16, fp32)      (residual stream / velocity)
  max-abs(B200 - fp32) <= 2.0 x max-abs(reference bf16 - fp32)
"""

from __future__ import annotations

import pytest
import torch

from oracle import flux_ref as R
from oracle import weights as OW

from .conftest import GOLDEN, cuda_ok

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a B200")]

BF16, F32 = torch.bfloat16, torch.float32
DEV = "cuda"
REL_FACTOR, MAX_FACTOR = 1.5, 2.0


@pytest.fixture(scope="module", autouse=True)
def _lib_ready():
    from selas_b200 import _lib

    _lib.lib()
    yield
    torch.cuda.synchronize()
    assert _lib.device_status() == 0


def rel_l2(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return ((a - b).norm() / b.norm()).item()


def max_abs(a, b):
    return (a.double().cpu() - b.double().cpu()).abs().max().item()


def resident(tensors: dict):
    from selas_b200.model import ResidentUnit

    raw = {}
    for n, t in tensors.items():
        raw[n] = t.to(DEV, F32 if n.endswith("_norm.scale") else BF16)
    return ResidentUnit(raw)


@pytest.fixture(scope="module")
def mini():
    g = torch.load(GOLDEN / "blocks_mini.pt", weights_only=False)
    a = OW.Arch(**g["arch"])
    units = {"double": OW.double_unit(a, 7, 0), "single": OW.single_unit(a, 7, 0), "globals": OW.globals_unit(a, 7)}
    return g, a, units


def _check(name, got, ref32, ref16):
    spread_rel, spread_max = rel_l2(ref16, ref32), max_abs(ref16, ref32)
    e_rel, e_max = rel_l2(got, ref32), max_abs(got, ref32)
    assert e_rel <= REL_FACTOR * spread_rel, (name, e_rel, spread_rel)
    assert e_max <= MAX_FACTOR * spread_max, (name, e_max, spread_max)


def test_blocks_match_reference_golden(mini):
    from selas_b200 import flux as B

    g, a, units = mini
    wd, ws, wg = resident(units["double"]), resident(units["single"]), resident(units["globals"])
    for key, case in g["cases"].items():
        i = {k: v.to(DEV) for k, v in case["inputs"].items()}
        lt = i["txt"].shape[1]
        oi, ot = B.double_block(wd, i["img"], i["txt"], i["dmod"].to(BF16), i["cos"], i["sin"], a, BF16, False)
        # feed the golden fp32 double-block output into the single block so each block is judged alone
        x = torch.cat((case["f32"]["double_txt"], case["f32"]["double_img"]), 1).to(DEV)
        xs = B.single_block(ws, x, i["smod"].to(BF16), i["cos"], i["sin"], a, BF16, False)
        fo = B.final_layer(wg, case["f32"]["single"][:, lt:].to(DEV), i["fmod"].to(BF16), BF16)
        f32, b16 = case["f32"], case["bf16"]
        # single/final inputs above are the fp32 golden ones, so compare them with fresh oracle runs
        with torch.no_grad():
            xs32 = R.single_block(units["single"], x.cpu(), case["inputs"]["smod"], case["inputs"]["cos"],
                                  case["inputs"]["sin"], a.heads, a.mlp_hidden, F32)
            xs16 = R.single_block(units["single"], x.cpu(), case["inputs"]["smod"].to(BF16), case["inputs"]["cos"],
                                  case["inputs"]["sin"], a.heads, a.mlp_hidden, BF16)
            fin = case["f32"]["single"][:, lt:]
            fo32 = R.final_layer(units["globals"], fin, case["inputs"]["fmod"], F32)
            fo16 = R.final_layer(units["globals"], fin, case["inputs"]["fmod"].to(BF16), BF16)
        _check(f"{key}/double_img", oi, f32["double_img"], b16["double_img"])
        _check(f"{key}/double_txt", ot, f32["double_txt"], b16["double_txt"])
        _check(f"{key}/single", xs, xs32, xs16)
        _check(f"{key}/final", fo, fo32, fo16)


def test_blocks_are_deterministic(mini):
    from selas_b200 import flux as B

    g, a, units = mini
    wd = resident(units["double"])
    i = {k: v.to(DEV) for k, v in g["cases"]["b2_li64_lt16"]["inputs"].items()}
    r1 = B.double_block(wd, i["img"], i["txt"], i["dmod"].to(BF16), i["cos"], i["sin"], a, BF16, False)
    r2 = B.double_block(wd, i["img"], i["txt"], i["dmod"].to(BF16), i["cos"], i["sin"], a, BF16, False)
    assert torch.equal(r1[0], r2[0]) and torch.equal(r1[1], r2[1])


def test_segment_kernels_match_eager_segments(mini):
    """B200Kernels' seven segments against the oracle's eager segments (flux.py:164-200)."""
    from selas_b200.flux import B200Kernels

    k = B200Kernels()
    assert k.compiled is True
    gen = torch.Generator().manual_seed(3)
    x = torch.randn(2, 24, 256, generator=gen)
    mod = torch.randn(2, 3 * 256, generator=gen).to(BF16)
    sh, sc, gt = mod.float().unsqueeze(1).chunk(3, dim=-1)
    got = k.mod_in(x.to(DEV), sh.to(DEV), sc.to(DEV), BF16).cpu()
    torch.testing.assert_close(got.float(), R.mod_in(x, sh, sc, BF16).float(), rtol=2 ** -7, atol=1e-6)
    y = torch.randn(2, 24, 256, generator=gen).to(BF16)
    assert torch.equal(k.gated_add(x.to(DEV), gt.to(DEV), y.to(DEV), False).cpu(), R.gated_add(x, gt, y, False))
    h = torch.randn(2, 24, 1024, generator=gen).to(BF16)
    torch.testing.assert_close(k.gelu(h.to(DEV)).cpu().float(), R.gelu_tanh(h).float(), rtol=2 ** -7, atol=1e-6)


@pytest.mark.parametrize("batch", [1])
def test_full_size_double_block_c2(batch):
    """C2: one full FLUX double block (D=3072, 24 heads, MLP 12288), 512 text + 4096 image tokens,
    against the fp32 oracle on the CPU; the bf16 spread is measured on the same inputs."""
    from selas_b200 import flux as B

    a = OW.Arch()
    torch.set_num_threads(max(torch.get_num_threads(), 8))
    unit = OW.double_unit(a, 1, 0)
    img, txt, dmod, _, _ = OW.block_inputs(a, 2, 4096, 512, batch)
    cos, sin = R.rope_tables(torch.cat((R.text_ids(512), R.image_ids(1024, 1024)), 0), a.axes_dim)
    oi, ot = B.double_block(resident(unit), img.to(DEV), txt.to(DEV), dmod.to(DEV, BF16), cos.to(DEV), sin.to(DEV),
                            a, BF16, False)
    with torch.no_grad():
        ri, rt = R.double_block(unit, img, txt, dmod, cos, sin, a.heads, F32)
        bi, bt = R.double_block(unit, img, txt, dmod.to(BF16), cos, sin, a.heads, BF16)
    _check("c2/img", oi, ri, bi)
    _check("c2/txt", ot, rt, bt)


def test_full_size_single_block_c2():
    """One full FLUX single block (D=3072, 24 heads, MLP 12288; linear1 N=21504, linear2 K=15360) on the
    C2 joint sequence of 512 + 4096 tokens, against the fp32 oracle on the CPU, with the bf16 spread
    measured on the same inputs."""
    from selas_b200 import flux as B

    a = OW.Arch()
    torch.set_num_threads(max(torch.get_num_threads(), 8))
    unit = OW.single_unit(a, 1, 0)
    img, txt, _, smod, _ = OW.block_inputs(a, 3, 4096, 512, 1)
    x = torch.cat((txt, img), 1)
    cos, sin = R.rope_tables(torch.cat((R.text_ids(512), R.image_ids(1024, 1024)), 0), a.axes_dim)
    got = B.single_block(resident(unit), x.to(DEV), smod.to(DEV, BF16), cos.to(DEV), sin.to(DEV), a, BF16, False)
    with torch.no_grad():
        r32 = R.single_block(unit, x, smod, cos, sin, a.heads, a.mlp_hidden, F32)
        r16 = R.single_block(unit, x, smod.to(BF16), cos, sin, a.heads, a.mlp_hidden, BF16)
    _check("c2/single", got, r32, r16)


def test_mini_model_denoise_matches_oracle():
    """A whole 2-step denoise of a small FLUX (2 double + 2 single blocks, head_dim 128) through
    FluxStepper against the oracle's fp32 and bf16 runs: final-latent PSNR vs fp32 must be within
    3 dB of the reference bf16 path's."""
    from selas_b200.model import FluxArch, FluxStepper, ResidentUnit

    arch = OW.Arch(hidden=256, heads=2, mlp_hidden=1024, depth_double=2, depth_single=2, in_channels=64,
                   context_dim=256, vec_dim=256, axes_dim=(16, 56, 56))
    units = OW.all_units(arch, 3)
    dev_units = {n: resident(u) for n, u in units.items()}
    fa = FluxArch(**arch.__dict__)
    gen = torch.Generator().manual_seed(0)
    txt = torch.randn(1, 16, 256, generator=gen)
    pooled = torch.randn(1, 256, generator=gen)
    x0 = R.pack(R.get_noise(0, 128, 128))
    img_ids, txt_ids = R.image_ids(128, 128), R.text_ids(16)
    sig = R.get_schedule(2, x0.shape[1])
    st = FluxStepper(dev_units, fa)
    cond = st.prepare(sig, 3.5, pooled.to(DEV), txt.to(DEV), img_ids.to(DEV), txt_ids.to(DEV))
    out = st.denoise(x0.to(DEV), cond).cpu()
    with torch.no_grad():
        c32 = R.prepare(units, arch, sig, 3.5, pooled, txt, img_ids, txt_ids, F32)
        ref32, _ = R.denoise(units, arch, x0, c32, F32)
        c16 = R.prepare(units, arch, sig, 3.5, pooled, txt, img_ids, txt_ids, BF16)
        ref16, _ = R.denoise(units, arch, x0, c16, BF16)

    def psnr(a, b):
        mse = (a.double() - b.double()).pow(2).mean().item()
        peak = b.double().abs().max().item()
        return 10 * torch.log10(torch.tensor(peak * peak / max(mse, 1e-30))).item()

    assert torch.isfinite(out).all()
    assert psnr(out, ref32) >= psnr(ref16, ref32) - 3.0, (psnr(out, ref32), psnr(ref16, ref32))


def test_mini_model_denoise_matches_selas_runner():
    """FluxStepper on the B200 against selas's own FluxRunner (golden ``mini_runner.pt``, written by
    the reference over a real container): 4 Euler steps of a small FLUX (2 double + 2 single blocks,
    head_dim 128). Every step's velocity must be as close to selas's fp32 run as selas's bf16 run is
    (rel-L2 <= 1.5x, max-abs <= 2x that spread), and the final latent's PSNR against fp32 within 3 dB of
    selas's bf16 run's."""
    from selas_b200.model import FluxArch, FluxStepper

    g = torch.load(GOLDEN / "mini_runner.pt", weights_only=False)
    arch = OW.Arch(**g["arch"])
    units = OW.all_units(arch, 3)
    st = FluxStepper({n: resident(u) for n, u in units.items()}, FluxArch(**arch.__dict__))
    cond = st.prepare(g["sigmas"], 3.5, g["pooled"].to(DEV), g["txt"].to(DEV), g["img_ids"].to(DEV),
                      g["txt_ids"].to(DEV))
    x = g["x0"].to(DEV)
    sig = g["sigmas"]
    for s in range(len(sig) - 1):
        v = st.step(s, x, cond)
        _check(f"runner/step{s}", v.float().cpu(), g["f32"]["velocities"][s], g["bf16"]["velocities"][s])
        x = x + (sig[s + 1] - sig[s]) * v.float()
    out = x.cpu()

    def psnr(a, b):
        mse = (a.double() - b.double()).pow(2).mean().item()
        peak = b.double().abs().max().item()
        return 10 * torch.log10(torch.tensor(peak * peak / max(mse, 1e-30))).item()

    ref32, ref16 = g["f32"]["final"], g["bf16"]["final"]
    assert torch.isfinite(out).all()
    assert psnr(out, ref32) >= psnr(ref16, ref32) - 3.0, (psnr(out, ref32), psnr(ref16, ref32))
