"""The eager-PyTorch blocks that `python -m selas_b200.microbench --kernel block / step_yardstick` time
as the GPU bar of selas's default path (cuBLAS Linears, SDPA, fp32 LayerNorm / RMSNorm / RoPE) must compute
selas's block: it is checked here, on the CPU, against the oracle's bf16 double block, which
tests/test_oracle_golden.py pins bit for bit to selas's own."""

from __future__ import annotations

import torch

from oracle import flux_ref as R


def test_eager_double_block_equals_the_oracle():
    from selas_b200 import microbench as M
    from selas_b200.model import FluxArch, random_unit, rope_tables

    a = FluxArch(hidden=256, heads=2, mlp_hidden=1024)
    w = random_unit(a, "double", torch.Generator().manual_seed(0), "cpu")
    lt, li, d = 8, 16, a.hidden
    g = torch.Generator().manual_seed(1)
    img, txt = torch.randn(1, li, d, generator=g), torch.randn(1, lt, d, generator=g)
    mod = torch.randn(1, 12 * d, generator=g).to(torch.bfloat16)
    ids = torch.zeros(lt + li, 3)
    ids[lt:, 1] = torch.arange(li) // 4
    ids[lt:, 2] = torch.arange(li) % 4
    cos, sin = rope_tables(ids, a.axes_dim, a.theta)
    e_img, e_txt = M.yardstick_double(w, img, txt, mod, cos, sin, a.heads, M.YardstickSegments(False))
    weights = {n: w.get(n) for n in w.spec.tensors}
    r_img, r_txt = R.double_block(weights, img, txt, mod, cos, sin, a.heads, torch.bfloat16)
    assert torch.equal(e_img, r_img) and torch.equal(e_txt, r_txt)


def test_eager_single_block_equals_the_oracle():
    from selas_b200 import microbench as M
    from selas_b200.model import FluxArch, random_unit, rope_tables

    a = FluxArch(hidden=256, heads=2, mlp_hidden=1024)
    w = random_unit(a, "single", torch.Generator().manual_seed(2), "cpu")
    l, d = 24, a.hidden
    g = torch.Generator().manual_seed(4)
    x = torch.randn(2, l, d, generator=g)
    mod = torch.randn(2, 3 * d, generator=g).to(torch.bfloat16)
    ids = torch.zeros(l, 3)
    ids[:, 2] = torch.arange(l)
    cos, sin = rope_tables(ids, a.axes_dim, a.theta)
    got = M.yardstick_single(w, x, mod, cos, sin, a.heads, a.mlp_hidden, M.YardstickSegments(False))
    ref = R.single_block({n: w.get(n) for n in w.spec.tensors}, x, mod, cos, sin, a.heads, a.mlp_hidden, torch.bfloat16)
    assert torch.equal(got, ref)


def test_eager_whole_step_equals_the_oracle():
    """The yardstick step (img_in, every block, final layer) on a 1 + 1 block model, against the
    oracle's bf16 step on the same conditioning."""
    from selas_b200 import microbench as M
    from selas_b200.model import Conditioning, FluxArch, random_unit

    a = FluxArch(hidden=256, heads=2, mlp_hidden=512, depth_double=1, depth_single=1, context_dim=64, vec_dim=32)
    gen = torch.Generator().manual_seed(5)
    units = {"globals": random_unit(a, "globals", gen, "cpu")}
    for k in ("double", "single"):
        units[f"{k}.0"] = random_unit(a, k, gen, "cpu")
        units[f"{k}.0.mod"] = random_unit(a, k + "_mod", gen, "cpu")
    weights = {n: {t: u.get(t) for t in u.spec.tensors} for n, u in units.items()}
    g = torch.Generator().manual_seed(6)
    txt, pooled = torch.randn(1, 8, 64, generator=g), torch.randn(1, 32, generator=g)
    sig = R.get_schedule(4, 16)
    c = R.prepare(weights, a, sig, 3.5, pooled, txt, R.image_ids(64, 64), R.text_ids(8), torch.bfloat16)
    cond = Conditioning(c["sigmas"], c["mods"], c["final_mod"], c["txt"], c["cos"], c["sin"], c["l_txt"])
    x = torch.randn(1, 16, 64, generator=g)
    got = M.yardstick_step(units, a, 1, x, cond, M.YardstickSegments(False))
    ref = R.step(weights, a, 1, x, c, torch.bfloat16)
    assert torch.equal(got, ref)
