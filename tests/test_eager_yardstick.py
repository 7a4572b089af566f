"""The eager-PyTorch double block that `python -m selas_b200.microbench --kernel block` times as the
GPU bar of selas's default path (cuBLAS Linears, SDPA, fp32 LayerNorm / RMSNorm / RoPE) must compute
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
    e_img, e_txt = M._eager_double(w, img, txt, mod, cos, sin, a.heads)
    weights = {n: w.get(n) for n in w.spec.tensors}
    r_img, r_txt = R.double_block(weights, img, txt, mod, cos, sin, a.heads, torch.bfloat16)
    assert torch.equal(e_img, r_img) and torch.equal(e_txt, r_txt)
