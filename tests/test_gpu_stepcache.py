"""The step-cache kernels (csrc/stepcache.cu) on a B200, through the C-ABI, against the oracle:

* the reference trajectories of tests/golden/stepcache.npz replayed with the CUDA kernels: the same
  decisions, distances to fp64-sum precision and bit-identical predicted residuals;
* the kernels at the size of a 1024^2 hidden state (4096 x 3072 fp32) against the oracle: residual
  and prediction bit-exact, sums to 1e-12 relative;
* FluxStepper with a cache on a mini FLUX: a threshold no step meets gives the uncached velocities bit
  for bit; a threshold every step meets follows the warmup / max_consecutive / tail_full schedule, and a
  skipped step's velocity is the final layer on the probe output plus the predicted tail residual.
"""

from __future__ import annotations

import sys

import numpy as np
import pytest
import torch

from oracle import flux_ref as R
from oracle import stepcache_ref as O
from oracle import weights as OW

from .conftest import GOLDEN, cuda_ok

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a B200")]
sys.path.insert(0, str(GOLDEN))
import make_golden as MG  # noqa: E402

DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _lib_ready():
    from selas_b200 import _lib

    _lib.lib()
    yield
    torch.cuda.synchronize()
    assert _lib.device_status() == 0


@pytest.mark.parametrize("name", sorted(MG.STEPCACHE_SCENARIOS))
def test_reference_trajectories_on_device(name):
    from selas_b200 import ops

    from .test_stepcache import replay

    gold = np.load(GOLDEN / "stepcache.npz")
    dec, dist, pt, pbi, pbt, pbs = replay(name, ops, DEV)
    assert list(dec) == list(gold[f"{name}_decisions"])
    ref, got = gold[f"{name}_distances"], np.array(dist)
    np.testing.assert_allclose(got[~np.isnan(got)], ref[~np.isnan(ref)], rtol=1e-5)
    for k, v in (("tail", pt), ("bi", pbi), ("bt", pbt), ("bs", pbs)):
        assert np.array_equal(torch.stack(v).numpy(), gold[f"{name}_pred_{k}"]), k


def test_kernels_full_size_match_oracle():
    from selas_b200 import ops

    g = torch.Generator().manual_seed(9)
    shape = (1, 4096, 3072)
    x, x_in, ref, r0 = (torch.randn(shape, generator=g) for _ in range(4))
    resid = torch.empty(shape, device=DEV)
    sums = ops.probe_distance(x.to(DEV), x_in.to(DEV), ref.to(DEV), resid)
    resid_o = torch.empty(shape)
    sums_o = O.probe_distance(x, x_in, ref, resid_o)
    assert torch.equal(resid.cpu(), resid_o)
    np.testing.assert_allclose(sums, sums_o, rtol=1e-12)
    for dt in (torch.float32, torch.bfloat16):
        r1d = ops.residual_diff(x.to(DEV), x_in.to(DEV), dt)
        r1o = O.residual_diff(x, x_in, dt)
        assert torch.equal(r1d.cpu(), r1o)
        r0d = r0.to(dt)
        for a in (0.0, -1.0 / 3.0, 0.7):
            got = ops.residual_predict(ref.to(DEV), r1d, r0d.to(DEV), a)
            assert torch.equal(got.cpu(), O.residual_predict(ref, r1o, r0d, a))
        assert torch.equal(ops.residual_predict(None, r1d, None, 0.0).cpu(), r1o.float())


def test_rejects_bad_layouts():
    from selas_b200 import _lib, ops

    x = torch.zeros(6, device=DEV)
    with pytest.raises(_lib.FluxB200Error, match="multiple of 4"):
        ops.probe_distance(x, None, x, None)
    with pytest.raises(_lib.FluxB200Error, match="fp32 or bf16"):
        ops.residual_predict(None, torch.zeros(8, device=DEV, dtype=torch.float16), None, 0.0)


def _mini():
    from selas_b200.model import FluxArch, FluxStepper, ResidentUnit

    arch = OW.Arch(hidden=256, heads=2, mlp_hidden=1024, depth_double=3, depth_single=2, in_channels=64,
                   context_dim=256, vec_dim=256, axes_dim=(16, 56, 56))
    units = {n: ResidentUnit({k: t.to(DEV, torch.float32 if k.endswith("_norm.scale") else torch.bfloat16)
                              for k, t in u.items()}) for n, u in OW.all_units(arch, 3).items()}
    gen = torch.Generator().manual_seed(0)
    txt, pooled = torch.randn(1, 16, 256, generator=gen), torch.randn(1, 256, generator=gen)
    x0 = R.pack(R.get_noise(0, 128, 128)).to(DEV)
    sig = R.get_schedule(6, x0.shape[1])
    st = FluxStepper(units, FluxArch(**arch.__dict__))
    cond = st.prepare(sig, 3.5, pooled.to(DEV), txt.to(DEV), R.image_ids(128, 128).to(DEV), R.text_ids(16).to(DEV))
    return st, cond, x0, sig


def test_stepper_with_cache():
    from selas_b200 import flux as B
    from selas_b200 import ops
    from selas_b200.stepcache import StepCache, StepCacheConfig

    st, cond, x0, sig = _mini()
    steps = len(sig) - 1
    xs, plain = [x0], []
    for s in range(steps):
        plain.append(st.step(s, xs[-1], cond))
        xs.append(xs[-1] + (sig[s + 1] - sig[s]) * plain[-1])
    # never approximated: bit-identical velocities
    never = StepCache(StepCacheConfig(policy="fbcache", threshold=0.0), steps)
    for s in range(steps):
        assert torch.equal(st.step(s, xs[s], cond, cache=never), plain[s])
    assert [d for _, d, _ in never.log] == ["full"] * steps
    # always approximated where allowed: warmup 1, max_consecutive 2, tail_full 1
    cfg = StepCacheConfig(policy="fbcache", threshold=1e9, predict="linear", warmup=1, tail_full=1, max_consecutive=2)
    always = StepCache(cfg, steps)
    for s in range(steps):
        v = st.step(s, xs[s], cond, cache=always)
        if always.log[-1][1] == "skip":  # redo the probe and the predicted tail by hand
            img = ops.linear(xs[s].to(torch.bfloat16), B.weight(st.g, "img_in.weight"), B.bias(st.g, "img_in"),
                             out_dtype=torch.float32)
            img, _ = st._double("double.0", img, cond.txt, cond, s, None)
            expect = B.final_layer(st.g, img + always.tail_residual(sig[s]), cond.final_mod[s], torch.bfloat16)
            assert torch.equal(v, expect)
        assert torch.isfinite(v).all()
    assert [d for _, d, _ in always.log] == ["full", "skip", "skip", "full", "skip", "full"]
