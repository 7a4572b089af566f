"""selas_b200.stepcache on the CPU, its kernels replaced by the oracle's restatements
(oracle/stepcache_ref.py): the host logic (policies, guards, histories, prediction coefficients) must
make the reference's decisions and predictions on the trajectories of tests/golden/stepcache.npz,
written by selas's own StepCache. The CUDA kernels are checked against the same oracle in
tests/test_gpu_stepcache.py."""

from __future__ import annotations

import sys

import numpy as np
import pytest
import torch

from oracle import stepcache_ref as O

from .conftest import GOLDEN

sys.path.insert(0, str(GOLDEN))
import make_golden as MG  # noqa: E402


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLDEN / "stepcache.npz")


def _cache(kernels, **kw):
    from selas_b200.stepcache import StepCache, StepCacheConfig

    streamed = kw.pop("streamed", ())
    sd = kw.pop("store_dtype", torch.float32)
    steps = kw.pop("steps", 10)
    return StepCache(StepCacheConfig(**kw), steps, streamed=set(streamed), store_dtype=sd, kernels=kernels)


def replay(name, kernels, device="cpu"):
    kw, streamed, sd, steps, _ = MG.STEPCACHE_SCENARIOS[name]
    sig, *traj = MG.stepcache_inputs(name)
    traj = [[t.to(device) for t in seq] for seq in traj]
    c = _cache(kernels, streamed=streamed, store_dtype=getattr(torch, sd), steps=steps, **kw)
    return MG.drive_stepcache(c, sig, *traj, streamed)


@pytest.mark.parametrize("name", sorted(MG.STEPCACHE_SCENARIOS))
def test_host_logic_matches_reference(gold, name):
    dec, dist, pt, pbi, pbt, pbs = replay(name, O)
    assert list(dec) == list(gold[f"{name}_decisions"])
    ref = gold[f"{name}_distances"]
    got = np.array(dist)
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    np.testing.assert_allclose(got[~np.isnan(got)], ref[~np.isnan(ref)], rtol=1e-5)
    for k, v in (("tail", pt), ("bi", pbi), ("bt", pbt), ("bs", pbs)):
        assert np.array_equal(torch.stack(v).numpy(), gold[f"{name}_pred_{k}"]), k  # bit-exact


def test_reference_unit_scenarios(gold):
    c = _cache(O, threshold=0.1, warmup=2, tail_full=2, max_consecutive=10, streamed={"double.3"}, policy="fbcache")
    r = torch.ones(4, 4)
    assert [c.decide(s, 1 - s / 10, r * (1 + 0.01 * s))[0] for s in range(10)] == list(gold["warmup_tail_decisions"])
    c = _cache(O, threshold=1.0, warmup=1, tail_full=0, max_consecutive=2, policy="fbcache")
    assert [c.decide(s, 0.5, torch.ones(4))[0] for s in range(7)] == list(gold["max_consecutive_decisions"])
    c = _cache(O, threshold=0.05, policy="fbcache")
    c.decide(0, 1.0, torch.ones(8))
    d, x = c.decide(1, 0.9, torch.full((8,), 2.0))
    assert (d == "full", x) == (bool(gold["large_change"][0]), gold["large_change"][1])


def test_linear_prediction_and_fused_forms():
    from selas_b200.stepcache import StepCache, StepCacheConfig

    c = StepCache(StepCacheConfig(policy="fbcache", predict="linear"), 10, kernels=O)
    c.put_tail(1.0, torch.tensor([1.0, 1.0, 1.0, 1.0]))
    c.put_tail(0.8, torch.tensor([2.0, 2.0, 2.0, 2.0]))
    assert c.tail_residual(0.6)[0].item() == pytest.approx(3.0)  # slope -5 per unit sigma
    x = torch.arange(4.0)
    assert torch.equal(c.apply_tail(x, 0.6), x + c.tail_residual(0.6))
    c2 = StepCache(StepCacheConfig(policy="fbcache", predict="reuse"), 10, kernels=O)
    c2.put_tail_from(1.0, torch.full((4,), 3.0), torch.ones(4))
    c2.put_tail(0.8, torch.full((4,), 2.0))
    assert c2.tail_residual(0.6)[0].item() == 2.0
    # decide_from == decide on the difference
    g = torch.Generator().manual_seed(0)
    a, b, ref = (torch.randn(64, generator=g) for _ in range(3))
    for cc in (c, c2):
        cc.ref_probe = ref
    d1 = c.decide_from(3, 0.5, a, b)
    d2 = c2.decide(3, 0.5, a - b)
    assert d1[1] == pytest.approx(d2[1], rel=1e-12)
    assert torch.equal(c.ref_probe, a - b) or d1[0] != "full"


def test_bf16_block_store_rounds_to_nearest_even():
    x = torch.tensor([1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -(1.0 + 2 ** -8), 0.0])
    r = O.residual_diff(x, torch.zeros(4), torch.bfloat16)
    assert torch.equal(r, x.to(torch.bfloat16))


def test_bad_config_rejected():
    from selas_b200.stepcache import StepCacheConfig

    with pytest.raises(ValueError):
        StepCacheConfig(policy="lru")
    with pytest.raises(ValueError):
        StepCacheConfig(policy="fbcache", predict="cubic")
