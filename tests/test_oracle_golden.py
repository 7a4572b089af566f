"""Pin the CPU oracle to golden vectors written by the reference itself (tests/golden/make_golden.py)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import flux_ref as R
from oracle import fp8_ref as F8
from oracle import int8_ref as I
from oracle import nf4_ref as N
from oracle import weights as OW

from .conftest import GOLDEN


@pytest.fixture(scope="module")
def nf4():
    return dict(np.load(GOLDEN / "nf4.npz"))


def test_nf4_packing_order_high_nibble_first(nf4):
    packed, absmax = N.encode(np.array([-1.0, 1.0] + [0.0] * 62, np.float32))
    assert packed[0] == 0x0F and absmax[0] == 1.0
    assert np.array_equal(packed, nf4["kat_packed"]) and np.array_equal(absmax, nf4["kat_absmax"])


@pytest.mark.parametrize("case,bs", [("s1", 64), ("b128", 128)])
def test_nf4_encode_matches_reference(nf4, case, bs):
    packed, absmax = N.encode(nf4[f"{case}_values"], bs)
    assert np.array_equal(packed, nf4[f"{case}_packed"])
    assert np.array_equal(absmax, nf4[f"{case}_absmax"])


def test_nf4_encode_custom_code_matches_reference(nf4):
    g = torch.Generator().manual_seed(6)
    w = torch.randn(32, 128, generator=g).numpy()
    packed, absmax = N.encode(w, 64, nf4["cc_code"])
    assert np.array_equal(packed, nf4["cc_packed"]) and np.array_equal(absmax, nf4["cc_absmax"])


@pytest.mark.parametrize("case,bs", [("s1", 64), ("rb", 64), ("b128", 128), ("cc", 64)])
@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
def test_nf4_decode_bit_exact_vs_reference(nf4, case, bs, dt):
    code = nf4["cc_code"] if case == "cc" else N.NF4_CODE
    name = {"f32": "float32", "f16": "float16", "bf16": "bfloat16"}[dt]
    ours = N.decode(nf4[f"{case}_packed"], nf4[f"{case}_absmax"], bs, name, code)
    ref = nf4[f"{case}_out_{dt}"]
    assert ours.view(np.uint8).tobytes() == ref.view(np.uint8).tobytes()
    # the torch restatement the GPU tests use to decode whole NF4 models for the fp32 checker
    tdt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[dt]
    t = N.decode_torch(torch.from_numpy(nf4[f"{case}_packed"]), torch.from_numpy(nf4[f"{case}_absmax"]), bs,
                       (-1,), tdt, code)
    assert t.contiguous().view(torch.uint8).numpy().tobytes() == ref.view(np.uint8).tobytes()


@pytest.fixture(scope="module")
def mini():
    return torch.load(GOLDEN / "blocks_mini.pt", weights_only=False)


def _mini_units(g):
    a = OW.Arch(**g["arch"])
    units = {"double": OW.double_unit(a, 7, 0), "single": OW.single_unit(a, 7, 0), "globals": OW.globals_unit(a, 7)}
    s = sum(float(v.double().sum()) for u in units.values() for v in u.values())
    assert s == pytest.approx(g["checksum"], rel=0, abs=1e-9), "synthetic weight stream changed"
    return a, units


@pytest.mark.parametrize("dt,tol", [(torch.float32, 2e-5), (torch.bfloat16, 0.0)])
def test_oracle_blocks_match_reference(mini, dt, tol):
    a, units = _mini_units(mini)
    tag = "f32" if dt == torch.float32 else "bf16"
    for key, case in mini["cases"].items():
        i = case["inputs"]
        with torch.no_grad():
            oi, ot = R.double_block(units["double"], i["img"], i["txt"], i["dmod"].to(dt), i["cos"], i["sin"], a.heads, dt)
            x = torch.cat((ot, oi), 1)
            xs = R.single_block(units["single"], x, i["smod"].to(dt), i["cos"], i["sin"], a.heads, a.mlp_hidden, dt)
            fo = R.final_layer(units["globals"], xs[:, i["txt"].shape[1]:], i["fmod"].to(dt), dt)
        g = case[tag]
        for name, ours in (("double_img", oi), ("double_txt", ot), ("single", xs), ("final", fo)):
            ref = g[name]
            err = ((ours - ref).norm() / ref.norm()).item()
            assert err <= tol, (key, name, err)


def test_oracle_tiny_c1_four_steps_match_reference():
    g = torch.load(GOLDEN / "tiny_c1.pt", weights_only=False)
    a = OW.Arch(**g["arch"])
    units = OW.all_units(a, 0, bf16_exact=False)
    s = sum(float(v.double().sum()) for u in units.values() for v in u.values())
    assert s == pytest.approx(g["checksum"], rel=0, abs=1e-9)
    sig = R.get_schedule(4, g["x0"].shape[1])
    assert sig == pytest.approx(g["sigmas"], abs=0)
    with torch.no_grad():
        cond = R.prepare(units, a, sig, 3.5, g["pooled"], g["txt"], g["img_ids"], g["txt_ids"], torch.float32)
        x, preds = R.denoise(units, a, g["x0"], cond, torch.float32)
    torch.testing.assert_close(torch.stack(preds), g["velocities"], rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(x, g["final"], rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("tag,dt", [("f32", torch.float32), ("bf16", torch.bfloat16)])
def test_oracle_mini_runner_matches_reference(tag, dt):
    """The oracle's prepare + 4-step denoise on the head_dim-128 mini FLUX against selas's own
    FluxRunner over a real container (fp32, and its eager bf16 path on the CPU): identical."""
    g = torch.load(GOLDEN / "mini_runner.pt", weights_only=False)
    a = OW.Arch(**g["arch"])
    units = OW.all_units(a, 3)
    s = sum(float(v.double().sum()) for u in units.values() for v in u.values())
    assert s == pytest.approx(g["checksum"], rel=0, abs=1e-9)
    assert R.get_schedule(4, g["x0"].shape[1]) == pytest.approx(g["sigmas"], abs=0)
    with torch.no_grad():
        cond = R.prepare(units, a, g["sigmas"], 3.5, g["pooled"], g["txt"], g["img_ids"], g["txt_ids"], dt)
        x, preds = R.denoise(units, a, g["x0"], cond, dt)
    ref = g[tag]  # bit for bit, in fp32 and in bf16
    for s_, (v, r) in enumerate(zip(preds, ref["velocities"])):
        assert torch.equal(v.float(), r.float()), (tag, s_)
    assert torch.equal(x.float(), ref["final"].float()), tag


def test_sampling_helpers_match_reference():
    g = torch.load(GOLDEN / "tiny_c1.pt", weights_only=False)
    assert torch.equal(R.pack(R.get_noise(0, 128, 128)), g["x0"])
    assert torch.equal(R.image_ids(128, 128), g["img_ids"])
    assert torch.equal(R.text_ids(16), g["txt_ids"])


def test_int8_row_encode_and_decode_match_reference():
    """int8_row (selas/codecs.py:87-97, :272-276): q, the row scales and the bf16 decode bit for bit
    against the reference's own output, including an all-zero row, exact half-step ties (round half to
    even) and an outlier row; the fp32 decode is fp32(q) * scale."""
    d = dict(np.load(GOLDEN / "int8.npz"))
    q, scale = I.encode(d["values"])
    assert np.array_equal(q, d["q"]) and np.array_equal(scale, d["scale"])
    assert np.array_equal(I.decode_bf16(d["q"], d["scale"]), d["out_bf16"].view(np.uint16))
    assert np.array_equal((d["q"].astype(np.float32) * d["scale"][:, None]).astype(np.float32), d["out_f32"])
    assert scale[1] == 1.0 and not q[1].any()


@pytest.mark.parametrize("e5m2", [False, True])
def test_fp8_decode_matches_torch_cast(e5m2):
    """fp8 raw weights (selas/codecs.py:270-271 casts them with x.to(dtype)): the oracle's decode of all
    256 byte codes equals torch's cast, NaN codes included (as NaN)."""
    codes = np.arange(256, dtype=np.uint8)
    dt = torch.float8_e5m2 if e5m2 else torch.float8_e4m3fn
    ref = torch.from_numpy(codes).view(dt).to(torch.float32).numpy()
    got = F8.decode(codes, e5m2)
    nan = np.isnan(ref)
    assert np.array_equal(nan, np.isnan(got))
    assert np.array_equal(got[~nan], ref[~nan])


def _vae_mini():
    from oracle import vae_ref as VR

    g = torch.load(GOLDEN / "vae_mini.pt")
    cfg = dict(g["config"])
    seed = cfg.pop("seed")
    w = VR.random_decoder_weights(seed=seed, **cfg)
    return g, cfg, w


def test_vae_oracle_matches_reference():
    """oracle/vae_ref.py (explicit softmax attention) against selas's VaeDecoder.decode (SDPA), fp32 CPU."""
    from oracle import vae_ref as VR

    g, cfg, w = _vae_mini()
    dec = VR.Decoder(w, cfg["ch_mult"], cfg["num_res_blocks"])
    out = dec.decode(g["z"])
    assert (out - g["out"]).abs().max().item() < 2e-5
    # the fp64 restatement is the same function: fp32 rounding noise apart
    out64 = VR.Decoder(w, cfg["ch_mult"], cfg["num_res_blocks"], dtype=torch.float64).decode(g["z"])
    assert (out64 - g["out"]).abs().max().item() < 1e-4
