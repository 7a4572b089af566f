"""Write the golden vectors under tests/golden/ by running the REFERENCE (tcox-coding/selas) itself.

Run once in a container where the reference source is importable:

    python tests/golden/make_golden.py --reference <path to the selas checkout>

Nothing at test time imports the reference; the tests only read the files written here.
Outputs:

* ``nf4.npz`` — NF4 known answers: the packing-order case of ``tests/test_codecs.py:47-51``, the seed-1
  96x128 decode of ``tests/test_codecs.py:54-63``, the random-byte self-check vector of
  ``selas/codecs.py:244-253``, a blocksize-128 case and a custom code table, each decoded by
  ``selas.codecs.nf4_dequant_torch`` to fp32, fp16 and bf16.
* ``blocks_mini.pt`` — ``double_block`` / ``single_block`` / ``final_layer`` of ``selas/models/flux.py`` on a
  small FLUX architecture with head_dim 128 (hidden 256, 2 heads, MLP 1024), 16 text + 64 image tokens,
  batch 1 and 2, in fp32 and bf16 on the CPU, plus the RoPE tables.
* ``int8.npz`` — int8_row known answers: ``selas.codecs.encode_int8_row`` of seeded weight-like rows
  (plus an all-zero row, a row of exact half-step ties and a row with an outlier) and
  ``selas.codecs.decode("int8_row", ...)`` of them to bf16 and fp32.
* ``stepcache.npz`` — ``selas.stepcache.StepCache`` driven through seeded probe/tail/block residual
  trajectories (fbcache linear and reuse, tiered with bf16 block residuals, and the scenarios of
  ``tests/test_stepcache_sampling.py``): every decision, distance and predicted residual.
* ``tiny_c1.pt`` — the tiny CPU configuration (hidden 256, 4 heads x 64, MLP 1024, 2 double + 4 single
  blocks, axes (16, 24, 24)): 4 Euler steps through the reference ``FluxRunner`` over a real container.
"""

from __future__ import annotations

import argparse
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from oracle import weights as OW  # noqa: E402

MINI = OW.Arch(hidden=256, heads=2, mlp_hidden=1024, depth_double=1, depth_single=1, in_channels=64, context_dim=256,
               vec_dim=256, axes_dim=(16, 56, 56))
TINY_C1 = OW.Arch(hidden=256, heads=4, mlp_hidden=1024, depth_double=2, depth_single=4, in_channels=64, context_dim=256,
                  vec_dim=256, axes_dim=(16, 24, 24))


class DictView:
    """The two methods of selas's UnitView that the block functions call (store.py:265-293)."""

    def __init__(self, tensors: dict, dtype):
        self.t, self.dtype = tensors, dtype

    def get(self, name, dtype=None):
        return self.t[name].to(dtype or self.dtype)

    def linear(self, x, prefix, dtype=None):
        import torch.nn.functional as F
        dt = dtype or self.dtype
        b = self.t.get(prefix + ".bias")
        return F.linear(x, self.t[prefix + ".weight"].to(dt), None if b is None else b.to(dt))


def checksum(units: dict) -> float:
    return float(sum(float(v.double().sum()) for u in units.values() for v in u.values()))


def make_nf4(codecs):
    out = {}
    # packing order (tests/test_codecs.py:47-51)
    e = codecs.encode_nf4("w", torch.tensor([-1.0, 1.0] + [0.0] * 62))
    out["kat_packed"], out["kat_absmax"] = e.parts["packed"].numpy(), e.parts["absmax"].numpy()
    # seed-1 96x128 (tests/test_codecs.py:54-63)
    g = torch.Generator().manual_seed(1)
    t = torch.randn(96, 128, generator=g)
    e = codecs.encode_nf4("w", t)
    out["s1_values"], out["s1_packed"], out["s1_absmax"] = t.numpy(), e.parts["packed"].numpy(), e.parts["absmax"].numpy()
    cases = {"s1": (e.parts["packed"], e.parts["absmax"], 64, codecs.NF4_CODE)}
    # self-check vector (codecs.py:244-246)
    g = torch.Generator(device="cpu").manual_seed(0)
    packed = torch.randint(0, 256, (4096,), dtype=torch.uint8, generator=g)
    absmax = torch.rand(128, generator=g) + 0.01
    out["rb_packed"], out["rb_absmax"] = packed.numpy(), absmax.numpy()
    cases["rb"] = (packed, absmax, 64, codecs.NF4_CODE)
    # blocksize 128, weight-like values
    g = torch.Generator().manual_seed(5)
    w = torch.randn(64, 256, generator=g) * 0.02
    e = codecs.encode_nf4("w", w, blocksize=128)
    out["b128_values"], out["b128_packed"], out["b128_absmax"] = w.numpy(), e.parts["packed"].numpy(), e.parts["absmax"].numpy()
    cases["b128"] = (e.parts["packed"], e.parts["absmax"], 128, codecs.NF4_CODE)
    # a runtime code table that is not NF4_CODE (Forge/bnb files carry their own quant_map)
    code = tuple(float(c) for c in (torch.tensor(codecs.NF4_CODE) * 0.75 + 0.01))
    g = torch.Generator().manual_seed(6)
    w = torch.randn(32, 128, generator=g)
    e = codecs.encode_nf4("w", w, code=code)
    out["cc_code"], out["cc_packed"], out["cc_absmax"] = np.array(code, np.float32), e.parts["packed"].numpy(), e.parts["absmax"].numpy()
    out["cc_values"] = w.numpy()
    cases["cc"] = (e.parts["packed"], e.parts["absmax"], 64, code)
    for name, (p, a, bs, c) in cases.items():
        for dt, tag in ((torch.float32, "f32"), (torch.float16, "f16"), (torch.bfloat16, "bf16")):
            ref = codecs.nf4_dequant_torch(p, a, bs, tuple(c), (p.numel() * 2,), dt)
            out[f"{name}_out_{tag}"] = ref.view(torch.int16).numpy() if dt == torch.bfloat16 else ref.numpy()
    out["code"] = np.array(codecs.NF4_CODE, np.float32)
    np.savez_compressed(HERE / "nf4.npz", **out)


def make_int8(codecs):
    g = torch.Generator().manual_seed(11)
    w = torch.randn(64, 192, generator=g) * 0.02
    w[1] = 0.0                                             # all-zero row: scale 1, q 0
    w[2] = torch.arange(192, dtype=torch.float32) - 95.5   # absmax 96 -> scale 96/127: many near-ties
    w[2, 0] = 127.0                                        # absmax 127 -> scale 1: w - 0.5 ties round to even
    w[3, 5] = 3.0                                          # one outlier dominates the row scale
    e = codecs.encode_int8_row("w", w)
    out = {"values": w.numpy(), "q": e.parts["q"].numpy(), "scale": e.parts["scale"].numpy()}
    for dt, tag in ((torch.bfloat16, "bf16"), (torch.float32, "f32")):
        dec = codecs.decode("int8_row", e.parts, {}, tuple(w.shape), dt)
        out[f"out_{tag}"] = dec.view(torch.int16).numpy() if dt == torch.bfloat16 else dec.numpy()
    np.savez_compressed(HERE / "int8.npz", **out)


STEPCACHE_SCENARIOS = {
    # name: (config kwargs, streamed units, store dtype, steps, jump steps)
    "fb_linear": (dict(policy="fbcache", threshold=0.1, predict="linear", warmup=1, tail_full=1, max_consecutive=3),
                  (), "float32", 14, (6,)),
    "fb_reuse": (dict(policy="fbcache", threshold=0.12, predict="reuse", warmup=2, tail_full=2, max_consecutive=2),
                 (), "float32", 12, (8,)),
    "tiered": (dict(policy="tiered", threshold=0.1, predict="linear", warmup=1, tail_full=1, max_consecutive=3),
               ("double.1", "single.0"), "bfloat16", 14, (5,)),
}


def stepcache_inputs(name: str):
    """The seeded residual trajectories of one scenario (also rebuilt by the tests from this function)."""
    _, _, _, steps, jumps = STEPCACHE_SCENARIOS[name]
    g = torch.Generator().manual_seed(sum(map(ord, name)))
    shape = (2, 40, 48)
    base = torch.randn(shape, generator=g)
    probes, tails, bis, bts, bss = [], [], [], [], []
    for s in range(steps):
        drift = 0.02 * s + (0.5 if s in jumps else 0.0)
        probes.append(base * (1 + drift) + 0.03 * torch.randn(shape, generator=g))
        tails.append(torch.randn(shape, generator=g) * (1 + 0.1 * s))
        bis.append(torch.randn(shape, generator=g) * 0.5)
        bts.append(torch.randn(2, 8, 48, generator=g) * 0.5)
        bss.append(torch.randn(2, 48, 48, generator=g) * 0.5)
    sig = [1.0 - s / steps for s in range(steps)]
    return sig, probes, tails, bis, bts, bss


def drive_stepcache(cache, sig, probes, tails, bis, bts, bss, streamed):
    """The runner's use of the cache (selas/models/flux.py:547-580) on given residuals: per step the
    decision and distance, and every predicted residual the step consumes (zeros where none)."""
    dec, dist, pt, pbi, pbt, pbs = [], [], [], [], [], []
    for s, sigma in enumerate(sig):
        d, x = cache.decide(s, sigma, probes[s])
        dec.append(d)
        dist.append(float("nan") if x is None else x)
        z = torch.zeros_like
        t = bi = bt = bs = None
        if d == "skip":
            t = cache.tail_residual(sigma)
        else:
            if d == "hybrid" and cache.substitutes("double.1"):
                bi, bt = cache.block_residual("double.1", sigma)
            if d == "hybrid" and cache.substitutes("single.0"):
                bs = cache.block_residual("single.0", sigma)[0]
            if d == "full":
                if cache.records("double.1"):
                    cache.put_block("double.1", sigma, (bis[s], bts[s]))
                if cache.records("single.0"):
                    cache.put_block("single.0", sigma, (bss[s],))
                cache.put_tail(sigma, tails[s])
        pt.append((t if t is not None else z(tails[s])).float().cpu())
        pbi.append((bi if bi is not None else z(bis[s])).float().cpu())
        pbt.append((bt if bt is not None else z(bts[s])).float().cpu())
        pbs.append((bs if bs is not None else z(bss[s])).float().cpu())
    return dec, dist, pt, pbi, pbt, pbs


def make_stepcache(stepcache):
    out = {}
    for name, (kw, streamed, sd, steps, _) in STEPCACHE_SCENARIOS.items():
        sig, probes, tails, bis, bts, bss = stepcache_inputs(name)
        cache = stepcache.StepCache(stepcache.StepCacheConfig(**kw), num_steps=steps, streamed=set(streamed),
                                    store_dtype=getattr(torch, sd))
        dec, dist, pt, pbi, pbt, pbs = drive_stepcache(cache, sig, probes, tails, bis, bts, bss, streamed)
        out[f"{name}_decisions"] = np.array(dec)
        out[f"{name}_distances"] = np.array(dist, np.float64)
        for k, v in (("tail", pt), ("bi", pbi), ("bt", pbt), ("bs", pbs)):
            out[f"{name}_pred_{k}"] = torch.stack(v).numpy()
    # the scenarios of tests/test_stepcache_sampling.py
    S = stepcache
    c = S.StepCache(S.StepCacheConfig(policy="fbcache", threshold=0.1, warmup=2, tail_full=2, max_consecutive=10), 10,
                    streamed={"double.3"}, store_dtype=torch.float32)
    r = torch.ones(4, 4)
    out["warmup_tail_decisions"] = np.array([c.decide(s, 1 - s / 10, r * (1 + 0.01 * s))[0] for s in range(10)])
    c = S.StepCache(S.StepCacheConfig(policy="fbcache", threshold=1.0, warmup=1, tail_full=0, max_consecutive=2), 10,
                    streamed={"double.3"}, store_dtype=torch.float32)
    out["max_consecutive_decisions"] = np.array([c.decide(s, 0.5, torch.ones(4))[0] for s in range(7)])
    c = S.StepCache(S.StepCacheConfig(policy="fbcache", threshold=0.05), 10, streamed={"double.3"},
                    store_dtype=torch.float32)
    c.decide(0, 1.0, torch.ones(8))
    d, x = c.decide(1, 0.9, torch.full((8,), 2.0))
    out["large_change"] = np.array([d == "full", x], dtype=np.float64)
    np.savez_compressed(HERE / "stepcache.npz", **out)


def make_blocks(flux):
    a = MINI
    units = {"double": OW.double_unit(a, 7, 0), "single": OW.single_unit(a, 7, 0), "globals": OW.globals_unit(a, 7)}
    res = {"arch": a.__dict__, "checksum": checksum(units), "cases": {}}
    for batch, l_img, l_txt in ((1, 64, 16), (2, 64, 16)):
        img, txt, dmod, smod, fmod = OW.block_inputs(a, 11, l_img, l_txt, batch)
        from selas.sampling import image_ids, text_ids
        side = int(round((l_img ** 0.5))) * 16
        ids = torch.cat((text_ids(l_txt), image_ids(side, side)), 0)
        cos, sin = flux.rope_tables(ids, a.axes_dim, a.theta)
        cfg = flux.FluxConfig(hidden=a.hidden, heads=a.heads, mlp_hidden=a.mlp_hidden, axes_dim=a.axes_dim)
        case = {"inputs": {"img": img, "txt": txt, "dmod": dmod, "smod": smod, "fmod": fmod, "cos": cos, "sin": sin}}
        for dt, tag in ((torch.float32, "f32"), (torch.bfloat16, "bf16")):
            with torch.no_grad():
                dv = DictView(units["double"], dt)
                oi, ot = flux.double_block(dv, img, txt, dmod.to(dt), cos, sin, cfg, dt, False)
                x = torch.cat((ot, oi), 1)
                xs = flux.single_block(DictView(units["single"], dt), x, smod.to(dt), cos, sin, cfg, dt, False)
                fo = flux.final_layer(DictView(units["globals"], dt), xs[:, l_txt:], fmod.to(dt), dt)
            case[tag] = {"double_img": oi, "double_txt": ot, "single": xs, "final": fo}
        res["cases"][f"b{batch}_li{l_img}_lt{l_txt}"] = case
    torch.save(res, HERE / "blocks_mini.pt")


def make_tiny_c1(ref_root: Path):
    from safetensors.torch import save_file
    from selas.container import Container
    from selas.convert import ConvertOptions, convert_flux, flux_view
    from selas.models.flux import FluxRunner
    from selas.sampling import get_noise, get_schedule, image_ids, pack, text_ids
    from selas.sources import TensorSource
    from selas.store import WeightStore

    a = TINY_C1
    units = OW.all_units(a, 0, bf16_exact=False)
    sd = {}
    for unit, tensors in units.items():
        if unit == "globals":
            prefix = ""
        else:
            kind, idx = unit.split(".")[:2]
            prefix = f"{kind}_blocks.{idx}."
        for k, v in tensors.items():
            sd[prefix + k] = v.contiguous()
    g = torch.Generator().manual_seed(0)
    txt = torch.randn(1, 16, a.context_dim, generator=g)
    pooled = torch.randn(1, a.vec_dim, generator=g)
    x0 = pack(get_noise(0, 128, 128))
    img_ids, txt_ids = image_ids(128, 128), text_ids(16)
    sigmas = get_schedule(4, x0.shape[1])
    with tempfile.TemporaryDirectory() as tmp:
        tmp = Path(tmp)
        save_file(sd, str(tmp / "m.safetensors"))
        convert_flux(flux_view(TensorSource([tmp / "m.safetensors"])), tmp / "c",
                     ConvertOptions(dtype=torch.float32, quant_report=False), axes_dim=a.axes_dim)
        c = Container(tmp / "c")
        from selas.models.flux import FluxConfig
        cfg = FluxConfig.from_dict(c.config)
        with WeightStore(c, {}, torch.device("cpu"), torch.float32) as st:
            runner = FluxRunner(st, cfg, torch.float32)
            cond = runner.prepare(sigmas, 3.5, pooled, txt, img_ids, txt_ids)
            x, preds = x0, []
            for s in range(4):
                v, _ = runner.step(s, x, cond)
                preds.append(v)
                x = x + (sigmas[s + 1] - sigmas[s]) * v
            runner.end()
    torch.save({"arch": a.__dict__, "checksum": checksum(units), "txt": txt, "pooled": pooled, "x0": x0,
                "img_ids": img_ids, "txt_ids": txt_ids, "sigmas": sigmas, "velocities": torch.stack(preds),
                "final": x}, HERE / "tiny_c1.pt")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    ap.add_argument("--only", choices=("nf4", "int8", "blocks", "c1", "stepcache"), help="write one file only")
    args = ap.parse_args()
    sys.path.insert(0, str(args.reference))
    torch.set_num_threads(8)
    import selas.codecs as codecs
    import selas.models.flux as flux
    if args.only in (None, "nf4"):
        make_nf4(codecs)
    if args.only in (None, "int8"):
        make_int8(codecs)
    if args.only in (None, "stepcache"):
        import selas.stepcache as stepcache
        make_stepcache(stepcache)
    if args.only in (None, "blocks"):
        make_blocks(flux)
    if args.only in (None, "c1"):
        make_tiny_c1(args.reference)
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
