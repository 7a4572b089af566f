"""Benchmark: FLUX-12B 1024^2 denoise steps/s on B200 (BASELINE.json `metric`, config C4).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--res 1024]

One process per GPU (torchrun for N > 1). Each rank holds a full random-init 12B FLUX replica in
HBM (19 double + 38 single blocks, bf16, weights N(0, 0.02)) and denoises its own seeded 1024^2
latent (4096 image + 512 text tokens): images are sharded one per GPU, with no collective on the
data path (the only collectives are the barrier around the timed region and the max-reduction of
the timings). A step is one full transformer forward (img_in, 19 double, 38 single blocks, final
layer) plus the Euler update; modulations are precomputed by the prologue before timing.

Printed JSON (rank 0): `value` = steps/s summed over all GPUs (device-timed, inputs resident), `e2e`
= the same through the public API with the step's latents copied from pinned host memory and the
updated latents copied back every step, `roofline` for the dominant kernel (the tcgen05 GEMM) and
`cpu_baseline` = the oracle (selas's eager block math restated on the CPU, fp32) timed on this
host's cores on a bounded sample (one double + one single block) and scaled to a step.

`--impl reference` times the reference path on the CPU the same way (the reference is pure
Python/PyTorch and cannot run on this box without its source; its arithmetic is the oracle's).
"""

from __future__ import annotations

import argparse
import atexit
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

STEPS_PER_IMAGE = 28
METRIC = "FLUX-12B 1024^2 denoise steps/sec (per GPU, images/sec at 1/2/4/8 B200); % roofline"
# Benchmark configurations (BASELINE.json `configs`): C4 is the headline (default); C5 runs the same
# 12B architecture with every block Linear in NF4 at 512^2, four images per GPU.
CONFIGS = {
    "c4": {"name": "C4: FLUX-12B (19 double + 38 single), bf16 weights", "res": 1024, "per_gpu": 1, "quant": "none"},
    "c5": {"name": "C5: FLUX-12B (19 double + 38 single), all block Linears NF4 (blocksize 64)", "res": 512,
           "per_gpu": 4, "quant": "nf4"},
    # C5's single-image latency case: one 1024^2 image per job, its tokens split over the ranks (Ulysses
    # sequence parallelism, two NCCL all-to-alls around each attention); strong scaling
    "c5u": {"name": "C5 single-image latency: FLUX-12B, all block Linears NF4, Ulysses sequence parallel over "
                    "the ranks", "res": 1024, "per_gpu": 1, "quant": "nf4", "sp": True},
}
UNIT = "steps/s"


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm": d["hbm_gbs"], "bf16": d["bf16_tflops"], "bf16_sustained": d["bf16_tflops_sustained"],
                "source": "measured"}
    return {"hbm": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


# ------------------------------------------------------------------------------------------ clocks


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms. Started before the warm-up (nvidia-smi
    takes a few hundred ms to print its first line); ``begin()`` marks the start of a timed region and
    ``stop()`` summarises the samples taken since (or, if the region was too short to catch one, those
    since the start, and says so). The sampler keeps running until ``close()``, so that every timed
    region (the device-timed steps and the end-to-end ones) runs with the same polling beside it."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[tuple[float, str]] = []
        self.t_begin = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.index), "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
            atexit.register(self.close)  # no polling process outlives the bench, on any exit path
        except (OSError, ValueError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.monotonic(), line.strip()))

    def begin(self):
        self.t_begin = time.monotonic()

    def close(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        t_end = time.monotonic()
        time.sleep(0.25)  # the sample that covers the region's last 200 ms is printed after it ends
        window = "timed region"
        lines = [ln for t, ln in list(self.lines) if self.t_begin is not None and self.t_begin <= t <= t_end + 0.2]
        if not lines:
            window, lines = "warm-up + timed region (the timed region alone was shorter than one sample)", \
                [ln for _, ln in list(self.lines)]
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm), "window": window}


# ------------------------------------------------------------------------------------------ CPU legs


_CPU_SAMPLE: dict = {}
EXTRAPOLATED = ("2 of 57 blocks timed per step (one double, one single), scaled by 19 + 38; img_in, the final "
                "layer and the Euler update are not timed (under 0.1 % of a step's FLOPs)")


def cpu_block_sample(threads: int | None = None) -> dict:
    """Time the oracle (fp32, CPU) on one full-size double block and one single block of the C4
    workload (512 text + 4096 image tokens, D=3072) and scale to one 57-block step."""
    from oracle import flux_ref as R
    from oracle import weights as OW

    if threads:
        torch.set_num_threads(threads)
    a = OW.Arch()
    if not _CPU_SAMPLE:  # weights and inputs are generated once, outside the timed calls
        _CPU_SAMPLE["units"] = (OW.double_unit(a, 0, 0, bf16_exact=False), OW.single_unit(a, 0, 0, bf16_exact=False))
        _CPU_SAMPLE["inputs"] = OW.block_inputs(a, 0, 4096, 512, 1)
        _CPU_SAMPLE["rope"] = R.rope_tables(torch.cat((R.text_ids(512), R.image_ids(1024, 1024)), 0), a.axes_dim)
    du, su = _CPU_SAMPLE["units"]
    img, txt, dmod, smod, _ = _CPU_SAMPLE["inputs"]
    cos, sin = _CPU_SAMPLE["rope"]
    with torch.no_grad():
        t0 = time.perf_counter()
        R.double_block(du, img, txt, dmod, cos, sin, a.heads, torch.float32)
        t1 = time.perf_counter()
        R.single_block(su, torch.cat((txt, img), 1), smod, cos, sin, a.heads, a.mlp_hidden, torch.float32)
        t2 = time.perf_counter()
    t_d, t_s = t1 - t0, t2 - t1
    step_s = a.depth_double * t_d + a.depth_single * t_s
    return {"double_s": t_d, "single_s": t_s, "step_s": step_s, "cores": torch.get_num_threads()}


def cpu_full_step(threads: int | None = None) -> dict:
    """One whole C4 step of the oracle (fp32, CPU): img_in, 19 double blocks, the txt||img join, 38 single
    blocks and the final layer, each block's output feeding the next. The same double / single unit
    stands in for every block (a block's time does not depend on its weights' values); weights and
    inputs are generated before the timed region."""
    from oracle import flux_ref as R
    from oracle import weights as OW

    if threads:
        torch.set_num_threads(threads)
    a = OW.Arch()
    cpu_block_sample(threads)  # builds the shared units and inputs
    du, su = _CPU_SAMPLE["units"]
    img, txt, dmod, smod, fmod = _CPU_SAMPLE["inputs"]
    cos, sin = _CPU_SAMPLE["rope"]
    g = OW.globals_unit(a, 0)
    lat = torch.randn(1, 4096, 64, generator=torch.Generator().manual_seed(0))
    with torch.no_grad():
        t0 = time.perf_counter()
        x_img = R.linear(g, lat, "img_in", torch.float32).float()
        x_txt = txt
        for _ in range(a.depth_double):
            x_img, x_txt = R.double_block(du, x_img, x_txt, dmod, cos, sin, a.heads, torch.float32)
        x = torch.cat((x_txt, x_img), 1)
        for _ in range(a.depth_single):
            x = R.single_block(su, x, smod, cos, sin, a.heads, a.mlp_hidden, torch.float32)
        v = R.final_layer(g, x[:, 512:], fmod[:, :2 * a.hidden], torch.float32)
        lat = lat + (-1.0 / 28) * v
        t1 = time.perf_counter()
    return {"step_s": t1 - t0, "cores": torch.get_num_threads()}


def run_reference(args, rank: int, world: int) -> None:
    """The reference arm: selas's eager block math (the oracle restatement) on the host CPU."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    if args.full_step:  # one whole step, timed once: the check of the per-block extrapolation
        c = cpu_full_step(threads)
        value = 1.0 / c["step_s"]
        print(json.dumps({"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
                          "steps": 1, "warmup": 0, "ms_per_step": c["step_s"] * 1e3, "higher_is_better": True,
                          "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                          "config": {"workload": "C4: FLUX-12B 1024^2, one whole step on the CPU (oracle, fp32)",
                                     "global_batch": 1, "seq_len": 4608},
                          "cpu_baseline": {"value": value, "unit": UNIT, "cores": c["cores"], "kind": "port",
                                           "sample": "one whole transformer step (57 blocks + img_in + final layer + "
                                                     "Euler update), timed once"},
                          "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
              flush=True)
        return
    for _ in range(args.warmup):
        cpu_block_sample()
    samples = [cpu_block_sample() for _ in range(args.steps)]
    step_s = statistics.median(s["step_s"] for s in samples)
    sample_s = statistics.median(s["double_s"] + s["single_s"] for s in samples)
    value = 1.0 / step_s
    sample = ("each timed step is a sample: one full-size double block + one single block (4608 tokens, "
              "D=3072, fp32), scaled by 19 + 38 blocks to one transformer step")
    cpu = {"value": value, "unit": UNIT, "cores": samples[0]["cores"], "kind": "port", "sample": sample,
           "extrapolated": EXTRAPOLATED}
    print(json.dumps({"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
                      "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_s * 1e3,
                      "extrapolated": EXTRAPOLATED, "sample_ms": sample_s * 1e3,
                      "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                      "data": "synthetic", "config": {"workload": "C4: FLUX-12B 1024^2, batch 1 per rank (CPU sample)",
                                                      "global_batch": 1, "seq_len": 4608},
                      "cpu_baseline": cpu, "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                                                   "d2h_bytes_per_step": 0}}), flush=True)


# ------------------------------------------------------------------------------------------ GPU arm


def run_b200(args, rank: int, world: int, dist) -> None:
    from selas_b200 import _lib, ops
    from selas_b200.model import FluxArch, FluxStepper, random_model
    from selas_b200 import profile as prof

    from selas_b200.dist import max_over_ranks, per_rank, shard

    dev = torch.device("cuda", torch.cuda.current_device())
    arch = FluxArch()
    cfg = CONFIGS[args.config]
    res = args.res or cfg["res"]
    side = res // 16
    l_img, l_txt = side * side, 512
    sp_mode = bool(cfg.get("sp"))
    # this rank's images of the global batch (sequence parallel: the one image, shared by all ranks)
    images = [0] if sp_mode else list(shard(cfg["per_gpu"] * world, rank, world))
    nb = len(images)
    _lib.lib()

    units = random_model(arch, dev, seed=0, std=0.02, quant=cfg["quant"])
    txts, pooleds, lats = [], [], []
    for i in images:
        gen = torch.Generator().manual_seed(1000 + i)
        txts.append(torch.randn(1, l_txt, arch.context_dim, generator=gen))
        pooleds.append(torch.randn(1, arch.vec_dim, generator=gen))
        noise = torch.randn(1, 16, 2 * side, 2 * side, generator=torch.Generator().manual_seed(i))
        lats.append(noise.view(1, 16, side, 2, side, 2).permute(0, 2, 4, 1, 3, 5).reshape(1, l_img, 64))
    txt, pooled, lat = torch.cat(txts), torch.cat(pooleds), torch.cat(lats)
    ids = torch.zeros(side, side, 3)
    ids[..., 1] = torch.arange(side)[:, None]
    ids[..., 2] = torch.arange(side)[None, :]
    img_ids, txt_ids = ids.reshape(-1, 3), torch.zeros(l_txt, 3)
    mu = (1.15 - 0.5) / (4096 - 256) * l_img + (0.5 - (1.15 - 0.5) / (4096 - 256) * 256)
    sig = [1.0 - i / STEPS_PER_IMAGE for i in range(STEPS_PER_IMAGE + 1)]
    sig = [0.0 if t <= 0 else 1.0 if t >= 1 else math.exp(mu) / (math.exp(mu) + (1 / t - 1)) for t in sig]

    stepper = FluxStepper(units, arch)
    # the prologue (selas/models/flux.py:411-465): vec embedding, all 28 steps' modulation vectors of
    # every block ([28, 3072] x [3072, 18432] per double block, [28, 3072] x [3072, 9216] per single block
    # and image), txt_in, RoPE tables; timed once warm, on the device
    pro_args = (sig, 3.5, pooled.to(dev), txt.to(dev), img_ids.to(dev), txt_ids.to(dev))
    stepper.prepare(*pro_args)
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record()
    cond = stepper.prepare(*pro_args)
    p1.record()
    torch.cuda.synchronize()
    prologue_ms = p0.elapsed_time(p1)
    sp = None
    if sp_mode and world > 1:
        from selas_b200.sp import Ulysses, UlyssesP2P

        sp = Ulysses()
        lat = lat[:, sp.span(l_img)].contiguous()  # this rank's img tokens
        cond = sp.localize(cond, l_img)
        if args.sp_exchange == "p2p":  # the epilogues' and attention's own stores over NVLink
            sp = UlyssesP2P(arch, cond.l_txt + lat.shape[1])
    for n in [n for n in units if n.endswith(".mod")]:
        del units[n]  # modulations are precomputed; the mod units are not part of the step
    torch.cuda.empty_cache()
    weight_bytes = sum(u.nbytes() for u in units.values())

    x = lat.to(dev)
    stream = torch.cuda.current_stream()

    def one_step(s: int, x):
        v = stepper.step(s % STEPS_PER_IMAGE, x, cond, sp)
        return x + (sig[s % STEPS_PER_IMAGE + 1] - sig[s % STEPS_PER_IMAGE]) * v

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    sampler = ClockSampler(dev.index if "CUDA_VISIBLE_DEVICES" not in os.environ else
                           int(os.environ["CUDA_VISIBLE_DEVICES"].split(",")[dev.index]))
    sampler.start()
    for s in range(args.warmup):
        x = one_step(s, x)
    barrier()

    # ---- device-timed region (inputs resident in HBM); nothing but the steps on the stream
    sampler.begin()
    ops.launch_count_reset()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for s in range(args.steps):
        x = one_step(s, x)
    e1.record(stream)
    barrier()
    launches = ops.launch_count()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1) / args.steps

    # ---- the per-kernel split (CUDA events around each of the library's launches): a second pass of
    # the same steps, kept out of the timed region above because its events sit between the kernels
    prof.enable()
    for s in range(args.steps):
        x = one_step(s, x)
    barrier()
    kstats = prof.collect()
    prof.disable()
    ms_max = max_over_ranks(ms, dev)
    # image denoise steps per second over the whole job (sequence parallel: the one image's steps/s)
    value = (1 if sp_mode else world * nb) * 1000.0 / ms_max

    # ---- end to end through the public API with host buffers (pinned) each step
    host_in = lat.clone().pin_memory()
    host_out = torch.empty(nb, lat.shape[1], 64).pin_memory()
    barrier()
    sampler.begin()  # the same nvidia-smi polling runs beside this region as beside the one above
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for s in range(args.steps):
        xd = host_in.to(dev, non_blocking=True)
        host_out.copy_(one_step(s, xd), non_blocking=True)  # the step and its Euler update, as timed above
    f1.record(stream)
    barrier()
    e2e_clocks = sampler.stop()
    sampler.close()
    e2e_ms = max_over_ranks(f0.elapsed_time(f1) / args.steps, dev)
    # which rank set the pace, and at what clock (same collectives, same order, on every rank)
    ranks_ms, ranks_mhz = per_rank(ms, dev), per_rank(clocks.get("sm_mhz"), dev)
    assert torch.isfinite(host_out).all(), "non-finite latents"
    _lib.raise_on_device_error()
    if sp is not None and hasattr(sp, "close"):
        sp.close()

    if rank != 0:
        return
    pk = peaks()
    gemm = kstats.get("gemm", {"flops": 0, "ms": 0, "launches": 0})
    attn = kstats.get("attention", {"flops": 0, "ms": 0, "launches": 0})
    g_tf = gemm["flops"] / (gemm["ms"] * 1e-3) / 1e12 if gemm["ms"] else 0.0
    a_tf = attn["flops"] / (attn["ms"] * 1e-3) / 1e12 if attn["ms"] else 0.0
    step_flops = sum(v["flops"] for v in kstats.values()) / args.steps
    # DRAM bytes per launch of the dominant GEMM of this configuration, from an ncu capture (per config)
    traffic = None
    tfile = ROOT / "profiles" / "traffic.json"
    if tfile.exists():
        traffic = json.loads(tfile.read_text()).get(args.config, {}).get("gemm_bytes_per_launch")
    cpu = None
    if world == 1 and not args.no_cpu_baseline and args.config == "c4":
        c = cpu_block_sample(os.cpu_count())
        cpu = {"value": 1.0 / c["step_s"], "unit": UNIT, "cores": c["cores"], "kind": "port",
               "sample": f"oracle fp32: one double block ({c['double_s']:.2f} s) + one single block "
                         f"({c['single_s']:.2f} s) at 4608 tokens, scaled to 19 + 38 blocks",
               "extrapolated": EXTRAPOLATED}
    jobs = 1 if sp_mode else world * nb  # images in flight over the whole job
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_max, "higher_is_better": True, "scaling": "strong" if sp_mode else "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init N(0,0.02) weights, seeded N(0,1) latents/text)",
        "config": {"workload": (f"{cfg['name']}, {res}^2, {l_img}+{l_txt} tokens, one image over {world} GPU(s)"
                                if sp_mode else f"{cfg['name']}, {res}^2, {l_img}+{l_txt} tokens, {nb} image(s) per GPU"),
                   "global_batch": jobs, "seq_len": l_img + l_txt,
                   "parallelism": (f"ulysses sp{world} ({args.sp_exchange})" if sp_mode and world > 1 else
                                   "single GPU" if sp_mode else f"images sharded dp{world}"),
                   "weights": cfg["quant"] if cfg["quant"] != "none" else "bf16",
                   "l2": "block weights (7-17 GB) streamed every step, far above the 126 MB L2"},
        "value_definition": ("denoise steps per second of the one image, all GPUs working on it (1 step = 1 "
                             "transformer pass + Euler update); ms_per_step is the single-image step latency"
                             if sp_mode else "image denoise steps per second, summed over all GPUs (1 step = 1 "
                             "transformer pass of 1 image + Euler update)"),
        "images_per_s": value / STEPS_PER_IMAGE,
        "e2e": {"value": jobs * 1000.0 / e2e_ms, "unit": UNIT, "h2d_bytes_per_step": host_in.numel() * 4,
                "d2h_bytes_per_step": host_out.numel() * 4},
        "roofline": {"bound": "tensor", "achieved": g_tf, "peak": pk["bf16_sustained"], "unit": "TFLOP/s",
                     "frac": g_tf / pk["bf16_sustained"], "traffic": traffic,
                     "kernel": "tcgen05 GEMM (all block Linears)", "peak_source": f"{pk['source']} bf16 sustained"},
        "kernels": {k: {"ms_per_step": v["ms"] / args.steps, "launches_per_step": v["launches"] / args.steps,
                        "tflops": (v["flops"] / (v["ms"] * 1e-3) / 1e12) if v["ms"] and v["flops"] else None,
                        "gbs": (v["bytes"] / (v["ms"] * 1e-3) / 1e9) if v["ms"] and v["bytes"] else None}
                    for k, v in kstats.items()},
        "attention_tflops": a_tf,
        "step_tflop": step_flops / 1e12,
        "step_frac_of_peak": step_flops / (ms_max * 1e-3) / 1e12 / pk["bf16_sustained"],
        "weights_gb": weight_bytes / 1e9,
        "prologue_ms": prologue_ms,
        "gpu_launches": launches,
        "clocks": clocks,
        "e2e_clocks": {k: e2e_clocks.get(k) for k in ("sm_mhz", "reasons", "samples")},
        "cpu_baseline": cpu,
    }
    if world > 1:
        line["per_rank"] = {"ms_per_step": ranks_ms, "sm_mhz_median": ranks_mhz,
                            "slowest_rank": max(range(world), key=lambda r: ranks_ms[r])}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="c4", choices=sorted(CONFIGS))
    ap.add_argument("--res", type=int, default=None, help="override the configuration's resolution")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--full-step", action="store_true",
                    help="--impl reference: time one whole CPU step once instead of extrapolating from two blocks")
    ap.add_argument("--sp-exchange", default="p2p", choices=["p2p", "nccl"],
                    help="sequence-parallel configs: exchange through peer memory, or NCCL all-to-alls")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as td

        td.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
        dist = td
    try:
        run_b200(args, rank, world, dist)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
