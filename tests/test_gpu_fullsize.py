"""The north_star tolerance at the configurations the benchmark measures, on a B200.

The checker is the oracle's block math (``oracle/flux_ref.py``, a restatement of selas's eager path)
run on the GPU through torch: in fp32 (TF32 off, SDPA's math backend) it is the reference, and in
bf16 (cuBLAS + SDPA, as selas's default ``Kernels()`` runs on a GPU) it is the reference's own bf16
eager path, whose distance from fp32 sets the bar. The method is the reference's
(``experiments/kernel_error.py:25-56``): record the bf16 eager trajectory, then from its latents at
several steps run one step with every variant and compare velocities with fp32's.

  C4 (FLUX-12B, bf16 weights, 1024^2, 28 steps, guidance 3.5): at step indices 0, 7, 14, 21, 27
     rel-L2(B200, fp32) <= 1.5 x rel-L2(reference bf16, fp32) and
     max-abs(B200 - fp32) <= 2 x max-abs(reference bf16 - fp32) of the velocity;
     after 28 steps from the same noise, PSNR(B200 final latent, fp32's) >= PSNR(reference bf16's) - 3 dB.
  C5 (the same architecture with every block Linear NF4, 512^2, 4 images in one batch): the same
     per-step velocity check; the fp32 reference decodes the NF4 weights to fp32 (selas's fp32 engine),
     the bf16 ones to bf16 (selas's bf16 engine), as this library does inside its GEMM.

Weights are random-init N(0, 0.02) (norm scales N(1, 0.1)), generated on the device; inputs are
seeded N(0, 1). With FB_REPORT_DIR set, the measured spreads and margins are written there as JSON.
"""

from __future__ import annotations

import contextlib
import json
import math
import os
from collections.abc import Mapping
from pathlib import Path

import pytest
import torch

from oracle import flux_ref as R
from oracle import nf4_ref as N

from .conftest import cuda_ok

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a B200")]

BF16, F32 = torch.bfloat16, torch.float32
DEV = "cuda"
REL_FACTOR, MAX_FACTOR, PSNR_MARGIN_DB = 1.5, 2.0, 3.0
STEPS, STEP_AT, GUIDANCE = 28, (0, 7, 14, 21, 27), 3.5


@pytest.fixture(autouse=True)
def _lib_ready():
    from selas_b200 import _lib

    _lib.lib()
    yield
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    torch.cuda.empty_cache()


class OracleView(Mapping):
    """A unit of this library's resident model as the oracle's weight mapping: raw tensors as stored,
    NF4 weights decoded (``oracle.nf4_ref.decode_torch``) on access to ``wdtype``."""

    def __init__(self, unit, wdtype):
        self.unit, self.wdtype = unit, wdtype

    def __getitem__(self, name):
        u = self.unit
        if name in u._nf4:
            e = u._nf4[name]
            return N.decode_torch(e["packed"], e["absmax"], e["blocksize"], e["shape"], self.wdtype, e["code"])
        return u._raw[name]

    def __iter__(self):
        return iter(list(self.unit._raw) + list(self.unit._nf4))

    def __len__(self):
        return len(self.unit._raw) + len(self.unit._nf4)


def oracle_units(units, wdtype):
    return {n: OracleView(u, wdtype) for n, u in units.items()}


@contextlib.contextmanager
def fp32_exact():
    """True fp32 for the reference: no TF32 in matmuls or convolutions, SDPA's math backend."""
    from torch.nn.attention import SDPBackend, sdpa_kernel

    prev = torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = torch.backends.cudnn.allow_tf32 = False
    try:
        with sdpa_kernel([SDPBackend.MATH]):
            yield
    finally:
        torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = prev


def rel_l2(a, b):
    a, b = a.double(), b.double()
    return ((a - b).norm() / b.norm()).item()


def max_abs(a, b):
    return (a.double() - b.double()).abs().max().item()


def psnr(a, b):
    mse = (a.double() - b.double()).pow(2).mean().item()
    peak = b.double().abs().max().item()
    return 10 * math.log10(peak * peak / max(mse, 1e-30))


def _inputs(arch, res: int, n_images: int):
    """Seeded inputs of the benchmark: per image i, noise get_noise(i), text [512, 4096] and pooled
    [768] N(0, 1) from generator 1000 + i; ids and the shifted 28-step schedule (sampling.py)."""
    txts, pooleds, lats = [], [], []
    for i in range(n_images):
        gen = torch.Generator().manual_seed(1000 + i)
        txts.append(torch.randn(1, 512, arch.context_dim, generator=gen))
        pooleds.append(torch.randn(1, arch.vec_dim, generator=gen))
        lats.append(R.pack(R.get_noise(i, res, res)))
    img_ids, txt_ids = R.image_ids(res, res), R.text_ids(512)
    sig = R.get_schedule(STEPS, img_ids.shape[0])
    d = lambda t: t.to(DEV)  # noqa: E731
    return sig, d(torch.cat(pooleds)), d(torch.cat(txts)), d(img_ids), d(txt_ids), d(torch.cat(lats))


def _report(name: str, data: dict) -> None:
    out = os.environ.get("FB_REPORT_DIR")
    if out:
        Path(out).mkdir(parents=True, exist_ok=True)
        (Path(out) / f"tolerance_{name}.json").write_text(json.dumps(data, indent=1))


def _per_step(units, arch, sig, pooled, txt, img_ids, txt_ids, x0, final: bool):
    """The reference bf16 trajectory, then per recorded step the three velocities from its latents
    (and, with ``final``, the final latents of 28 steps of each path from x0)."""
    from selas_b200.model import FluxStepper

    o16, o32 = oracle_units(units, BF16), oracle_units(units, F32)
    with torch.no_grad():
        c16 = R.prepare(o16, arch, sig, GUIDANCE, pooled, txt, img_ids, txt_ids, BF16)
        x, traj = x0, {}
        for s in range(STEPS):
            if s in STEP_AT:
                traj[s] = x.clone()
            x = x + (sig[s + 1] - sig[s]) * R.step(o16, arch, s, x, c16, BF16)
        final16 = x
        with fp32_exact():
            c32 = R.prepare(o32, arch, sig, GUIDANCE, pooled, txt, img_ids, txt_ids, F32)
    st = FluxStepper(units, arch)
    cond = st.prepare(sig, GUIDANCE, pooled, txt, img_ids, txt_ids)
    rows = []
    for s in STEP_AT:
        with torch.no_grad():
            with fp32_exact():
                v32 = R.step(o32, arch, s, traj[s], c32, F32)
            v16 = R.step(o16, arch, s, traj[s], c16, BF16)
        vb = st.step(s, traj[s], cond)
        assert torch.isfinite(vb).all(), s
        rows.append({"step": s, "sigma": sig[s], "rel_l2": rel_l2(vb, v32), "rel_l2_ref_bf16": rel_l2(v16, v32),
                     "max_abs": max_abs(vb, v32), "max_abs_ref_bf16": max_abs(v16, v32)})
    fin = None
    if final:
        out = st.denoise(x0, cond)
        with torch.no_grad(), fp32_exact():
            ref32, _ = R.denoise(o32, arch, x0, c32, F32)
        fin = {"psnr": psnr(out, ref32), "psnr_ref_bf16": psnr(final16, ref32)}
    return rows, fin


def _assert_rows(rows):
    for r in rows:
        assert r["rel_l2"] <= REL_FACTOR * r["rel_l2_ref_bf16"], r
        assert r["max_abs"] <= MAX_FACTOR * r["max_abs_ref_bf16"], r


def test_c4_12b_1024_velocity_per_step_and_final_latent_vs_fp32():
    from selas_b200.model import FluxArch, random_model

    arch = FluxArch()
    units = random_model(arch, DEV, seed=0, std=0.02)
    sig, pooled, txt, img_ids, txt_ids, x0 = _inputs(arch, 1024, 1)
    rows, fin = _per_step(units, arch, sig, pooled, txt, img_ids, txt_ids, x0, final=True)
    _report("c4", {"config": "C4: FLUX-12B bf16, 1024^2, 1 image", "per_step": rows, "final": fin,
                   "bars": {"rel_factor": REL_FACTOR, "max_factor": MAX_FACTOR, "psnr_margin_db": PSNR_MARGIN_DB}})
    _assert_rows(rows)
    assert fin["psnr"] >= fin["psnr_ref_bf16"] - PSNR_MARGIN_DB, fin


def test_c5_12b_nf4_512_batch4_velocity_per_step_vs_fp32():
    from selas_b200.model import FluxArch, random_model

    arch = FluxArch()
    units = random_model(arch, DEV, seed=0, std=0.02, quant="nf4")
    sig, pooled, txt, img_ids, txt_ids, x0 = _inputs(arch, 512, 4)
    rows, _ = _per_step(units, arch, sig, pooled, txt, img_ids, txt_ids, x0, final=False)
    _report("c5", {"config": "C5: FLUX-12B, block Linears NF4 (blocksize 64), 512^2, 4 images", "per_step": rows,
                   "bars": {"rel_factor": REL_FACTOR, "max_factor": MAX_FACTOR}})
    _assert_rows(rows)
