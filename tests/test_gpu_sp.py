"""Ulysses sequence parallelism on two B200s: one denoise step of a small FLUX (2 double + 2 single
blocks, head_dim 128, 2 heads) with each rank holding half of the txt and half of the img tokens must
give, for its tokens, the velocity of the same step on one GPU. The kernels are the same; only the
order in which attention visits the keys differs, so the two agree to bf16 rounding noise.

Both exchanges are checked: the NCCL all-to-alls (``Ulysses``) and the peer-memory one
(``UlyssesP2P``: the QKV epilogue and the attention kernel store into the other rank's buffers over
NVLink, with the device barrier between). The two move the same bytes to the same places, so their
velocities must be bit-identical; two steps in a row check that the buffers are reused safely.
Skipped unless the machine has at least two GPUs."""

from __future__ import annotations

import multiprocessing as mp
import os
import socket

import pytest
import torch

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs two GPUs")]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q_out):
    import datetime

    import torch.distributed as td

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    td.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                          device_id=dev)
    try:
        from oracle import flux_ref as R
        from oracle import weights as OW
        from selas_b200.model import FluxArch, FluxStepper, ResidentUnit
        from selas_b200.sp import Ulysses, UlyssesP2P

        arch = OW.Arch(hidden=256, heads=2, mlp_hidden=1024, depth_double=2, depth_single=2, in_channels=64,
                       context_dim=256, vec_dim=256, axes_dim=(16, 56, 56))
        units = {n: ResidentUnit({k: t.to(dev, torch.float32 if k.endswith("_norm.scale") else torch.bfloat16)
                                  for k, t in u.items()}) for n, u in OW.all_units(arch, 3).items()}
        gen = torch.Generator().manual_seed(0)
        txt = torch.randn(1, 16, 256, generator=gen)
        pooled = torch.randn(1, 256, generator=gen)
        x0 = R.pack(R.get_noise(0, 128, 128)).to(dev)
        sig = R.get_schedule(2, x0.shape[1])
        st = FluxStepper(units, FluxArch(**arch.__dict__))
        cond = st.prepare(sig, 3.5, pooled.to(dev), txt.to(dev), R.image_ids(128, 128).to(dev),
                          R.text_ids(16).to(dev))
        full = [st.step(s, x0, cond) for s in (0, 1)]
        sp = Ulysses()
        li = x0.shape[1]
        xl, cl = x0[:, sp.span(li)].contiguous(), sp.localize(cond, li)
        mine = [st.step(s, xl, cl, sp) for s in (0, 1)]
        p2p = UlyssesP2P(arch, cl.l_txt + xl.shape[1])
        mine_p2p = [st.step(s, xl, cl, p2p) for s in (0, 1)]
        p2p.close()
        torch.cuda.synchronize()
        rel = max(((m.double() - f[:, sp.span(li)].double()).norm() / f[:, sp.span(li)].double().norm()).item()
                  for m, f in zip(mine, full))
        same = all(torch.equal(a, b) for a, b in zip(mine, mine_p2p))
        q_out.put((rank, rel, bool(all(torch.isfinite(m).all() for m in mine)) and same))
    except Exception as e:
        q_out.put((rank, repr(e), False))
    finally:
        td.destroy_process_group()


def test_ulysses_step_two_gpus_matches_one_gpu_nccl_and_p2p():
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q_out.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
    for rank, rel, finite in res:
        assert isinstance(rel, float), (rank, rel)
        assert finite, rank
        assert rel < 2e-2, (rank, rel)
