"""Ulysses sequence parallelism on CPU: two gloo ranks run the all-to-all attention of
selas_b200.sp with the oracle's attention (selas/models/flux.py:135-138) in place of the tcgen05
kernel, and must reproduce attention over the whole sequence for their own tokens. This covers the
index math of both exchanges (head groups out, token rows back), the txt/img split of the local
rows, and the per-rank RoPE rows of ``Ulysses.localize``."""

from __future__ import annotations

import multiprocessing as mp
import os
import socket

import torch

from oracle import flux_ref as R


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ref_attention(q, k, v, out):
    out.copy_(R.attention(q.float(), k.float(), v.float()).to(out.dtype))


def _full_inputs(b=2, h=4, lt=6, li=10, d=16):
    g = torch.Generator().manual_seed(7)
    q, k, v = (torch.randn(b, h, lt + li, d, generator=g) for _ in range(3))
    return q, k, v


def _worker(rank: int, world: int, port: int, q_out):
    import datetime
    from dataclasses import dataclass

    import torch.distributed as td

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    td.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        from selas_b200.sp import Ulysses

        sp = Ulysses(attention_fn=_ref_attention)
        b, h, lt, li, d = 2, 4, 6, 10, 16
        q, k, v = _full_inputs(b, h, lt, li, d)
        ts, is_ = sp.span(lt), sp.span(li)
        rows = torch.cat((torch.arange(ts.start, ts.stop), lt + torch.arange(is_.start, is_.stop)))
        nt = ts.stop - ts.start
        full = R.attention(q, k, v)  # [B, L, H*D] over the whole sequence
        err = 0.0
        packed = torch.stack([t[:, :, rows] for t in (q, k, v)])  # one buffer, as the blocks allocate
        separate = [t[:, :, rows].contiguous() for t in (q, k, v)]
        for ql, kl, vl in (tuple(packed), tuple(separate)):
            out_img = torch.full((b, len(rows) - nt, h * d), float("nan"))
            out_txt = torch.full((b, nt, h * d), float("nan"))
            sp.attention(ql, kl, vl, out=out_img, split=nt, out_first=out_txt)
            err = max(err, (out_txt - full[:, ts]).abs().max().item(),
                      (out_img - full[:, lt + is_.start:lt + is_.stop]).abs().max().item())

        @dataclass
        class Cond:
            txt: torch.Tensor
            cos: torch.Tensor
            sin: torch.Tensor
            l_txt: int

        cos = torch.arange(lt + li, dtype=torch.float32)[:, None].expand(lt + li, 3).contiguous()
        c = sp.localize(Cond(torch.arange(b * lt * 2, dtype=torch.float32).view(b, lt, 2), cos, -cos, lt), li)
        loc_ok = (c.l_txt == nt and c.cos[:, 0].tolist() == rows.float().tolist()
                  and torch.equal(c.txt, torch.arange(b * lt * 2, dtype=torch.float32).view(b, lt, 2)[:, ts]))
        q_out.put((rank, err, loc_ok))
    except Exception as e:  # report, so that the test fails instead of hanging
        q_out.put((rank, repr(e), False))
    finally:
        td.destroy_process_group()


def test_ulysses_attention_two_ranks_matches_full_sequence():
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q_out.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    for rank, err, loc_ok in res:
        assert isinstance(err, float), (rank, err)
        assert err < 1e-5, (rank, err)
        assert loc_ok, rank
