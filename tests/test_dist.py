"""Host-side multi-GPU logic on CPU: image sharding, the max-over-ranks timing and the per-rank figures
bench.py reports, with two gloo ranks.
Also: a rank that fails is seen by the other ranks as an error, not a hang (short process-group timeout)."""

from __future__ import annotations

import multiprocessing as mp
import os
import socket

import pytest

from selas_b200.dist import shard


def test_shard_covers_every_image_once():
    for n in (1, 7, 8, 32, 33):
        for w in (1, 2, 3, 8):
            seen = [i for r in range(w) for i in shard(n, r, w)]
            assert seen == list(range(n))
            sizes = [len(shard(n, r, w)) for r in range(w)]
            assert max(sizes) - min(sizes) <= 1
    assert list(shard(32, 3, 8)) == [12, 13, 14, 15]  # C5: 4 images per GPU
    with pytest.raises(ValueError):
        shard(4, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, mode: str, q, start):
    import datetime

    import torch.distributed as td

    # every rank has imported torch before the rendezvous starts, so that the short process-group
    # timeout below measures the collective, not a slow interpreter start on a loaded machine
    start.wait(timeout=300)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    td.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    from selas_b200.dist import max_over_ranks, per_rank

    try:
        if mode == "ok":
            q.put((rank, max_over_ranks(10.0 + rank), list(shard(8, rank, world)),
                   per_rank(None if rank == 1 else 5.0 * (rank + 1))))
        else:
            if rank == 1:
                raise RuntimeError("rank 1 fails before the collective")
            try:
                max_over_ranks(1.0)
                q.put((rank, "no error"))
            except Exception as e:  # the peer never joins: gloo times out with an error
                q.put((rank, type(e).__name__))
    except RuntimeError as e:
        q.put((rank, str(e)))
    finally:
        try:
            td.destroy_process_group()
        except Exception:
            pass


def _run(mode: str, world: int = 2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    start = ctx.Barrier(world)
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, mode, q, start)) for r in range(world)]
    for p in ps:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(out, key=lambda t: t[0])


def test_two_gloo_ranks_max_timing_and_disjoint_shards():
    out = _run("ok")
    assert [o[1] for o in out] == [11.0, 11.0]  # every rank sees the slowest rank's time
    assert out[0][2] == [0, 1, 2, 3] and out[1][2] == [4, 5, 6, 7]
    assert out[0][3] == out[1][3] == [5.0, None]  # every rank's figure, in rank order; None survives


def test_failed_rank_surfaces_as_an_error_on_the_others():
    out = _run("fail")
    assert out[1][1] == "rank 1 fails before the collective"
    assert out[0][1] != "no error"  # rank 0's collective ended with an error instead of hanging
