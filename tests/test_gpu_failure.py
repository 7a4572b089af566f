"""Device-side failure detection, without a GPU fault: a kernel whose bounded wait runs out (on an
mbarrier that nothing completes, 20 ms budget) must record its code in the status word and return;
the host sees the code (and raise_on_device_error raises), and the CUDA context stays usable, so the
next kernel computes correctly. Every wait of the library's kernels goes through the same path."""

from __future__ import annotations

import pytest
import torch

from oracle import flux_ref as R

from .conftest import cuda_ok

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a B200")]

BF16 = torch.bfloat16


def test_timed_out_wait_sets_status_and_context_stays_usable():
    from selas_b200 import _lib, ops

    L = _lib.lib()
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == 0
    _lib.check(L.fb_selftest_wait_timeout(20, torch.cuda.current_stream().cuda_stream), "fb_selftest_wait_timeout")
    torch.cuda.synchronize()  # the kernel returned (no hang, no fault)
    assert _lib.device_status(clear=True) == 3  # FB_DEV_TIMEOUT_EPI
    assert _lib.device_status(clear=False) == 0  # cleared

    _lib.check(L.fb_selftest_wait_timeout(20, torch.cuda.current_stream().cuda_stream), "fb_selftest_wait_timeout")
    torch.cuda.synchronize()
    with pytest.raises(_lib.FluxB200Error, match="timeout"):
        _lib.raise_on_device_error()

    # the next kernel runs normally and correctly
    g = torch.Generator().manual_seed(2)
    x = torch.randn(2, 33, 3072, generator=g) * 3 + 0.5
    mod = torch.randn(2, 6144, generator=g).to(BF16)
    ref = R.mod_in(x, mod[:, None, :3072].float(), mod[:, None, 3072:].float(), BF16)
    got = ops.ln_mod(x.cuda(), mod[:, :3072].cuda(), mod[:, 3072:].cuda()).cpu()
    torch.testing.assert_close(got.float(), ref.float(), rtol=2 ** -7, atol=1e-6)
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == 0


def test_selftest_rejects_bad_budget():
    from selas_b200 import _lib

    L = _lib.lib()
    assert L.fb_selftest_wait_timeout(0, torch.cuda.current_stream().cuda_stream) == 1  # FB_ERR_ARG
    assert b"budget_ms" in L.fb_last_error()


def test_peer_barrier_times_out_when_a_rank_never_arrives():
    """fb_peer_barrier with a second 'rank' whose flags nobody writes (both flag arrays on this GPU): the
    wait for the missing rank must give up after its budget (30 ms), record FB_DEV_TIMEOUT_PEER, and
    leave the context usable; with the other rank's flag set first, the same barrier passes."""
    from selas_b200 import _lib, ops

    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == 0
    flags = [torch.zeros(8, dtype=torch.int32, device="cuda") for _ in range(2)]
    ptrs = [f.data_ptr() for f in flags]
    ops.peer_barrier(ptrs, 0, 1, 30)  # rank 0 waits for rank 1, which never arrives
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == 5  # FB_DEV_TIMEOUT_PEER
    assert flags[1][0].item() == 1  # rank 0 still posted its arrival in rank 1's array
    flags[0][1] = 2  # rank 1 "arrives" for epoch 2
    ops.peer_barrier(ptrs, 0, 2, 30)
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == 0
    with pytest.raises(_lib.FluxB200Error, match="world"):
        ops.peer_barrier(ptrs, 2, 1, 30)  # rank outside the world
