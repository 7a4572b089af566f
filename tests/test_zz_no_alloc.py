"""fb_linear_nf4_static: the NF4 Linear for callers that cannot allocate device memory.

Some callers of this library cannot call cudaMalloc: selas hands its weight arena every spare byte of
HBM and budgets the rest exactly, so an extra workspace mid-step risks running out of memory, and code
being captured into a CUDA graph may not allocate at all. For them fb_linear_nf4_static decodes the
NF4 weight into a fixed 16 MiB array inside the library instead of a caller workspace. This test calls
it through the C-ABI before the library's own fb_init has run (so nothing has allocated the status
word either), twice in a row with different problems, and checks both results against the workspace
entry point fb_linear_nf4 with the bit-exact tolerance the other NF4 Linear tests use, and directly
against the oracle (the reference's NF4 decode, then an fp32 matmul) within one bf16 ulp.
A kernel of this path that gives up on a bounded wait must be visible through
fb_linear_nf4_static_status, which allocates nothing either.

The file name sorts last so that a run stopping at the first failure has already run every other test.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import nf4_ref as N

from .conftest import cuda_ok

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a B200")]

BF16, F32 = torch.bfloat16, torch.float32
DEV = "cuda"


def _problem(m, n, k, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(m, k, generator=g).to(BF16).to(DEV)
    b = (torch.randn(n, generator=g) * 0.02).to(BF16).to(DEV)
    w = (torch.randn(n, k, generator=g) * 0.02).numpy()
    packed, absmax = N.encode(w, 64)
    packed, absmax = torch.from_numpy(packed).to(DEV), torch.from_numpy(absmax).to(DEV)
    code = torch.tensor(N.NF4_CODE, device=DEV)
    return a, b, packed, absmax, code


def _oracle(a, b, packed, absmax, n, k):
    """The reference's arithmetic: the NF4 decode of oracle.nf4_ref (bit-exact with selas's
    codecs.py:178-199) to bf16, then F.linear (store.py:289-293) as an fp32 matmul (TF32 off) with the
    bias, unrounded, on the GPU."""
    bits = N.decode(packed.cpu().numpy(), absmax.cpu().numpy(), 64, "bfloat16").astype(np.uint32) << 16
    w = torch.from_numpy(bits.view(np.float32).reshape(n, k)).to(DEV)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        return a.float() @ w.t() + b.float()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def _close_to_oracle(out, y, epi, extra):
    """Within one bf16 ulp of the fp32 result, as the other GEMM tests allow (the fp32 accumulation
    orders differ); for the gated residual, one ulp of the Linear output times the gate."""
    from selas_b200 import _lib

    if epi == _lib.FB_EPI_GATED_RESIDUAL:
        x, gate = extra
        ref = x + gate.float() * y.to(BF16).float()
        torch.testing.assert_close(out, ref, rtol=1e-5, atol=2 ** -7 * 8)
    else:
        torch.testing.assert_close(out.float(), y.to(BF16).float(), rtol=2 ** -7,
                                   atol=2 ** -7 * y.abs().max().item() * 1e-3)


def test_static_nf4_linear_matches_workspace_entry_and_oracle_on_two_calls():
    from selas_b200 import _lib, ops

    lib = _lib.load()  # symbols only: fb_init has not necessarily run in this process
    stream = torch.cuda.current_stream().cuda_stream
    cases = [  # (m, n, k, epilogue); k = 15360 needs three 512-row chunks of the fixed array
        (257, 1536, 15360, _lib.FB_EPI_STORE_BF16),
        (130, 768, 3072, _lib.FB_EPI_GATED_RESIDUAL),
    ]
    keep, results = [], []
    for i, (m, n, k, epi) in enumerate(cases):
        a, b, packed, absmax, code = _problem(m, n, k, 100 + i)
        out = torch.full((m, n), 3.0, dtype=F32 if epi == _lib.FB_EPI_GATED_RESIDUAL else BF16, device=DEV)
        p = ops.make_linear_nf4(a, packed, absmax, code, 64, n, b, m)
        p.out, p.ld_out = out.data_ptr(), n
        extra = []
        if epi == _lib.FB_EPI_GATED_RESIDUAL:
            x = torch.randn(m, n, device=DEV)
            gate = torch.randn(1, n, device=DEV).to(BF16)
            p.resid, p.ld_resid, p.gate, p.gate_batch_stride = x.data_ptr(), n, gate.data_ptr(), 0
            extra = [x, gate]
        rc = lib.fb_linear_nf4_static(ctypes.byref(p), epi, stream)
        assert rc == 0, lib.fb_last_error().decode()
        keep.append((a, b, packed, absmax, code, extra))
        results.append((p, epi, out))
    torch.cuda.synchronize()
    code_ = ctypes.c_int32(-1)
    assert lib.fb_linear_nf4_static_status(ctypes.byref(code_), 1) == 0 and code_.value == 0

    for (p, epi, out), (m, n, k, _), (a, b, packed, absmax, code, extra) in zip(results, cases, keep):
        ref = torch.full_like(out, -1.0)
        q = _lib.FbLinear.from_buffer_copy(p)
        q.out = ref.data_ptr()
        ws = torch.empty(n * k, dtype=BF16, device=DEV)  # the whole weight at once
        ops.run_linear_nf4(q, epi, ws)
        torch.cuda.synchronize()
        assert torch.equal(out, ref), f"static entry differs from fb_linear_nf4 for {m}x{n}x{k}"
        assert torch.isfinite(out.float()).all()

        _close_to_oracle(out, _oracle(a, b, packed, absmax, n, k), epi, extra)


def test_static_nf4_linear_rejects_k_beyond_the_fixed_array():
    from selas_b200 import _lib, ops

    lib = _lib.load()
    a, b, packed, absmax, code = _problem(16, 256, 40960, 7)
    out = torch.empty(16, 256, dtype=BF16, device=DEV)
    p = ops.make_linear_nf4(a, packed, absmax, code, 64, 256, b, 16)
    p.out, p.ld_out = out.data_ptr(), 256
    rc = lib.fb_linear_nf4_static(ctypes.byref(p), _lib.FB_EPI_STORE_BF16, torch.cuda.current_stream().cuda_stream)
    assert rc == 1  # FB_ERR_ARG, nothing launched
    assert "too large" in lib.fb_last_error().decode()


def test_static_status_word_reports_a_timed_out_wait():
    """A wait on the fixed array's status word that runs out (20 ms, on an mbarrier nothing completes)
    is reported by fb_linear_nf4_static_status, stays until a clearing read, and is not wiped by the
    next fb_linear_nf4_static call; raise_on_device_error sees it once the static path has been used."""
    from selas_b200 import _lib, ops

    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    assert _lib.static_status(clear=True) == 0
    assert lib.fb_selftest_static_wait_timeout(20, stream) == 0, lib.fb_last_error().decode()
    torch.cuda.synchronize()  # the kernel returned (no hang, no fault)
    # a call after the timeout keeps the recorded code, and still computes correctly
    a, b, packed, absmax, code = _problem(64, 256, 512, 3)
    out = torch.empty(64, 256, dtype=BF16, device=DEV)
    p = ops.make_linear_nf4(a, packed, absmax, code, 64, 256, b, 64)
    p.out, p.ld_out = out.data_ptr(), 256
    ops.run_linear_nf4_static(p, _lib.FB_EPI_STORE_BF16)
    assert _lib.static_status(clear=False) == 3  # FB_DEV_TIMEOUT_EPI, still there
    _close_to_oracle(out, _oracle(a, b, packed, absmax, 256, 512), _lib.FB_EPI_STORE_BF16, [])
    with pytest.raises(_lib.FluxB200Error, match="timeout"):
        _lib.raise_on_device_error()  # reads and clears the static word
    assert _lib.static_status(clear=False) == 0
    assert lib.fb_selftest_static_wait_timeout(0, stream) == 1  # FB_ERR_ARG
