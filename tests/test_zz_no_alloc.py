"""fb_linear_nf4_static: the NF4 Linear for callers that cannot allocate device memory.

Some callers of this library cannot call cudaMalloc: selas hands its weight arena every spare byte of
HBM and budgets the rest exactly, so an extra workspace mid-step risks running out of memory, and code
being captured into a CUDA graph may not allocate at all. For them fb_linear_nf4_static decodes the
NF4 weight into a fixed 16 MiB array inside the library instead of a caller workspace. This test calls
it through the C-ABI before the library's own fb_init has run (so nothing has allocated the status
word either), twice in a row with different problems, and checks both results against the workspace
entry point fb_linear_nf4 with the bit-exact tolerance the other NF4 Linear tests use.

The file name sorts last so that a run stopping at the first failure has already run every other test.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from oracle import nf4_ref as N

from .conftest import cuda_ok

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a B200")]

BF16, F32 = torch.bfloat16, torch.float32
DEV = "cuda"


def _problem(ops, m, n, k, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(m, k, generator=g).to(BF16).to(DEV)
    b = (torch.randn(n, generator=g) * 0.02).to(BF16).to(DEV)
    w = (torch.randn(n, k, generator=g) * 0.02).numpy()
    packed, absmax = N.encode(w, 64)
    packed, absmax = torch.from_numpy(packed).to(DEV), torch.from_numpy(absmax).to(DEV)
    code = torch.tensor(N.NF4_CODE, device=DEV)
    return a, b, packed, absmax, code


def test_static_nf4_linear_matches_workspace_entry_on_two_calls():
    from selas_b200 import _lib, ops

    lib = _lib.load()  # symbols only: fb_init has not necessarily run in this process
    stream = torch.cuda.current_stream().cuda_stream
    cases = [  # (m, n, k, epilogue); k = 15360 needs three 512-row chunks of the fixed array
        (257, 1536, 15360, _lib.FB_EPI_STORE_BF16),
        (130, 768, 3072, _lib.FB_EPI_GATED_RESIDUAL),
    ]
    keep, results = [], []
    for i, (m, n, k, epi) in enumerate(cases):
        a, b, packed, absmax, code = _problem(ops, m, n, k, 100 + i)
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

    for (p, epi, out), (m, n, k, _) in zip(results, cases):
        ref = torch.full_like(out, -1.0)
        q = _lib.FbLinear.from_buffer_copy(p)
        q.out = ref.data_ptr()
        ws = torch.empty(n * k, dtype=BF16, device=DEV)  # the whole weight at once
        ops.run_linear_nf4(q, epi, ws)
        torch.cuda.synchronize()
        assert torch.equal(out, ref), f"static entry differs from fb_linear_nf4 for {m}x{n}x{k}"
        assert torch.isfinite(out.float()).all()


def test_static_nf4_linear_rejects_k_beyond_the_fixed_array():
    from selas_b200 import _lib, ops

    lib = _lib.load()
    a, b, packed, absmax, code = _problem(ops, 16, 256, 40960, 7)
    out = torch.empty(16, 256, dtype=BF16, device=DEV)
    p = ops.make_linear_nf4(a, packed, absmax, code, 64, 256, b, 16)
    p.out, p.ld_out = out.data_ptr(), 256
    rc = lib.fb_linear_nf4_static(ctypes.byref(p), _lib.FB_EPI_STORE_BF16, torch.cuda.current_stream().cuda_stream)
    assert rc == 1  # FB_ERR_ARG, nothing launched
    assert "too large" in lib.fb_last_error().decode()
