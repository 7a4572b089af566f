"""selas's kernel warm-up on the B200 kernels (selas/models/flux.py:263-294).

selas's ``warm_kernels`` runs the three blocks once on zeros, with ``_ShapeOnly`` stand-ins for the
weight views (``get`` returns zeros of the right shape, ``linear`` returns zeros, and there is no
``codec``/``parts``/``spec``), from a background thread while the weights load
(pipeline.py:375-394). The B200 object must take that call: with the one-line block dispatch
(``getattr(self.k, "double_block", double_block)`` at flux.py:502/504, likewise for the single block
and the final layer) the runner calls ``k.double_block`` / ``k.single_block`` / ``k.final_layer`` with
those views, and without it selas's own block bodies call ``k``'s seven segments. Both are exercised here,
the second through the microbench's restatement of selas's block bodies (checked against the oracle
in tests/test_eager_yardstick.py), with ``_ShapeOnly`` restated from its interface.
"""

from __future__ import annotations

import threading

import pytest
import torch

from .conftest import cuda_ok

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a B200")]

BF16, F32 = torch.bfloat16, torch.float32


class ShapeOnly:
    """The interface of selas's ``_ShapeOnly`` (flux.py:263-273): shapes, dt, device, get, linear."""

    def __init__(self, shapes, dt, device):
        self.shapes, self.dt, self.device = shapes, dt, device

    def get(self, name, dtype=None):
        return torch.zeros(self.shapes[name], dtype=dtype or self.dt, device=self.device)

    def linear(self, x, prefix, dtype=None):
        return torch.zeros(*x.shape[:-1], self.shapes[prefix + ".weight"][0], dtype=x.dtype, device=x.device)


def _shapes(arch):
    from selas_b200.model import _lin_shapes, _norm_names

    out = {}
    for kind in ("double", "single", "globals"):
        s = {}
        for name, (n, k) in _lin_shapes(arch, kind).items():
            s[name + ".weight"] = (n, k)
            s[name + ".bias"] = (n,)
        for name in _norm_names(kind):
            s[name] = (arch.head_dim,)
        out[kind] = s
    return out


def _warm(k, arch, shapes, l_img, l_txt, batch, dt, dev, blocks):
    """The body of selas's warm_kernels (flux.py:277-294) with the block functions given."""
    double, single, final = blocks
    z = lambda *s, d=F32: torch.zeros(*s, dtype=d, device=dev)  # noqa: E731
    d = arch.hidden
    img, txt = z(batch, l_img, d), z(batch, l_txt, d)
    cos, sin = z(l_txt + l_img, arch.head_dim // 2), z(l_txt + l_img, arch.head_dim // 2)
    oi, ot = double(ShapeOnly(shapes["double"], dt, dev), img, txt, z(batch, 12 * d, d=dt), cos, sin, arch, dt, False, k)
    x = torch.cat((txt, img), 1)
    xs = single(ShapeOnly(shapes["single"], dt, dev), x, z(batch, 3 * d, d=dt), cos, sin, arch, dt, False, k)
    fo = final(ShapeOnly(shapes["globals"], dt, dev), x[:, l_txt:], z(batch, 2 * d, d=dt), dt, k)
    torch.cuda.synchronize(dev)
    return oi, ot, xs, fo


@pytest.mark.parametrize("batch", [1, 2])
def test_warm_kernels_through_block_dispatch_on_shape_only_views(batch):
    from selas_b200 import _lib
    from selas_b200.flux import B200Kernels
    from selas_b200.model import FluxArch

    arch = FluxArch(hidden=256, heads=2, mlp_hidden=1024)
    k = B200Kernels()
    dev = torch.device("cuda")
    blocks = (k.double_block, k.single_block, k.final_layer)  # what the dispatched runner calls
    outs = _warm(k, arch, _shapes(arch), 64, 16, batch, BF16, dev, blocks)
    for t in outs:
        assert torch.isfinite(t.float()).all() and t.abs().max().item() == 0.0  # zeros in, zero weights: zeros out
    assert _lib.device_status() == 0


def test_warm_kernels_from_a_background_thread_while_the_main_thread_computes():
    """The reference runs the warm-up on a background thread (pipeline.py:375-394): the library's
    set-up and launches from two host threads at once must both complete, the main thread's result
    unaffected."""
    from selas_b200 import _lib, ops
    from selas_b200.flux import B200Kernels
    from selas_b200.model import FluxArch

    arch = FluxArch(hidden=256, heads=2, mlp_hidden=1024)
    k = B200Kernels()
    dev = torch.device("cuda")
    blocks = (k.double_block, k.single_block, k.final_layer)  # what the dispatched runner calls
    err = []

    def bg():
        try:
            with torch.cuda.stream(torch.cuda.Stream()):
                _warm(k, arch, _shapes(arch), 64, 16, 1, BF16, dev, blocks)
        except Exception as e:  # surfaced below
            err.append(e)

    g = torch.Generator().manual_seed(0)
    a = torch.randn(300, 512, generator=g).to(BF16).to(dev)
    w = (torch.randn(768, 512, generator=g) * 0.02).to(BF16).to(dev)
    ref = ops.linear(a, w)
    t = threading.Thread(target=bg)
    t.start()
    got = [ops.linear(a, w) for _ in range(20)]
    t.join(timeout=120)
    assert not t.is_alive() and not err, err
    torch.cuda.synchronize()
    assert all(torch.equal(x, ref) for x in got)
    assert _lib.device_status() == 0


def test_warm_kernels_through_selas_block_bodies_with_b200_segments():
    """Without the block dispatch, selas's block bodies call the seven segments of ``k`` with its
    own argument shapes on the zero inputs (restated block bodies, flux.py:298-343)."""
    from selas_b200 import _lib
    from selas_b200 import microbench as M
    from selas_b200.flux import B200Kernels
    from selas_b200.model import FluxArch

    arch = FluxArch(hidden=256, heads=2, mlp_hidden=1024)
    k = B200Kernels()
    dev = torch.device("cuda")
    d = arch.hidden
    sh = _shapes(arch)
    z = lambda *s, d_=F32: torch.zeros(*s, dtype=d_, device=dev)  # noqa: E731
    img, txt = z(1, 64, d), z(1, 16, d)
    cos, sin = z(80, 64), z(80, 64)
    oi, ot = M.yardstick_double(ShapeOnly(sh["double"], BF16, dev), img, txt, z(1, 12 * d, d_=BF16), cos, sin,
                                arch.heads, k)
    xs = M.yardstick_single(ShapeOnly(sh["single"], BF16, dev), torch.cat((ot, oi), 1), z(1, 3 * d, d_=BF16), cos, sin,
                            arch.heads, arch.mlp_hidden, k)
    torch.cuda.synchronize()
    for t in (oi, ot, xs):
        assert torch.isfinite(t).all() and t.abs().max().item() == 0.0
    assert _lib.device_status() == 0
