"""fp8 raw weights (e4m3fn and e5m2) decoded inside the tcgen05 GEMM mainloop, through the C-ABI.

selas keeps fp8 sources raw and casts them at use (selas/convert.py:178-180, codecs.py:270-271). The
reference for every case: the bf16 GEMM on the cast weight, the cast itself checked bit for bit
against the oracle's fp8 decode. The two GEMMs differ only by fp32 accumulation order: at most 1 bf16
ulp. The weights cover every finite fp8 code (subnormals, the largest normals, negative zero).
Block level: fp8 double/single blocks against the CPU oracle on the cast weights.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import flux_ref as R
from oracle import fp8_ref as F8
from oracle import weights as OW

from .conftest import cuda_ok

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a B200")]

BF16, F32 = torch.bfloat16, torch.float32
DEV = "cuda"
FMT = {False: torch.float8_e4m3fn, True: torch.float8_e5m2}


@pytest.fixture(scope="module", autouse=True)
def _lib_ready():
    from selas_b200 import _lib

    _lib.lib()
    yield
    torch.cuda.synchronize()
    assert _lib.device_status() == 0


def _ulp_close(got, ref):
    torch.testing.assert_close(got.float(), ref.float(), rtol=2 ** -7, atol=1e-6)


def _finite_codes(e5m2: bool) -> np.ndarray:
    codes = np.arange(256, dtype=np.uint8)
    return codes[np.isfinite(F8.decode(codes, e5m2))]


def _weight(n, k, e5m2, seed, scale_codes=True):
    """fp8 [n, k]: N(0, 0.02) weights cast to fp8, with the first rows cycling through every finite code."""
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(n, k, generator=g) * 0.02).to(FMT[e5m2])
    if scale_codes:
        codes = _finite_codes(e5m2)
        flat = np.resize(codes, (min(n, 4), k))
        w.view(torch.uint8)[: flat.shape[0]] = torch.from_numpy(flat)
    return w


def _cast(w8: torch.Tensor, e5m2: bool) -> torch.Tensor:
    wd = w8.to(DEV).to(BF16)
    ref = torch.from_numpy(F8.decode(w8.view(torch.uint8).numpy(), e5m2)).to(BF16)
    assert torch.equal(wd.cpu().view(torch.int16), ref.view(torch.int16))
    return wd


@pytest.mark.parametrize("e5m2", [False, True])
@pytest.mark.parametrize("epi_name,out_dtype", [("bf16", BF16), ("resid", F32)])
@pytest.mark.parametrize("shapes", [[(300, 1280, 512)], [(40, 384, 192), (300, 384, 192)]])
def test_fused_fp8_matches_cast_bf16(e5m2, epi_name, out_dtype, shapes):
    from selas_b200 import _lib, ops

    epi = {"bf16": _lib.FB_EPI_STORE_BF16, "resid": _lib.FB_EPI_GATED_RESIDUAL}[epi_name]
    outs = {True: [], False: []}
    keep = []
    data = []
    for i, (m, n, k) in enumerate(shapes):
        g = torch.Generator().manual_seed(40 + i)
        a = (torch.randn(m, k, generator=g) * 0.1).to(BF16).to(DEV)
        b = (torch.randn(n, generator=g) * 0.02).to(BF16).to(DEV)
        w8 = _weight(n, k, e5m2, 50 + i)
        data.append((a, b, w8, (m, n, k)))
    for fused in (True, False):
        probs = []
        for a, b, w8, (m, n, k) in data:
            out = torch.full((m, n), 5.0, dtype=out_dtype, device=DEV)
            if fused:
                wd = w8.to(DEV)
                p = ops.make_linear_f8(a, wd, b, m)
            else:
                wd = _cast(w8, e5m2)
                p = ops.make_linear(a, wd, b, m)
            keep.append(wd)
            p.out, p.ld_out = out.data_ptr(), n
            if epi_name == "resid":
                x = torch.arange(m * n, device=DEV, dtype=F32).reshape(m, n).mul_(1e-4).sin_()
                gate = torch.linspace(-2, 2, n, device=DEV).to(BF16).reshape(1, n)
                keep += [x, gate]
                p.resid, p.ld_resid, p.gate, p.gate_batch_stride = x.data_ptr(), n, gate.data_ptr(), 0
            probs.append(p)
            outs[fused].append(out)
        ops.run_linears(probs, epi)
    torch.cuda.synchronize()
    for f, r in zip(outs[True], outs[False]):
        assert torch.isfinite(f).all()
        _ulp_close(f, r)


def _fp8_unit(tensors: dict, e5m2: bool):
    from selas_b200.model import ResidentUnit

    raw, decoded = {}, {}
    for name, t in tensors.items():
        if name.endswith(".weight") and t.dim() == 2:
            w8 = t.to(FMT[e5m2])
            raw[name] = w8.to(DEV)
            decoded[name] = torch.from_numpy(F8.decode(w8.view(torch.uint8).numpy(), e5m2)).reshape(t.shape)
        else:
            raw[name] = t.to(DEV, F32 if name.endswith("_norm.scale") else BF16)
            decoded[name] = t
    return ResidentUnit(raw), decoded


@pytest.mark.parametrize("e5m2", [False, True])
def test_fp8_blocks_match_oracle_on_cast_weights(e5m2):
    from selas_b200 import flux as B

    a = OW.Arch(hidden=256, heads=2, mlp_hidden=1024, depth_double=1, depth_single=1, context_dim=256, vec_dim=256)
    du, dd = _fp8_unit(OW.double_unit(a, 5, 0), e5m2)
    su, sd = _fp8_unit(OW.single_unit(a, 5, 0), e5m2)
    img, txt, dmod, smod, _ = OW.block_inputs(a, 6, 256, 64, 2)
    cos, sin = R.rope_tables(torch.cat((R.text_ids(64), R.image_ids(256, 256)), 0), a.axes_dim)
    oi, ot = B.double_block(du, img.to(DEV), txt.to(DEV), dmod.to(DEV, BF16), cos.to(DEV), sin.to(DEV), a, BF16, False)
    x = torch.cat((txt, img), 1)
    xs = B.single_block(su, x.to(DEV), smod.to(DEV, BF16), cos.to(DEV), sin.to(DEV), a, BF16, False)
    with torch.no_grad():
        r32 = R.double_block(dd, img, txt, dmod, cos, sin, a.heads, F32)
        r16 = R.double_block(dd, img, txt, dmod.to(BF16), cos, sin, a.heads, BF16)
        s32 = R.single_block(sd, x, smod, cos, sin, a.heads, a.mlp_hidden, F32)
        s16 = R.single_block(sd, x, smod.to(BF16), cos, sin, a.heads, a.mlp_hidden, BF16)

    def check(got, ref32, ref16):
        got, ref32, ref16 = got.cpu().double(), ref32.double(), ref16.double()
        spread = ((ref16 - ref32).norm() / ref32.norm()).item()
        err = ((got - ref32).norm() / ref32.norm()).item()
        assert err <= 1.5 * spread, (err, spread)
        assert (got - ref32).abs().max().item() <= 2.0 * (ref16 - ref32).abs().max().item()

    check(oi, r32[0], r16[0])
    check(ot, r32[1], r16[1])
    check(xs, s32, s16)
