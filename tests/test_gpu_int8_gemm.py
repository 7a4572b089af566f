"""The int8_row decoding GEMM (decode inside the tcgen05 mainloop) on a B200, through the C-ABI.

Reference for every case: the same Linear through the bf16 GEMM on the weight decoded by selas's
formula q.to(bf16) * scale.to(bf16) (selas/codecs.py:272-276), which is first checked bit for bit
against the oracle's restatement. The fused kernel decodes to the same bf16 values in shared memory,
so the two differ only by the fp32 accumulation order inside the tensor core: at most 1 bf16 ulp.
Block level: int8_row double/single blocks against the CPU oracle on the decoded weights, with the
"no further from fp32 than the reference's own bf16 path" rule of the bf16 blocks.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import flux_ref as R
from oracle import int8_ref as I
from oracle import weights as OW

from .conftest import assert_no_further, cuda_ok, ideal_linear

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a B200")]

BF16, F32 = torch.bfloat16, torch.float32
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _lib_ready():
    from selas_b200 import _lib

    _lib.lib()
    yield
    torch.cuda.synchronize()
    assert _lib.device_status() == 0


def _ulp_close(got, ref):
    torch.testing.assert_close(got.float(), ref.float(), rtol=2 ** -7, atol=1e-6)


def _case(m, n, k, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(m, k, generator=g).to(BF16).to(DEV)
    b = (torch.randn(n, generator=g) * 0.02).to(BF16).to(DEV)
    w = (torch.randn(n, k, generator=g) * 0.02).numpy()
    q, scale = I.encode(w)
    return a, b, torch.from_numpy(q).to(DEV), torch.from_numpy(scale).to(DEV)


def _decoded(q, scale):
    from selas_b200 import codec

    wd = codec.decode_int8_row(q, scale, BF16)
    ref_bits = I.decode_bf16(q.cpu().numpy(), scale.cpu().numpy())
    assert np.array_equal(wd.cpu().view(torch.int16).numpy().view(np.uint16), ref_bits)
    return wd


def _run_pair(cases, epi, out_dtype, with_resid=False):
    """The same grouped problems twice: fused int8_row, and bf16 on the decoded weights."""
    from selas_b200 import ops

    outs = {True: [], False: []}
    keep = []
    for fused in (True, False):
        probs = []
        for (a, b, q, scale), (m, n, k) in cases:
            out = torch.full((m, n), 5.0, dtype=out_dtype, device=DEV)
            if fused:
                p = ops.make_linear_i8(a, q, scale, b, m)
            else:
                w = _decoded(q, scale)
                keep.append(w)
                p = ops.make_linear(a, w, b, m)
            p.out, p.ld_out = out.data_ptr(), n
            if with_resid:
                x = torch.arange(m * n, device=DEV, dtype=F32).reshape(m, n).mul_(1e-4).sin_()
                gate = torch.linspace(-2, 2, n, device=DEV).to(BF16).reshape(1, n)
                keep += [x, gate]
                p.resid, p.ld_resid, p.gate, p.gate_batch_stride = x.data_ptr(), n, gate.data_ptr(), 0
            probs.append(p)
            outs[fused].append(out)
        ops.run_linears(probs, epi)
    torch.cuda.synchronize()
    return outs[True], outs[False]


@pytest.mark.parametrize("epi_name,out_dtype", [("bf16", BF16), ("f32", F32), ("gelu", BF16), ("resid", F32)])
@pytest.mark.parametrize("shapes", [[(300, 1280, 512)], [(77, 160, 3072)], [(40, 384, 192), (300, 384, 192)]])
def test_fused_int8_matches_decoded_bf16(epi_name, out_dtype, shapes):
    from selas_b200 import _lib

    epi = {"bf16": _lib.FB_EPI_STORE_BF16, "f32": _lib.FB_EPI_STORE_F32, "gelu": _lib.FB_EPI_GELU,
           "resid": _lib.FB_EPI_GATED_RESIDUAL}[epi_name]
    cases = [(_case(m, n, k, 30 + i), (m, n, k)) for i, (m, n, k) in enumerate(shapes)]
    fused, ref = _run_pair(cases, epi, out_dtype, with_resid=epi_name == "resid")
    for ((a, b, q, scale), (m, n, k)), f, r in zip(cases, fused, ref):
        assert torch.isfinite(f).all()
        if k >= 2048:  # one tile: the launch splits K (another accumulation order)
            assert_no_further(f, r, ideal_linear(a, _decoded(q, scale), b, "bf16" if epi_name == "f32" else epi_name))
        else:
            _ulp_close(f, r)


def test_fused_int8_c3_shape_and_special_rows():
    """M=4608 tokens, K=3072, N=3072, with an all-zero weight row (scale 1) and a row whose scale comes
    from one outlier: nearly every output bit-identical to the decoded-bf16 GEMM."""
    from selas_b200 import _lib

    m, n, k = 4608, 3072, 3072
    g = torch.Generator().manual_seed(4)
    a = torch.randn(m, k, generator=g).to(BF16).to(DEV)
    w = (torch.randn(n, k, generator=g) * 0.02).numpy()
    w[7] = 0.0
    w[9, 3] = 5.0
    q, scale = I.encode(w)
    case = (a, None, torch.from_numpy(q).to(DEV), torch.from_numpy(scale).to(DEV))
    fused, ref = _run_pair([(case, (m, n, k))], _lib.FB_EPI_STORE_BF16, BF16)
    _ulp_close(fused[0], ref[0])
    assert (fused[0] == ref[0]).float().mean().item() > 0.99
    assert not fused[0][:, 7].float().any()


def test_fused_int8_qkv_epilogue_matches_decoded():
    from selas_b200 import _lib, ops

    heads, seq, mlp = 2, 300, 512
    m, n, k = seq, 3 * heads * 128 + mlp, 256
    a, b, q, scale = _case(m, n, k, 21)
    g = torch.Generator().manual_seed(3)
    cos, sin = torch.rand(seq, 64, generator=g).to(DEV), torch.rand(seq, 64, generator=g).to(DEV)
    qs, ks = (1 + 0.1 * torch.randn(128, generator=g)).to(DEV), (1 + 0.1 * torch.randn(128, generator=g)).to(DEV)
    w = _decoded(q, scale)
    res = []
    for fused in (True, False):
        qq = torch.zeros(1, heads, seq, 128, dtype=BF16, device=DEV)
        kk, v = torch.zeros_like(qq), torch.zeros_like(qq)
        cat = torch.zeros(m, 256 + mlp, dtype=BF16, device=DEV)
        p = ops.make_linear_i8(a, q, scale, b, m) if fused else ops.make_linear(a, w, b, m)
        p.q, p.k_out, p.v, p.q_scale, p.k_scale = qq.data_ptr(), kk.data_ptr(), v.data_ptr(), qs.data_ptr(), ks.data_ptr()
        p.rope_cos, p.rope_sin = cos.data_ptr(), sin.data_ptr()
        p.heads, p.head_dim, p.seq_total, p.seq_offset, p.qkv_cols = heads, 128, seq, 0, 3 * heads * 128
        p.out, p.ld_out, p.gelu_col0 = cat.data_ptr(), 256 + mlp, 256
        ops.run_linears([p], _lib.FB_EPI_QKV)
        res.append((qq, kk, v, cat[:, 256:]))
    for f, r in zip(*res):
        _ulp_close(f, r)


def test_int8_rejects_k_not_multiple_of_64():
    from selas_b200 import _lib, ops

    a, b, q, scale = _case(64, 256, 96, 5)
    p = ops.make_linear_i8(a, q, scale, b, 64)
    out = torch.empty(64, 256, dtype=BF16, device=DEV)
    p.out, p.ld_out = out.data_ptr(), 256
    with pytest.raises(_lib.FluxB200Error, match="k % 64"):
        ops.run_linears([p], _lib.FB_EPI_STORE_BF16)


def _int8_unit(tensors: dict):
    """A ResidentUnit whose 2-D Linear weights are int8_row (selas --quant int8), plus the fp32 dict of
    the decoded values for the oracle."""
    from selas_b200.model import ResidentUnit

    raw, i8, decoded = {}, {}, {}
    for name, t in tensors.items():
        if name.endswith(".weight") and t.dim() == 2:
            q, scale = I.encode(t.numpy())
            i8[name] = {"q": torch.from_numpy(q).to(DEV), "scale": torch.from_numpy(scale).to(DEV)}
            bits = I.decode_bf16(q, scale)
            decoded[name] = torch.from_numpy((bits.astype(np.uint32) << 16).view(np.float32)).reshape(t.shape)
        else:
            raw[name] = t.to(DEV, F32 if name.endswith("_norm.scale") else BF16)
            decoded[name] = t
    return ResidentUnit(raw, None, i8), decoded


def test_int8_blocks_match_oracle_on_decoded_weights():
    from selas_b200 import flux as B

    a = OW.Arch(hidden=256, heads=2, mlp_hidden=1024, depth_double=1, depth_single=1, context_dim=256, vec_dim=256)
    du, dd = _int8_unit(OW.double_unit(a, 5, 0))
    su, sd = _int8_unit(OW.single_unit(a, 5, 0))
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
