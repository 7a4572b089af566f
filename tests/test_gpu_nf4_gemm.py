"""The fused NF4 GEMM (decode inside the tcgen05 mainloop) on a B200, through the C-ABI.

Reference for every case: the same Linear run through the bf16 GEMM on the weight decoded by the
bit-exact NF4 kernel (whose output equals selas's nf4_dequant_torch bit for bit). The fused kernel
decodes to the same bf16 values in shared memory, so the two may differ only by the fp32
accumulation order inside the tensor core: at most 1 bf16 ulp on the rounded outputs.
Block level: NF4 double/single blocks against the CPU oracle on the decoded weights, with the same
"no further from fp32 than the reference's own bf16 path" rule as the bf16 blocks.
"""

from __future__ import annotations

import pytest
import torch

from oracle import flux_ref as R
from oracle import nf4_ref as N
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
    """<= 1 bf16 ulp apart, elementwise (relative 2^-7 of the reference magnitude, tiny absolute floor)."""
    torch.testing.assert_close(got.float(), ref.float(), rtol=2 ** -7, atol=1e-6)


def _case(m, n, k, seed, code=None):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(m, k, generator=g).to(BF16).to(DEV)
    b = (torch.randn(n, generator=g) * 0.02).to(BF16).to(DEV)
    w = (torch.randn(n, k, generator=g) * 0.02).numpy()
    code = N.NF4_CODE if code is None else code
    packed, absmax = N.encode(w, 64, code)
    packed, absmax = torch.from_numpy(packed).to(DEV), torch.from_numpy(absmax).to(DEV)
    code_t = torch.tensor(code, dtype=F32, device=DEV)
    return a, b, packed, absmax, code_t


def _run_pair(cases, epi, out_dtype, with_resid=False):
    """Run the same grouped problems twice: fused NF4, and bf16 on the decoded weights."""
    from selas_b200 import ops

    outs = {True: [], False: []}
    keep = []
    for fused in (True, False):
        probs = []
        for (a, b, packed, absmax, code), (m, n, k) in cases:
            out = torch.full((m, n), 5.0, dtype=out_dtype, device=DEV)
            if fused:
                p = ops.make_linear_nf4(a, packed, absmax, code, 64, n, b, m)
            else:
                w = ops.nf4_dequant(packed, absmax, 64, code, (n, k), BF16)
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
@pytest.mark.parametrize("shapes", [[(300, 1280, 512)], [(77, 160, 3072)], [(40, 384, 256), (300, 384, 256)]])
def test_fused_nf4_matches_decoded_bf16(epi_name, out_dtype, shapes):
    from selas_b200 import _lib

    epi = {"bf16": _lib.FB_EPI_STORE_BF16, "f32": _lib.FB_EPI_STORE_F32, "gelu": _lib.FB_EPI_GELU,
           "resid": _lib.FB_EPI_GATED_RESIDUAL}[epi_name]
    from selas_b200 import ops

    cases = [(_case(m, n, k, 10 + i), (m, n, k)) for i, (m, n, k) in enumerate(shapes)]
    fused, ref = _run_pair(cases, epi, out_dtype, with_resid=epi_name == "resid")
    for ((a, b, packed, absmax, code), (m, n, k)), f, r in zip(cases, fused, ref):
        assert torch.isfinite(f).all()
        if k >= 2048:  # one tile: the launch splits K (another accumulation order)
            w = ops.nf4_dequant(packed, absmax, 64, code, (n, k), BF16)
            assert_no_further(f, r, ideal_linear(a, w, b, "bf16" if epi_name == "f32" else epi_name))
        else:
            _ulp_close(f, r)


def test_fused_nf4_runtime_code_table():
    from selas_b200 import _lib

    code = tuple(float(c) * 0.75 + 0.01 for c in N.NF4_CODE)  # a quant_map that is not NF4_CODE
    cases = [(_case(200, 256, 512, 3, code), (200, 256, 512))]
    fused, ref = _run_pair(cases, _lib.FB_EPI_STORE_BF16, BF16)
    _ulp_close(fused[0], ref[0])


def test_fused_nf4_c3_shape_9216():
    """C3: M=4608 tokens, K=3072, N=9216 (the QKV weight), N(0, 0.02) weights before quantisation."""
    from selas_b200 import _lib

    cases = [(_case(4608, 9216, 3072, 4), (4608, 9216, 3072))]
    fused, ref = _run_pair(cases, _lib.FB_EPI_STORE_BF16, BF16)
    _ulp_close(fused[0], ref[0])
    exact = (fused[0] == ref[0]).float().mean().item()
    assert exact > 0.99, exact  # nearly every element is bit-identical


@pytest.mark.parametrize("n,k", [(3072, 3072), (9216, 3072), (12288, 3072), (3072, 12288)])
def test_fused_nf4_c3_shapes_vs_oracle(n, k):
    """C3, every weight shape at M=4608 tokens: the fused NF4 GEMM against the oracle (the reference's
    NF4 decode in oracle.nf4_ref, then an fp32 matmul with TF32 off and the bias), within one bf16 ulp."""
    from selas_b200 import _lib, ops

    m = 4608
    a, b, packed, absmax, code = _case(m, n, k, 40 + n // 1024)
    out = torch.empty(m, n, dtype=BF16, device=DEV)
    p = ops.make_linear_nf4(a, packed, absmax, code, 64, n, b, m)
    p.out, p.ld_out = out.data_ptr(), n
    ops.run_linears([p], _lib.FB_EPI_STORE_BF16)
    # the decode to bf16 (one fp32 multiply, then round to nearest even: codecs.py:178-199)
    w = N.decode_torch(packed, absmax, 64, (n, k), BF16).float()
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ref = (a.float() @ w.t() + b.float()).to(BF16)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    torch.testing.assert_close(out.float(), ref.float(), rtol=2 ** -7, atol=2 ** -7 * ref.float().abs().max().item() * 1e-3)


@pytest.mark.parametrize("k,seq,batch", [(256, 300, 1), (3072, 300, 1), (256, 320, 1), (256, 160, 2)])
def test_fused_nf4_qkv_epilogue_matches_decoded(k, seq, batch):
    """linear1-shaped NF4 Linear with the QKV + GELU split epilogue, against the bf16 GEMM on the decoded
    weights. k = 3072 makes few tiles, so the NF4 launch splits K four ways. Where every image's rows
    are a multiple of 32 (seq 320; two images of 160) the bf16 kernel reads the RoPE tables through
    shared memory (TMA boxes of 32 positions, restarting at each image) while the NF4 kernel reads them
    from global memory, so the staged tables are checked against the direct reads."""
    from selas_b200 import _lib, ops

    heads, mlp = 2, 512
    m, n = seq * batch, 3 * heads * 128 + mlp
    (a, b, packed, absmax, code) = _case(m, n, k, 21)
    g = torch.Generator().manual_seed(3)
    cos, sin = torch.rand(seq, 64, generator=g).to(DEV), torch.rand(seq, 64, generator=g).to(DEV)
    qs, ks = (1 + 0.1 * torch.randn(128, generator=g)).to(DEV), (1 + 0.1 * torch.randn(128, generator=g)).to(DEV)
    w = ops.nf4_dequant(packed, absmax, 64, code, (n, k), BF16)
    res = []
    for fused in (True, False):
        q = torch.zeros(batch, heads, seq, 128, dtype=BF16, device=DEV)
        kk, v = torch.zeros_like(q), torch.zeros_like(q)
        cat = torch.zeros(m, 256 + mlp, dtype=BF16, device=DEV)
        p = ops.make_linear_nf4(a, packed, absmax, code, 64, n, b, seq) if fused else ops.make_linear(a, w, b, seq)
        p.q, p.k_out, p.v, p.q_scale, p.k_scale = q.data_ptr(), kk.data_ptr(), v.data_ptr(), qs.data_ptr(), ks.data_ptr()
        p.rope_cos, p.rope_sin = cos.data_ptr(), sin.data_ptr()
        p.heads, p.head_dim, p.seq_total, p.seq_offset, p.qkv_cols = heads, 128, seq, 0, 3 * heads * 128
        p.out, p.ld_out, p.gelu_col0 = cat.data_ptr(), 256 + mlp, 256
        ops.run_linears([p], _lib.FB_EPI_QKV)
        res.append((q, kk, v, cat[:, 256:]))
    for f, r in zip(*res):
        if k >= 2048:  # split K: another fp32 accumulation order; RMSNorm and RoPE carry a flipped
            # rounding of the projection a little further, so allow 2 bf16 ulp on at most 0.1 % of values
            close = torch.isclose(f.float(), r.float(), rtol=2 ** -6, atol=1e-5)
            assert close.float().mean().item() > 0.999
            torch.testing.assert_close(f.float(), r.float(), rtol=0.05, atol=2e-2)
        else:
            _ulp_close(f, r)


@pytest.mark.parametrize("epi_name,out_dtype", [("bf16", BF16), ("resid", F32), ("gelu", BF16)])
@pytest.mark.parametrize("shapes", [
    [(64, 1536, 3072), (512, 1536, 3072)],   # 18 pair tiles: K split 4 ways (48 K steps -> 12 each)
    [(64, 3072, 3072), (512, 3072, 3072)],   # 36 tiles (an 8-way sequence-parallel rank's proj): 2 ways
    [(576, 3072, 15360)],                    # linear2 of such a rank: 36 tiles, 2 ways of 120 steps
])
def test_split_k_matches_decoded_and_is_deterministic(epi_name, out_dtype, shapes):
    """Launches whose tiles leave more than half of the 74 CTA pairs idle split K (whole 4-step NF4 groups);
    the CTA completing a tile sums the splits in split order. Same 1-ulp bound against the unsplit
    bf16 GEMM on the decoded weights, and bit-identical results when run again."""
    from selas_b200 import _lib

    from selas_b200 import ops

    epi = {"bf16": _lib.FB_EPI_STORE_BF16, "gelu": _lib.FB_EPI_GELU, "resid": _lib.FB_EPI_GATED_RESIDUAL}[epi_name]
    cases = [(_case(m, n, k, 60 + i), (m, n, k)) for i, (m, n, k) in enumerate(shapes)]
    fused, ref = _run_pair(cases, epi, out_dtype, with_resid=epi_name == "resid")
    again, _ = _run_pair(cases, epi, out_dtype, with_resid=epi_name == "resid")
    for ((a, b, packed, absmax, code), (m, n, k)), f, r, f2 in zip(cases, fused, ref, again):
        assert torch.isfinite(f).all()
        w = ops.nf4_dequant(packed, absmax, 64, code, (n, k), BF16)
        assert_no_further(f, r, ideal_linear(a, w, b, epi_name))
        assert torch.equal(f, f2)


def _nf4_unit(tensors: dict):
    """A ResidentUnit whose 2-D Linear weights are NF4 (as selas's converter writes them with --quant
    nf4), plus the fp32 dict of the decoded values for the oracle."""
    from selas_b200.model import ResidentUnit

    raw, nf4, decoded = {}, {}, {}
    for name, t in tensors.items():
        if name.endswith(".weight") and t.dim() == 2:
            packed, absmax = N.encode(t.numpy(), 64)
            nf4[name] = {"packed": torch.from_numpy(packed).to(DEV), "absmax": torch.from_numpy(absmax).to(DEV),
                         "blocksize": 64, "code": N.NF4_CODE, "shape": tuple(t.shape)}
            decoded[name] = torch.from_numpy(N.decode_f32(packed, absmax, 64)).reshape(t.shape)
            decoded[name] = decoded[name].to(BF16).float()
        else:
            raw[name] = t.to(DEV, F32 if name.endswith("_norm.scale") else BF16)
            decoded[name] = t
    return ResidentUnit(raw, nf4), decoded


def test_nf4_blocks_match_oracle_on_decoded_weights():
    from selas_b200 import flux as B

    a = OW.Arch(hidden=256, heads=2, mlp_hidden=1024, depth_double=1, depth_single=1, context_dim=256, vec_dim=256)
    du, dd = _nf4_unit(OW.double_unit(a, 5, 0))
    su, sd = _nf4_unit(OW.single_unit(a, 5, 0))
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
