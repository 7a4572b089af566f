"""Kernel-level parity on a B200, through the C-ABI (selas_b200.ops wraps libflux_b200.so).

* NF4 decode: bit-exact against the golden vectors written by the reference and against the numpy
  oracle, every output dtype, aligned and unaligned buffers, empty input, a full C3 weight.
* LayerNorm + modulation, gated add, GELU, QK-RMSNorm + RoPE: against the CPU oracle.
* tcgen05 GEMM, every epilogue: against a torch fp32 reference of the same op (bf16 inputs, fp32
  accumulate, the same bf16 rounding points), ragged M, grouped launches, determinism.
* tcgen05 attention: against an fp32 softmax reference, ragged L, batch > 1, split outputs.
Tolerances are stated at each assert.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import flux_ref as R
from oracle import nf4_ref as N

from .conftest import GOLDEN, cuda_ok

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a B200")]

BF16, F32 = torch.bfloat16, torch.float32
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _lib_ready():
    from selas_b200 import _lib

    _lib.lib()
    yield
    torch.cuda.synchronize()
    assert _lib.device_status() == 0, "a kernel reported a device-side error"


def ops():
    from selas_b200 import ops as o

    return o


def rel_l2(a, b):
    a, b = a.double(), b.double()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


# ------------------------------------------------------------------------------------------ NF4


@pytest.fixture(scope="module")
def nf4g():
    return dict(np.load(GOLDEN / "nf4.npz"))


@pytest.mark.parametrize("case,bs", [("s1", 64), ("rb", 64), ("b128", 128), ("cc", 64)])
@pytest.mark.parametrize("dt", [F32, torch.float16, BF16])
def test_nf4_decode_bit_exact_vs_golden(nf4g, case, bs, dt):
    code = nf4g["cc_code"] if case == "cc" else nf4g["code"]
    packed = torch.from_numpy(nf4g[f"{case}_packed"]).to(DEV)
    absmax = torch.from_numpy(nf4g[f"{case}_absmax"]).to(DEV)
    out = ops().nf4_dequant(packed, absmax, bs, tuple(code.tolist()), (packed.numel() * 2,), dt)
    tag = {F32: "f32", torch.float16: "f16", BF16: "bf16"}[dt]
    ref = nf4g[f"{case}_out_{tag}"]
    got = out.cpu().view(torch.int16).numpy() if dt == BF16 else out.cpu().numpy()
    assert got.tobytes() == ref.tobytes()  # bit-exact


@pytest.mark.parametrize("case,bs", [("s1", 64), ("b128", 128), ("cc", 64)])
def test_nf4_encode_device_matches_reference(nf4g, case, bs):
    """NF4 encoding on the device (conversion time; selas/codecs.py:99-119): packed bytes and absmax bit
    for bit equal to the reference's encode_nf4 output, for the default code, blocksize 128 and a
    custom code table; exact half-way values go to the lower code."""
    from selas_b200 import codec

    code = tuple(float(c) for c in nf4g["cc_code"]) if case == "cc" else codec.NF4_CODE
    values = torch.from_numpy(nf4g[f"{case}_values"])
    packed, absmax = codec.encode_device(values.to(DEV), bs, code)
    assert np.array_equal(packed.cpu().numpy(), nf4g[f"{case}_packed"])
    assert np.array_equal(absmax.cpu().numpy(), nf4g[f"{case}_absmax"])
    # ties: normalised values exactly on the midpoints between codes go to the lower code (as the oracle)
    c = np.asarray(codec.NF4_CODE, np.float32)
    mids = ((c[1:] + c[:-1]) / np.float32(2)).astype(np.float32)
    block = np.concatenate([mids, [np.float32(1.0)], np.zeros(64 - len(mids) - 1, np.float32)]).astype(np.float32)
    p_dev, a_dev = codec.encode_device(torch.from_numpy(block).to(DEV), 64)
    p_ref, a_ref = N.encode(block, 64)
    assert np.array_equal(p_dev.cpu().numpy(), p_ref) and np.array_equal(a_dev.cpu().numpy(), a_ref)


@pytest.mark.parametrize("dt", [F32, BF16, torch.float16])
@pytest.mark.parametrize("bs", [64, 128, 32])  # 64 / 128: 8 values per lane; 32: the generic kernel
def test_nf4_encode_device_input_dtypes(dt, bs):
    """fb_nf4_encode reads bf16 / fp16 weights directly: the same bytes as encoding their fp32 values
    (selas/codecs.py:100 widens to fp32 first), checked against the oracle's restatement."""
    from selas_b200 import codec

    g = torch.Generator().manual_seed(31)
    w = (torch.randn(96, 256, generator=g) * 0.02).to(dt)
    w[3, :bs] = 0.0  # an all-zero block
    packed, absmax = codec.encode_device(w.to(DEV), bs)
    p_ref, a_ref = N.encode(w.float().numpy(), bs)
    assert np.array_equal(packed.cpu().numpy(), p_ref) and np.array_equal(absmax.cpu().numpy(), a_ref)


@pytest.mark.parametrize("dt", [F32, BF16])
def test_int8_row_encode_device_matches_reference(dt):
    """int8_row encoding on the device (selas/codecs.py:87-97): bit for bit the reference's q and scale
    for the golden rows (all-zero row, half-step ties, an outlier), and the oracle on bf16 input."""
    from selas_b200 import codec

    from oracle import int8_ref as I

    gold = np.load(GOLDEN / "int8.npz")
    if dt == F32:
        w = torch.from_numpy(gold["values"])
        q_ref, s_ref = gold["q"], gold["scale"]
    else:
        w = (torch.randn(64, 3072, generator=torch.Generator().manual_seed(8)) * 0.02).to(BF16)
        q_ref, s_ref = I.encode(w.float().numpy())
    q, scale = codec.encode_int8_row_device(w.to(DEV))
    assert np.array_equal(q.cpu().numpy(), q_ref.reshape(q.shape))
    assert np.array_equal(scale.cpu().numpy(), s_ref)


@pytest.mark.parametrize("n,k", [(3072, 3072), (9216, 3072), (12288, 3072), (3072, 12288)])
def test_nf4_decode_c3_weights_bit_exact(n, k):
    g = torch.Generator().manual_seed(n + k)
    w = (torch.randn(n, k, generator=g) * 0.02).numpy()
    packed, absmax = N.encode(w, 64)
    out = ops().nf4_dequant(torch.from_numpy(packed).to(DEV), torch.from_numpy(absmax).to(DEV), 64, N.NF4_CODE, (n, k), BF16)
    ref = N.decode(packed, absmax, 64, "bfloat16")
    assert np.array_equal(out.cpu().view(torch.int16).numpy().view(np.uint16).reshape(-1), ref)


def test_nf4_decode_unaligned_and_odd_blocks():
    rng = np.random.default_rng(3)
    for bs, nbytes, off in ((64, 4096, 1), (6, 3 * 1001, 0), (128, 640, 3)):
        raw = rng.integers(0, 256, nbytes + off, dtype=np.uint8)
        absmax = rng.random(nbytes * 2 // bs, dtype=np.float32) + 0.01
        pk = torch.from_numpy(raw).to(DEV)[off:]  # misaligned view -> scalar path
        out = ops().nf4_dequant(pk, torch.from_numpy(absmax).to(DEV), bs, N.NF4_CODE, (nbytes * 2,), F32)
        assert np.array_equal(out.cpu().numpy(), N.decode_f32(raw[off:], absmax, bs))


def test_nf4_decode_empty():
    out = ops().nf4_dequant(torch.empty(0, dtype=torch.uint8, device=DEV), torch.empty(0, device=DEV), 64, N.NF4_CODE,
                            (0,), BF16)
    assert out.numel() == 0


# ------------------------------------------------------------------------------------------ glue


@pytest.mark.parametrize("b,l,d", [(1, 80, 256), (2, 33, 3072), (1, 7, 384),
                                   (3, 1000, 3072)])  # more rows than CTAs: each walks rows of several images
def test_ln_mod_vs_oracle(b, l, d):
    g = torch.Generator().manual_seed(d + l)
    x = torch.randn(b, l, d, generator=g) * 3 + 0.5
    mod = torch.randn(b, 2 * d, generator=g).to(BF16)
    ref = R.mod_in(x, mod[:, None, :d].float(), mod[:, None, d:].float(), BF16)
    got = ops().ln_mod(x.to(DEV), mod[:, :d].to(DEV), mod[:, d:].to(DEV)).cpu()
    # bf16 outputs: at most one bf16 ulp apart (different fp32 summation order for mean/var)
    torch.testing.assert_close(got.float(), ref.float(), rtol=2 ** -7, atol=1e-6)


@pytest.mark.parametrize("b,lt,li", [(1, 512, 4096), (2, 33, 70), (1, 0, 64)])
def test_ln_mod_grouped_equals_separate_launches(b, lt, li):
    """The double block's txt and img LN-mods in one launch (fb_ln_mod_grouped): bit-identical to two
    fb_ln_mod launches, with a strided modulation batch and an empty stream."""
    o = ops()
    g = torch.Generator().manual_seed(lt + li)
    d = 3072
    xt = (torch.randn(b, lt, d, generator=g) * 2 - 0.3).to(DEV)
    xi = (torch.randn(b, li, d, generator=g) * 3 + 0.5).to(DEV)
    mod = torch.randn(b, 12 * d, generator=g).to(BF16).to(DEV)
    items = [(xt, mod[:, 6 * d:7 * d], mod[:, 7 * d:8 * d]), (xi, mod[:, :d], mod[:, d:2 * d])]
    got = o.ln_mod_grouped(items)
    for (x, sh, sc), gg in zip(items, got):
        assert torch.equal(gg, o.ln_mod(x, sh, sc))
    ref = R.mod_in(xi.cpu(), mod[:, None, :d].float().cpu(), mod[:, None, d:2 * d].float().cpu(), BF16)
    torch.testing.assert_close(got[1].cpu().float(), ref.float(), rtol=2 ** -7, atol=1e-6)


def test_gated_add_vs_oracle():
    g = torch.Generator().manual_seed(1)
    x = torch.randn(2, 40, 256, generator=g)
    y = (torch.randn(2, 40, 256, generator=g) * 1e5).to(BF16)
    gate = torch.randn(2, 256, generator=g).to(BF16)
    for guard in (False, True):
        ref = R.gated_add(x, gate[:, None].float(), y, guard)
        got = ops().gated_add(x.to(DEV), gate.to(DEV), y.to(DEV), guard).cpu()
        assert torch.equal(got, ref)  # one fp32 multiply and one add, as in the reference


def test_gelu_vs_torch():
    h = (torch.randn(4096, generator=torch.Generator().manual_seed(2)) * 4).to(BF16)
    ref = F.gelu(h.float(), approximate="tanh").to(BF16)
    got = ops().gelu_tanh(h.to(DEV)).cpu()
    torch.testing.assert_close(got.float(), ref.float(), rtol=2 ** -7, atol=1e-6)  # <= 1 bf16 ulp


@pytest.mark.parametrize("hd", [128, 64])
def test_qk_norm_rope_vs_oracle(hd):
    g = torch.Generator().manual_seed(hd)
    b, heads, lt, li = 2, 3, 5, 12
    seq = lt + li
    axes = (hd // 8, 7 * hd // 16, 7 * hd // 16)
    ids = torch.cat((R.text_ids(lt), torch.randint(0, 30, (li, 3), generator=g).float()), 0)
    cos, sin = R.rope_tables(ids, axes)
    tq = (torch.randn(b, lt, 3 * heads * hd, generator=g) * 2).to(BF16)
    iq = (torch.randn(b, li, 3 * heads * hd, generator=g) * 2).to(BF16)
    sc = [1 + 0.1 * torch.randn(hd, generator=g) for _ in range(4)]
    th, ih = R.split_heads(tq, heads), R.split_heads(iq, heads)
    rq = R.apply_rope(torch.cat((R.qk_rms(th[0], sc[0]), R.qk_rms(ih[0], sc[2])), 2), cos, sin).to(BF16)
    rk = R.apply_rope(torch.cat((R.qk_rms(th[1], sc[1]), R.qk_rms(ih[1], sc[3])), 2), cos, sin).to(BF16)
    rv = torch.cat((th[2], ih[2]), 2)
    q = torch.empty(b, heads, seq, hd, dtype=BF16, device=DEV)
    k, v = torch.empty_like(q), torch.empty_like(q)
    o = ops()
    o.qk_norm_rope(tq.to(DEV), heads, sc[0].to(DEV), sc[1].to(DEV), cos.to(DEV), sin.to(DEV), q, k, v, 0)
    o.qk_norm_rope(iq.to(DEV), heads, sc[2].to(DEV), sc[3].to(DEV), cos.to(DEV), sin.to(DEV), q, k, v, lt)
    assert torch.equal(v.cpu(), rv)
    torch.testing.assert_close(q.cpu().float(), rq.float(), rtol=2 ** -7, atol=1e-5)
    torch.testing.assert_close(k.cpu().float(), rk.float(), rtol=2 ** -7, atol=1e-5)


# ------------------------------------------------------------------------------------------ GEMM


def _gemm_inputs(m, n, k, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(m, k, generator=g).to(BF16)
    w = (torch.randn(n, k, generator=g) * 0.02).to(BF16)
    b = (torch.randn(n, generator=g) * 0.02).to(BF16)
    return a.to(DEV), w.to(DEV), b.to(DEV)


def _ref_lin(a, w, b):
    return (a.float() @ w.float().t() + b.float()).to(BF16)  # torch fp32 reference, rounded like F.linear


def _bf16_close(got, ref):
    """<= 1 bf16 ulp (the fp32 accumulation order differs from cuBLAS's)."""
    torch.testing.assert_close(got.float(), ref.float(), rtol=2 ** -7, atol=2 ** -7 * ref.float().abs().max().item() * 1e-3)


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (80, 768, 256), (300, 512, 3072), (4608, 3072, 3072), (77, 64, 256),
                                   (513, 9216, 3072), (64, 3072, 64)])
def test_linear_store_bf16_and_f32(m, n, k):
    o = ops()
    a, w, b = _gemm_inputs(m, n, k, m + n + k)
    ref = _ref_lin(a, w, b)
    got = o.linear(a, w, b)
    _bf16_close(got, ref)
    got32 = o.linear(a, w, b, out_dtype=F32)
    assert got32.dtype == F32 and torch.equal(got32.to(BF16), got)


def test_linear_is_deterministic():
    o = ops()
    a, w, b = _gemm_inputs(1000, 1024, 1024, 5)
    r1 = o.linear(a, w, b)
    r2 = o.linear(a, w, b)
    assert torch.equal(r1, r2)


def test_linear_gelu_epilogue():
    from selas_b200 import _lib

    o = ops()
    a, w, b = _gemm_inputs(200, 1024, 256, 9)
    out = torch.empty(200, 1024, dtype=BF16, device=DEV)
    p = o.make_linear(a, w, b, 200)
    p.out, p.ld_out = out.data_ptr(), 1024
    o.run_linears([p], _lib.FB_EPI_GELU)
    ref = F.gelu(_ref_lin(a, w, b).float(), approximate="tanh").to(BF16)
    torch.testing.assert_close(out.float(), ref.float(), rtol=2 ** -6, atol=1e-3)  # two roundings -> <= 2 ulp


@pytest.mark.parametrize("batch,d,pad,inplace", [(1, 256, 0, False), (3, 256, 0, False), (2, 288, 64, True),
                                                 (1, 544, 32, False), (2, 544, 0, True)])
def test_linear_gated_residual_grouped(batch, d, pad, inplace):
    """out = resid + gate * (x W^T + b) on grouped problems: partial row tiles, an output width that
    ends in a partial column tile (288, 544), a residual with a row stride wider than the output
    (`pad` extra columns) and the in-place update (out is the residual) of the residual stream."""
    from selas_b200 import _lib

    o = ops()
    outs, refs, probs, keep, pads = [], [], [], [], []  # keep: operands stay alive until the launch is queued
    for rows, seed in ((40, 1), (300, 2)):
        a, w, b = _gemm_inputs(batch * rows, d, 512, seed)
        xbuf = torch.randn(batch * rows, d + pad, device=DEV)
        x = xbuf[:, :d]
        mod = torch.randn(batch, 6 * d, device=DEV).to(BF16)
        gate = mod[:, 2 * d:3 * d]
        img = torch.arange(batch * rows, device=DEV) // rows
        refs.append(x + gate.float()[img] * _ref_lin(a, w, b).float())
        out = x if inplace else torch.empty(batch * rows, d, device=DEV)
        p = o.make_linear(a, w, b, rows)
        p.resid, p.ld_resid = x.data_ptr(), d + pad
        p.gate, p.gate_batch_stride = gate.data_ptr(), gate.stride(0) if batch > 1 else 0
        p.out, p.ld_out = out.data_ptr(), out.stride(0)
        probs.append(p)
        outs.append(out)
        keep += [a, w, b, xbuf, mod]
        pads.append((xbuf, xbuf[:, d:].clone()))
    o.run_linears(probs, _lib.FB_EPI_GATED_RESIDUAL)
    for got, ref in zip(outs, refs):
        torch.testing.assert_close(got, ref, rtol=1e-5, atol=2 ** -7 * 8)  # ~1 bf16 ulp of the Linear output * |gate|
    for xbuf, before in pads:
        assert torch.equal(xbuf[:, d:], before)  # columns past the output width are never written


# ------------------------------------------------------------------------------------------ attention


def _ref_attn(q, k, v):
    s = (q.float() @ k.float().transpose(-1, -2)) / math.sqrt(q.shape[-1])
    return torch.softmax(s, dim=-1) @ v.float()


@pytest.mark.parametrize("b,h,l", [(1, 2, 80), (2, 3, 257), (1, 2, 1024), (1, 1, 4608), (4, 2, 1536)])
def test_attention_vs_fp32(b, h, l):
    """Against fp32 attention on the same bf16 q, k, v, no further than the reference's own bf16 SDPA
    (torch's scaled_dot_product_attention in bf16, what selas's _attention calls, flux.py:135-138):
    rel-L2 <= 1.5 x and max-abs <= 2 x its spread from fp32, as the block tests bound the blocks."""
    g = torch.Generator().manual_seed(l)
    q, k, v = (torch.randn(b, h, l, 128, generator=g).to(BF16).to(DEV) for _ in range(3))
    q = q * 2
    got = ops().attention(q.contiguous(), k, v)  # [B, L, H*128]
    ref = _ref_attn(q, k, v).transpose(1, 2).reshape(b, l, h * 128)
    sdpa = F.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(b, l, h * 128)
    err, spread = rel_l2(got.float(), ref), rel_l2(sdpa.float(), ref)
    assert err <= 1.5 * spread, (err, spread)
    emax, smax = (got.float() - ref).abs().max().item(), (sdpa.float() - ref).abs().max().item()
    assert emax <= 2.0 * smax, (emax, smax)


def test_attention_rising_max_rescales():
    """Scores that rise far above the first KV tile's maximum in later tiles: spikes in the first and in
    the second 64-key half of later tiles, the last one in the partial last tile, for half of the
    queries only (so lanes of one warp disagree). The running reference max has to be raised (O and l
    rescaled) each time; the result must still match fp32 attention as closely as bf16 SDPA does."""
    b, h, l = 1, 2, 1000
    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(b, h, l, 128, generator=g) for _ in range(3))
    u = torch.randn(128, generator=g)
    u = u / u.norm()
    q[:, :, ::2] += 8.0 * u  # every other query leans towards u
    # tile 2 first half, tile 5 second half, tile 7 (partial) second half; each spike lies 27-31 above the
    # previous maximum in the log2 domain for the leaning queries, 4-12 for the others
    for key, beta in ((300, 40.0), (720, 80.0), (990, 120.0)):
        k[:, :, key] = beta * u
    q, k, v = (t.to(BF16).to(DEV) for t in (q, k, v))
    got = ops().attention(q.contiguous(), k.contiguous(), v.contiguous())
    ref = _ref_attn(q, k, v).transpose(1, 2).reshape(b, l, h * 128)
    sdpa = F.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(b, l, h * 128)
    assert torch.isfinite(got.float()).all()
    err, spread = rel_l2(got.float(), ref), rel_l2(sdpa.float(), ref)
    assert err <= max(1.5 * spread, 4e-3), (err, spread)
    emax, smax = (got.float() - ref).abs().max().item(), (sdpa.float() - ref).abs().max().item()
    assert emax <= max(2.0 * smax, 2e-2), (emax, smax)


def test_attention_split_and_strided_outputs():
    b, h, lt, li = 2, 2, 16, 200
    l = lt + li
    g = torch.Generator().manual_seed(7)
    q, k, v = (torch.randn(b, h, l, 128, generator=g).to(BF16).to(DEV) for _ in range(3))
    ref = _ref_attn(q, k, v).transpose(1, 2).reshape(b, l, h * 128)
    o = ops()
    a_t = torch.empty(b, lt, h * 128, dtype=BF16, device=DEV)
    a_i = torch.empty(b, li, h * 128, dtype=BF16, device=DEV)
    o.attention(q, k, v, out=a_i, split=lt, out_first=a_t)
    assert rel_l2(a_t.float(), ref[:, :lt]) < 8e-3 and rel_l2(a_i.float(), ref[:, lt:]) < 8e-3
    wide = torch.zeros(b, l, h * 128 + 512, dtype=BF16, device=DEV)
    o.attention(q, k, v, out=wide[:, :, :h * 128])
    assert rel_l2(wide[:, :, :h * 128].float(), ref) < 8e-3
    assert wide[:, :, h * 128:].abs().max().item() == 0  # nothing written past the slice


# ------------------------------------------------------------------------------------------ NF4 Linear


def _nf4_weight(n, k, seed, bs=64):
    w = (torch.randn(n, k, generator=torch.Generator().manual_seed(seed)) * 0.02).numpy()
    packed, absmax = N.encode(w, bs)
    return torch.from_numpy(packed).to(DEV), torch.from_numpy(absmax).to(DEV)


@pytest.mark.parametrize("ws_rows", [None, 256, 512])
def test_linear_nf4_matches_decode_then_linear(ws_rows):
    """fb_linear_nf4 (decode into a workspace, chunked when it is small) is bit-identical to decoding
    the weight with fb_nf4_dequant and running fb_linear_grouped on it."""
    from selas_b200 import _lib

    o = ops()
    m, n, k = 300, 1280, 512
    a, _, b = _gemm_inputs(m, n, k, 11)
    packed, absmax = _nf4_weight(n, k, 12)
    code = torch.tensor(N.NF4_CODE, device=DEV)
    w = o.nf4_dequant(packed, absmax, 64, code, (n, k), BF16)
    x = torch.randn(m, n, device=DEV)
    gate = torch.randn(1, n, device=DEV).to(BF16)
    ws = torch.empty(((ws_rows or n) * k * 2) // 2, dtype=BF16, device=DEV)
    for epi, dt in ((_lib.FB_EPI_STORE_BF16, BF16), (_lib.FB_EPI_GATED_RESIDUAL, F32), (_lib.FB_EPI_GELU, BF16)):
        ref = torch.empty(m, n, dtype=dt, device=DEV)
        got = torch.full((m, n), 7.0, dtype=dt, device=DEV)
        for out, nf4 in ((ref, False), (got, True)):
            p = o.make_linear_nf4(a, packed, absmax, code, 64, n, b, m) if nf4 else o.make_linear(a, w, b, m)
            p.out, p.ld_out = out.data_ptr(), n
            if epi == _lib.FB_EPI_GATED_RESIDUAL:
                p.resid, p.ld_resid, p.gate, p.gate_batch_stride = x.data_ptr(), n, gate.data_ptr(), 0
            if nf4:
                o.run_linear_nf4(p, epi, ws)
            else:
                o.run_linears([p], epi)
        assert torch.equal(got, ref), epi


def test_linear_nf4_qkv_epilogue_across_chunks():
    """linear1-shaped NF4 Linear (q|k|v|mlp columns) with a 256-row workspace: chunk boundaries cross
    the q/k/v/mlp sections; q/k/v and the GELU columns must equal the unchunked bf16 path."""
    from selas_b200 import _lib

    o = ops()
    heads, seq, mlp = 2, 144, 512
    m, n, k = seq, 3 * heads * 128 + mlp, 256
    a, _, b = _gemm_inputs(m, n, k, 21)
    packed, absmax = _nf4_weight(n, k, 22)
    code = torch.tensor(N.NF4_CODE, device=DEV)
    w = o.nf4_dequant(packed, absmax, 64, code, (n, k), BF16)
    g = torch.Generator().manual_seed(3)
    cos, sin = torch.rand(seq, 64, generator=g).to(DEV), torch.rand(seq, 64, generator=g).to(DEV)
    qs, ks = (1 + 0.1 * torch.randn(128, generator=g)).to(DEV), (1 + 0.1 * torch.randn(128, generator=g)).to(DEV)
    ws = torch.empty(256 * k, dtype=BF16, device=DEV)
    outs = []
    for nf4 in (False, True):
        q = torch.zeros(1, heads, seq, 128, dtype=BF16, device=DEV)
        kk, v = torch.zeros_like(q), torch.zeros_like(q)
        cat = torch.zeros(m, 256 + mlp, dtype=BF16, device=DEV)
        p = o.make_linear_nf4(a, packed, absmax, code, 64, n, b, m) if nf4 else o.make_linear(a, w, b, m)
        p.q, p.k_out, p.v, p.q_scale, p.k_scale = q.data_ptr(), kk.data_ptr(), v.data_ptr(), qs.data_ptr(), ks.data_ptr()
        p.rope_cos, p.rope_sin = cos.data_ptr(), sin.data_ptr()
        p.heads, p.head_dim, p.seq_total, p.seq_offset, p.qkv_cols = heads, 128, seq, 0, 3 * heads * 128
        p.out, p.ld_out, p.gelu_col0 = cat.data_ptr(), 256 + mlp, 256
        if nf4:
            o.run_linear_nf4(p, _lib.FB_EPI_QKV, ws)
        else:
            o.run_linears([p], _lib.FB_EPI_QKV)
        outs.append((q, kk, v, cat))
    for r, t in zip(*outs):
        assert torch.equal(r, t)
    assert outs[0][3][:, 256:].abs().sum().item() > 0


def test_linear_nf4_rejects_a_small_workspace():
    from selas_b200 import _lib

    o = ops()
    a, _, b = _gemm_inputs(64, 512, 256, 1)
    packed, absmax = _nf4_weight(512, 256, 2)
    p = o.make_linear_nf4(a, packed, absmax, torch.tensor(N.NF4_CODE, device=DEV), 64, 512, b, 64)
    out = torch.empty(64, 512, dtype=BF16, device=DEV)
    p.out, p.ld_out = out.data_ptr(), 512
    with pytest.raises(_lib.FluxB200Error, match="workspace too small"):
        o.run_linear_nf4(p, _lib.FB_EPI_STORE_BF16, torch.empty(255 * 256, dtype=BF16, device=DEV))
