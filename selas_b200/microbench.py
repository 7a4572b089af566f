"""Per-kernel microbenchmarks on one B200, timed with CUDA events on the launching stream.

    python -m selas_b200.microbench --kernel gemm --shape 4608x3072x15360 [--epi resid] [--iters 20]
    python -m selas_b200.microbench --kernel gemm --shape 4096x9216x3072+512x9216x3072 --epi qkv
    python -m selas_b200.microbench --kernel attention --shape 1x24x4608
    python -m selas_b200.microbench --kernel ln_mod --shape 4608x3072
    python -m selas_b200.microbench --kernel step_yardstick --shape 1024   # C4 step: ours vs selas's GPU paths
    python -m selas_b200.microbench --kernel nf4 --shape 3072x12288
    python -m selas_b200.microbench --suite c4          # every kernel shape of a 1024^2 FLUX step
    python -m selas_b200.microbench --suite c4_cublas   # C4 GEMMs / attention beside cuBLAS / cuDNN
    python -m selas_b200.microbench --kernel vae --shape 1x128x128     # VAE decode of a 1024^2 latent
    python -m selas_b200.microbench --kernel vae_conv --shape 1x1024x1024x128x128x3
    python -m selas_b200.microbench --kernel stepcache --shape 4096x3072   # step-cache streams (1024^2 img)
    python -m selas_b200.microbench --kernel encode --shape 3072x12288      # NF4 / int8_row encoders

Each kernel runs `--warmup` untimed launches, then `--iters` timed launches; a 256 MB buffer is
written between timed launches so memory-bound kernels read from HBM, not L2. Prints one JSON line
per case: average ms, achieved TFLOP/s (GEMM, attention) or GB/s of algorithmic bytes (memory-bound
kernels) and the fraction of the MEASURED_PEAKS.json peak (burst figures: kernels timed alone).
"""

from __future__ import annotations

import argparse
import json
import math
from pathlib import Path

import torch

from . import _lib, ops

BF16, F32 = torch.bfloat16, torch.float32
ROOT = Path(__file__).resolve().parent.parent


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm": d["hbm_gbs"], "bf16": d["bf16_tflops"], "source": "measured"}
    return {"hbm": 6650.0, "bf16": 1590.0, "source": "fallback"}


def _time(fn, warmup: int, iters: int, flush: torch.Tensor | None) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    total = 0.0
    for _ in range(iters):
        if flush is not None:
            flush.add_(1.0)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        fn()
        e1.record(s)
        e1.synchronize()
        total += e0.elapsed_time(e1)
    return total / iters


def _shape(s: str) -> list[list[int]]:
    return [[int(v) for v in part.split("x")] for part in s.split("+")]


EPI = {"bf16": _lib.FB_EPI_STORE_BF16, "f32": _lib.FB_EPI_STORE_F32, "gelu": _lib.FB_EPI_GELU,
       "resid": _lib.FB_EPI_GATED_RESIDUAL, "qkv": _lib.FB_EPI_QKV}


def bench_gemm(shapes: list[list[int]], epi: str, warmup: int, iters: int, flush) -> dict:
    dev = torch.device("cuda")
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    probs, keep = [], []
    flops = 0.0
    for (m, n, k) in shapes:
        a = torch.randn(m, k, device=dev, generator=g).to(BF16)
        w = (torch.randn(n, k, device=dev, generator=g) * 0.02).to(BF16)
        b = (torch.randn(n, device=dev, generator=g) * 0.02).to(BF16)
        p = ops.make_linear(a, w, b, m)
        keep += [a, w, b]
        if epi == "qkv":
            heads = min(24, n // 384)
            qkv_cols = 3 * heads * 128
            seq = sum(s[0] for s in shapes)
            q = torch.empty(1, heads, seq, 128, dtype=BF16, device=dev)
            kk, v = torch.empty_like(q), torch.empty_like(q)
            sc = torch.ones(128, device=dev)
            cos = torch.rand(seq, 64, device=dev)
            sin = torch.rand(seq, 64, device=dev)
            off = sum(s[0] for s in shapes[:len(probs)])
            p.q, p.k_out, p.v, p.q_scale, p.k_scale = q.data_ptr(), kk.data_ptr(), v.data_ptr(), sc.data_ptr(), sc.data_ptr()
            p.rope_cos, p.rope_sin = cos.data_ptr(), sin.data_ptr()
            p.heads, p.head_dim, p.seq_total, p.seq_offset, p.qkv_cols = heads, 128, seq, off, qkv_cols
            keep += [q, kk, v, sc, cos, sin]
            if n > qkv_cols:
                out = torch.empty(m, 3072 + (n - qkv_cols), dtype=BF16, device=dev)
                p.out, p.ld_out, p.gelu_col0 = out.data_ptr(), out.stride(0), 3072
                keep.append(out)
        else:
            out = torch.empty(m, n, dtype=F32 if epi in ("f32", "resid") else BF16, device=dev)
            p.out, p.ld_out = out.data_ptr(), n
            keep.append(out)
            if epi == "resid":
                x = torch.randn(m, n, device=dev, generator=g)
                gate = torch.randn(1, n, device=dev, generator=g).to(BF16)
                p.resid, p.ld_resid, p.gate, p.gate_batch_stride = x.data_ptr(), n, gate.data_ptr(), 0
                keep += [x, gate]
        probs.append(p)
        flops += 2.0 * m * n * k
    ms = _time(lambda: ops.run_linears(probs, EPI[epi]), warmup, iters, flush)
    tf = flops / (ms * 1e-3) / 1e12
    return {"kernel": "gemm", "epilogue": epi, "shape": shapes, "ms": ms, "tflops": tf, "frac": tf / peaks()["bf16"]}


def bench_gemm_cublas(shapes: list[list[int]], warmup: int, iters: int, flush) -> dict:
    """Yardstick only, not the product path: the same problems as torch.nn.functional.linear (cuBLAS,
    bf16 in and out, fp32 accumulation, bias added by cuBLAS's epilogue), one call per problem, which is
    what selas's UnitView.linear issues for each Linear."""
    dev = torch.device("cuda")
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    args, flops = [], 0.0
    for (m, n, k) in shapes:
        a = torch.randn(m, k, device=dev, generator=g).to(BF16)
        w = (torch.randn(n, k, device=dev, generator=g) * 0.02).to(BF16)
        b = (torch.randn(n, device=dev, generator=g) * 0.02).to(BF16)
        args.append((a, w, b))
        flops += 2.0 * m * n * k

    def fn():
        for a, w, b in args:
            torch.nn.functional.linear(a, w, b)

    ms = _time(fn, warmup, iters, flush)
    tf = flops / (ms * 1e-3) / 1e12
    return {"kernel": "gemm_cublas", "shape": shapes, "ms": ms, "tflops": tf, "frac": tf / peaks()["bf16"]}


def bench_gemm_i8(m: int, n: int, k: int, warmup: int, iters: int, flush) -> dict:
    """An int8_row Linear (selas --quant int8; weights N(0, 0.02) before quantisation) on M x K bf16
    activations, decoded inside the GEMM mainloop."""
    from . import codec

    dev = torch.device("cuda")
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    a = torch.randn(m, k, device=dev, generator=g).to(BF16)
    q, scale = codec.encode_int8_row_device(torch.randn(n, k, device=dev, generator=g) * 0.02)
    b = (torch.randn(n, device=dev, generator=g) * 0.02).to(BF16)
    out = torch.empty(m, n, dtype=BF16, device=dev)

    def run():
        p = ops.make_linear_i8(a, q, scale, b, m)
        p.out, p.ld_out = out.data_ptr(), n
        ops.run_linears([p], _lib.FB_EPI_STORE_BF16)

    ms = _time(run, warmup, iters, flush)
    tf = 2.0 * m * n * k / (ms * 1e-3) / 1e12
    nbytes = m * k * 2 + n * k + n * 4 + m * n * 2
    return {"kernel": "gemm_i8", "shape": [m, n, k], "ms": ms, "tflops": tf, "frac": tf / peaks()["bf16"],
            "gbs_algorithmic": nbytes / (ms * 1e-3) / 1e9}


def bench_gemm_f8(m: int, n: int, k: int, warmup: int, iters: int, flush) -> dict:
    """A raw-fp8 (e4m3fn) Linear on M x K bf16 activations, cast to bf16 inside the GEMM mainloop."""
    dev = torch.device("cuda")
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    a = torch.randn(m, k, device=dev, generator=g).to(BF16)
    w8 = (torch.randn(n, k, device=dev, generator=g) * 0.02).to(torch.float8_e4m3fn)
    b = (torch.randn(n, device=dev, generator=g) * 0.02).to(BF16)
    out = torch.empty(m, n, dtype=BF16, device=dev)

    def run():
        p = ops.make_linear_f8(a, w8, b, m)
        p.out, p.ld_out = out.data_ptr(), n
        ops.run_linears([p], _lib.FB_EPI_STORE_BF16)

    ms = _time(run, warmup, iters, flush)
    tf = 2.0 * m * n * k / (ms * 1e-3) / 1e12
    nbytes = m * k * 2 + n * k + m * n * 2
    return {"kernel": "gemm_f8", "shape": [m, n, k], "ms": ms, "tflops": tf, "frac": tf / peaks()["bf16"],
            "gbs_algorithmic": nbytes / (ms * 1e-3) / 1e9}


def bench_gemm_nf4(m: int, n: int, k: int, warmup: int, iters: int, flush, fused: bool = True,
                   epi: str = "bf16") -> dict:
    """C3: an NF4 Linear (blocksize 64, weights N(0, 0.02) before quantisation) on M x K bf16 activations.
    fused: the decode-in-mainloop GEMM; otherwise decode into a bf16 buffer, then the bf16 GEMM.
    epi: "bf16" stores bf16; "resid" is the gated residual (fp32 residual in, fp32 out), as the proj,
    MLP-out and linear2 Linears of a block use it; "qkv" the RMSNorm + RoPE split into q/k/v of the QKV
    Linear (n a multiple of 384, up to 24 heads; the columns past 3 x heads x 128 take the GELU store,
    as in linear1)."""
    from . import codec

    dev = torch.device("cuda")
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    a = torch.randn(m, k, device=dev, generator=g).to(BF16)
    w = torch.randn(n, k, device=dev, generator=g) * 0.02
    packed, absmax = codec.encode_device(w, 64)
    del w
    code = torch.tensor(codec.NF4_CODE, device=dev)
    b = (torch.randn(n, device=dev, generator=g) * 0.02).to(BF16)
    resid = epi == "resid"
    out = torch.empty(m, n, dtype=F32 if resid else BF16, device=dev)
    wbuf = torch.empty(n, k, dtype=BF16, device=dev)
    x = torch.randn(m, n, device=dev, generator=g) if resid else None
    gate = torch.randn(1, n, device=dev, generator=g).to(BF16) if resid else None
    if epi == "qkv":
        heads = min(24, n // 384)
        qkv_cols = 3 * heads * 128
        qb = torch.empty(1, heads, m, 128, dtype=BF16, device=dev)
        kb, vb = torch.empty_like(qb), torch.empty_like(qb)
        sc = torch.ones(128, device=dev)
        cos, sin = torch.rand(m, 64, device=dev), torch.rand(m, 64, device=dev)
        cat = torch.empty(m, 3072 + max(n - qkv_cols, 0), dtype=BF16, device=dev)

    def run():
        if fused:
            p = ops.make_linear_nf4(a, packed, absmax, code, 64, n, b, m)
        else:
            ops.nf4_dequant(packed, absmax, 64, code, (n, k), BF16, out=wbuf.view(-1))
            p = ops.make_linear(a, wbuf, b, m)
        p.out, p.ld_out = out.data_ptr(), n
        if resid:
            p.resid, p.ld_resid, p.gate, p.gate_batch_stride = x.data_ptr(), n, gate.data_ptr(), 0
        if epi == "qkv":
            p.q, p.k_out, p.v, p.q_scale, p.k_scale = qb.data_ptr(), kb.data_ptr(), vb.data_ptr(), sc.data_ptr(), sc.data_ptr()
            p.rope_cos, p.rope_sin = cos.data_ptr(), sin.data_ptr()
            p.heads, p.head_dim, p.seq_total, p.seq_offset, p.qkv_cols = heads, 128, m, 0, qkv_cols
            p.out, p.ld_out, p.gelu_col0 = cat.data_ptr(), cat.stride(0), 3072
        ops.run_linears([p], EPI[epi])

    ms = _time(run, warmup, iters, flush)
    flops = 2.0 * m * n * k
    nbytes = m * k * 2 + n * k * 0.5 + n * k / 64 * 4 + m * n * 2
    tf = flops / (ms * 1e-3) / 1e12
    return {"kernel": "gemm_nf4" if fused else "gemm_nf4_decode_then_bf16", "epilogue": epi, "shape": [m, n, k],
            "ms": ms, "tflops": tf,
            "frac": tf / peaks()["bf16"], "gbs_algorithmic": nbytes / (ms * 1e-3) / 1e9}


def bench_attention(b: int, h: int, l: int, warmup: int, iters: int, flush) -> dict:
    dev = torch.device("cuda")
    q, k, v = (torch.randn(b, h, l, 128, device=dev).to(BF16) for _ in range(3))
    out = torch.empty(b, l, h * 128, dtype=BF16, device=dev)
    ms = _time(lambda: ops.attention(q, k, v, out=out), warmup, iters, flush)
    flops = 4.0 * b * h * l * l * 128
    tf = flops / (ms * 1e-3) / 1e12
    return {"kernel": "attention", "shape": [b, h, l, 128], "ms": ms, "tflops": tf, "frac": tf / peaks()["bf16"]}


def bench_attention_cudnn(b: int, h: int, l: int, warmup: int, iters: int, flush) -> dict:
    """Yardstick only, not the product path: torch's scaled_dot_product_attention restricted to its
    cuDNN backend on the same shape and dtype, [B, H, L, 128] in and out (no token-major output)."""
    from torch.nn.attention import SDPBackend, sdpa_kernel

    dev = torch.device("cuda")
    q, k, v = (torch.randn(b, h, l, 128, device=dev).to(BF16) for _ in range(3))
    with sdpa_kernel([SDPBackend.CUDNN_ATTENTION]):
        ms = _time(lambda: torch.nn.functional.scaled_dot_product_attention(q, k, v), warmup, iters, flush)
    tf = 4.0 * b * h * l * l * 128 / (ms * 1e-3) / 1e12
    return {"kernel": "attention_cudnn", "shape": [b, h, l, 128], "ms": ms, "tflops": tf,
            "frac": tf / peaks()["bf16"]}


# ------------------------------------------------------------------------------------------ yardstick
# The GPU paths selas itself runs, restated for timing only (never on this library's product path):
# F.linear through cuBLAS, SDPA, and the seven fp32 glue segments of selas/models/flux.py:164-200,
# either eager (``Kernels()``) or each one torch.compile'd with dynamic=False, fullgraph=True
# (``Kernels(compiled=True)``, flux.py:203-232). tests/test_eager_yardstick.py checks the eager blocks
# against the oracle bit for bit on the CPU.


def _y_ln(x):
    return torch.nn.functional.layer_norm(x, (x.shape[-1],), eps=1e-6)


def _y_rms(x, scale):
    xf = x.float()
    return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * scale


def _y_rope(x, cos, sin):
    a, b = x[..., 0::2], x[..., 1::2]
    return torch.stack((a * cos - b * sin, a * sin + b * cos), dim=-1).flatten(-2)


def _y_heads(qkv, heads):
    b, l, _ = qkv.shape
    t = qkv.view(b, l, 3, heads, -1).permute(2, 0, 3, 1, 4)
    return t[0], t[1], t[2]


def _y_mod_in(x, shift, scale, dt):
    return (_y_ln(x) * (1 + scale) + shift).to(dt)


def _y_gated_add(x, g, y, guard):
    y = y.float()
    return x + g * (y.clamp(-65504.0, 65504.0) if guard else y)


def _y_gated_add_mod(x, g, y, shift, scale, dt, guard):
    x = _y_gated_add(x, g, y, guard)
    return x, _y_mod_in(x, shift, scale, dt)


def _y_qkv_double(tqkv, iqkv, tqs, tks, iqs, iks, cos, sin, heads, dt):
    tq, tk, tv = _y_heads(tqkv, heads)
    iq, ik, iv = _y_heads(iqkv, heads)
    q = _y_rope(torch.cat((_y_rms(tq, tqs), _y_rms(iq, iqs)), dim=2), cos, sin).to(dt)
    k = _y_rope(torch.cat((_y_rms(tk, tks), _y_rms(ik, iks)), dim=2), cos, sin).to(dt)
    return q, k, torch.cat((tv, iv), dim=2)


def _y_qkv_single(qkv, qs, ks, cos, sin, heads, dt):
    q, k, v = _y_heads(qkv, heads)
    return _y_rope(_y_rms(q, qs), cos, sin).to(dt), _y_rope(_y_rms(k, ks), cos, sin).to(dt), v.contiguous()


def _y_gelu(h):
    return torch.nn.functional.gelu(h, approximate="tanh")


def _y_attn_mlp(attn, mlp):
    return torch.cat((attn, _y_gelu(mlp)), dim=2)


class YardstickSegments:
    """The seven segments, eager or compiled one by one."""

    def __init__(self, compiled: bool = False):
        self.compiled = compiled
        for name, fn in (("mod_in", _y_mod_in), ("gated_add", _y_gated_add), ("gated_add_mod", _y_gated_add_mod),
                         ("qkv_double", _y_qkv_double), ("qkv_single", _y_qkv_single), ("gelu", _y_gelu),
                         ("attn_mlp", _y_attn_mlp)):
            setattr(self, name, torch.compile(fn, dynamic=False, fullgraph=True) if compiled else fn)


def _y_linear(w, x, prefix):
    return torch.nn.functional.linear(x, w.get(prefix + ".weight"), w.get(prefix + ".bias"))


def _y_attention(q, k, v):
    b, h, l, d = q.shape
    return torch.nn.functional.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(b, l, h * d)


def yardstick_double(w, img, txt, mod, cos, sin, heads, seg, dt=BF16, guard=False):
    """The double block as selas runs it on a GPU (flux.py:298-324) with segments ``seg``."""
    m = mod.float().unsqueeze(1).chunk(12, dim=-1)
    lt = txt.shape[1]
    iqkv = _y_linear(w, seg.mod_in(img, m[0], m[1], dt), "img_attn.qkv")
    tqkv = _y_linear(w, seg.mod_in(txt, m[6], m[7], dt), "txt_attn.qkv")
    q, k, v = seg.qkv_double(tqkv, iqkv, w.get("txt_attn.norm.query_norm.scale"), w.get("txt_attn.norm.key_norm.scale"),
                             w.get("img_attn.norm.query_norm.scale"), w.get("img_attn.norm.key_norm.scale"), cos, sin,
                             heads, dt)
    attn = _y_attention(q, k, v)
    outs = []
    for x, att, p, o in ((img, attn[:, lt:], "img", 0), (txt, attn[:, :lt], "txt", 6)):
        x, h = seg.gated_add_mod(x, m[o + 2], _y_linear(w, att, p + "_attn.proj"), m[o + 3], m[o + 4], dt, guard)
        h = _y_linear(w, h, p + "_mlp.0")
        outs.append(seg.gated_add(x, m[o + 5], _y_linear(w, seg.gelu(h), p + "_mlp.2"), guard))
    return outs[0], outs[1]


def yardstick_single(w, x, mod, cos, sin, heads, mlp_hidden, seg, dt=BF16, guard=False):
    """The single block as selas runs it on a GPU (flux.py:327-338)."""
    sh, sc, g = mod.float().unsqueeze(1).chunk(3, dim=-1)
    h = _y_linear(w, seg.mod_in(x, sh, sc, dt), "linear1")
    qkv, mlp = h.split([3 * x.shape[-1], mlp_hidden], dim=-1)
    q, k, v = seg.qkv_single(qkv, w.get("norm.query_norm.scale"), w.get("norm.key_norm.scale"), cos, sin, heads, dt)
    return seg.gated_add(x, g, _y_linear(w, seg.attn_mlp(_y_attention(q, k, v), mlp), "linear2"), guard)


def yardstick_step(units, arch, s, latents, cond, seg, dt=BF16):
    """One velocity prediction through the yardstick blocks (FluxRunner.step, flux.py:527-582)."""
    g = units["globals"]
    img = _y_linear(g, latents.to(dt), "img_in").float()
    txt = cond.txt
    for i in range(arch.depth_double):
        img, txt = yardstick_double(units[f"double.{i}"], img, txt, cond.mods[f"double.{i}"][s], cond.cos, cond.sin,
                                    arch.heads, seg, dt)
    x = torch.cat((txt, img), dim=1)
    for i in range(arch.depth_single):
        x = yardstick_single(units[f"single.{i}"], x, cond.mods[f"single.{i}"][s], cond.cos, cond.sin, arch.heads,
                             arch.mlp_hidden, seg, dt)
    sh, sc = cond.final_mod[s].float().unsqueeze(1).chunk(2, dim=-1)
    return _y_linear(g, seg.mod_in(x[:, cond.l_txt:], sh, sc, dt), "final_layer.linear").float()


def bench_step_yardstick(res: int, warmup: int, iters: int, flush) -> list[dict]:
    """A full FLUX-12B step (C4 at res=1024) through this library and through the yardstick restatement
    of selas's two GPU paths (eager and compiled glue), same weights, inputs and conditioning."""
    import torch._dynamo

    from .model import FluxArch, FluxStepper, random_model

    dev = torch.device("cuda")
    a = FluxArch()
    units = random_model(a, dev, seed=0, std=0.02)
    side, lt = res // 16, 512
    g = torch.Generator().manual_seed(1000)
    txt, pooled = torch.randn(1, lt, a.context_dim, generator=g), torch.randn(1, a.vec_dim, generator=g)
    ids = torch.zeros(side, side, 3)
    ids[..., 1], ids[..., 2] = torch.arange(side)[:, None], torch.arange(side)[None, :]
    sig = [1.0 - i / 28 for i in range(29)]
    st = FluxStepper(units, a)
    cond = st.prepare(sig, 3.5, pooled.to(dev), txt.to(dev), ids.reshape(-1, 3).to(dev), torch.zeros(lt, 3, device=dev))
    for n in [n for n in units if n.endswith(".mod")]:
        del units[n]
    x = torch.randn(1, side * side, 64, generator=g).to(dev)
    l = side * side + lt
    flops = 57 * (2.0 * l * (4 * a.hidden ** 2 + 2 * a.hidden * a.mlp_hidden) + 4.0 * l * l * a.hidden)
    torch._dynamo.config.cache_size_limit = max(torch._dynamo.config.cache_size_limit, 64)
    out = []
    with torch.no_grad():
        for name, fn in (("step_b200", lambda: st.step(5, x, cond)),
                         ("step_selas_eager_yardstick", lambda: yardstick_step(units, a, 5, x, cond, YardstickSegments(False))),
                         ("step_selas_compiled_yardstick", (lambda seg: lambda: yardstick_step(units, a, 5, x, cond, seg))(
                             YardstickSegments(True)))):
            ms = _time(fn, warmup, iters, flush)
            out.append({"kernel": name, "shape": [1, lt, side * side, a.hidden], "ms": ms,
                        "tflops": flops / (ms * 1e-3) / 1e12, "frac": flops / (ms * 1e-3) / 1e12 / peaks()["bf16"]})
    return out


def bench_block(lt: int, li: int, warmup: int, iters: int, flush) -> list[dict]:
    """The C2 double and single block through this library's block API, and the double block as eager
    cuBLAS / SDPA calls (the GPU path selas runs by default) on the same weights, as a yardstick."""
    from . import flux as B
    from .model import FluxArch, random_unit, rope_tables

    dev = torch.device("cuda")
    a = FluxArch()
    d, heads = a.hidden, a.heads
    g = torch.Generator(device=dev).manual_seed(0)
    wd = random_unit(a, "double", g, dev)
    ws = random_unit(a, "single", g, dev)
    img = torch.randn(1, li, d, device=dev)
    txt = torch.randn(1, lt, d, device=dev)
    mod_d = torch.randn(1, 12 * d, device=dev).to(BF16)
    mod_s = torch.randn(1, 3 * d, device=dev).to(BF16)
    side = int(round((li * 4) ** 0.5))  # tokens = (side/2)^2 for a side x side image at 8x VAE + 2x2 patches
    ids = torch.zeros(lt + li, 3, device=dev)
    ids[lt:, 1] = torch.arange(li, device=dev).div(side // 2, rounding_mode="floor").float()
    ids[lt:, 2] = torch.arange(li, device=dev).remainder(side // 2).float()
    cos, sin = rope_tables(ids, a.axes_dim, a.theta)
    x = torch.cat([txt, img], 1)
    flops = 2.0 * (lt + li) * (4 * d * d + 2 * d * a.mlp_hidden) + 4.0 * (lt + li) ** 2 * d
    out = []
    for name, fn in (("double_block", lambda: B.double_block(wd, img, txt, mod_d, cos, sin, a, BF16, False)),
                     ("single_block", lambda: B.single_block(ws, x, mod_s, cos, sin, a, BF16, False)),
                     ("double_block_eager_torch", lambda: yardstick_double(wd, img, txt, mod_d, cos, sin, heads,
                                                                           YardstickSegments(False)))):
        ms = _time(fn, warmup, iters, flush)
        tf = flops / (ms * 1e-3) / 1e12
        out.append({"kernel": name, "shape": [1, lt, li, d], "ms": ms, "tflops": tf, "frac": tf / peaks()["bf16"]})
    return out


def bench_ln_mod(rows: int, d: int, warmup: int, iters: int, flush) -> dict:
    dev = torch.device("cuda")
    x = torch.randn(1, rows, d, device=dev)
    mod = torch.randn(1, 2 * d, device=dev).to(BF16)
    out = torch.empty(1, rows, d, dtype=BF16, device=dev)
    ms = _time(lambda: ops.ln_mod(x, mod[:, :d], mod[:, d:], out=out), warmup, iters, flush)
    nbytes = rows * d * 6 + 4 * d
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {"kernel": "ln_mod", "shape": [rows, d], "ms": ms, "gbs": gbs, "frac": gbs / peaks()["hbm"]}


def bench_nf4(n: int, k: int, warmup: int, iters: int, flush) -> dict:
    dev = torch.device("cuda")
    packed = torch.randint(0, 256, (n * k // 2,), dtype=torch.uint8, device=dev)
    absmax = torch.rand(n * k // 64, device=dev) + 0.01
    out = torch.empty(n * k, dtype=BF16, device=dev)
    code = (-1.0, -0.6962, -0.5251, -0.3949, -0.2844, -0.1848, -0.0911, 0.0, 0.0796, 0.1609, 0.2461, 0.3379, 0.4407,
            0.5626, 0.7230, 1.0)
    code_t = torch.tensor(code, device=dev)
    ms = _time(lambda: ops.nf4_dequant(packed, absmax, 64, code_t, (n, k), BF16, out=out), warmup, iters, flush)
    nbytes = n * k * (0.5 + 2) + n * k / 64 * 4
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {"kernel": "nf4_dequant", "shape": [n, k], "ms": ms, "gbs": gbs, "frac": gbs / peaks()["hbm"]}


C4_SUITE = [
    ("gemm", "4096x9216x3072+512x9216x3072", "qkv"),
    ("gemm", "4096x3072x3072+512x3072x3072", "resid"),
    ("gemm", "4096x12288x3072+512x12288x3072", "gelu"),
    ("gemm", "4096x3072x12288+512x3072x12288", "resid"),
    ("gemm", "4608x21504x3072", "qkv"),
    ("gemm", "4608x3072x15360", "resid"),
    ("gemm", "4096x64x3072", "f32"),
    ("attention", "1x24x4608", None),
    ("ln_mod", "4608x3072", None),
    ("nf4", "3072x12288", None),
]


def bench_vae(b: int, h: int, w: int, warmup: int, iters: int, flush) -> dict:
    """The FLUX VAE decoder (random weights, FLUX's shape) on a [b, 16, h, w] latent, and the share of
    its time in the tf32 convolutions (CUDA events per launch, selas_b200.profile)."""
    from . import profile as prof
    from .vae import VaeConfig, VaeDecoder, random_weights

    dec = VaeDecoder(random_weights(VaeConfig(), "cuda"), VaeConfig())
    z = torch.randn(b, 16, h, w, device="cuda")
    ms = _time(lambda: dec.decode(z), warmup, iters, flush)
    prof.enable()
    dec.decode(z)
    st = prof.collect()
    prof.disable()
    conv = st.get("vae_conv", {"flops": 0.0, "ms": 0.0, "launches": 0})
    parts = {k: v for k, v in st.items() if k != "vae_conv"}
    glue = {"ms": sum(v["ms"] for v in parts.values()), "bytes": sum(v["bytes"] for v in parts.values())}
    pk = peaks()
    tf32_peak = pk["bf16"] / 2  # tf32 tensor-core rate: half the bf16 rate (dense)
    tf = conv["flops"] / (conv["ms"] * 1e-3) / 1e12 if conv["ms"] else 0.0
    return {"kernel": "vae_decode", "shape": f"{b}x16x{h}x{w} -> {b}x3x{8 * h}x{8 * w}", "ms": ms,
            "conv_ms": conv["ms"], "conv_launches": conv["launches"], "conv_tflop": conv["flops"] / 1e12,
            "conv_tflops": tf, "conv_frac_of_tf32_peak": tf / tf32_peak, "glue_ms": glue["ms"],
            "glue_gbs": glue["bytes"] / (glue["ms"] * 1e-3) / 1e9 if glue["ms"] else None,
            "parts": {k: {"ms": v["ms"], "launches": v["launches"],
                          "gbs": v["bytes"] / (v["ms"] * 1e-3) / 1e9 if v["ms"] else None} for k, v in parts.items()},
            "tf32_peak": tf32_peak, "peak_source": f"{pk['source']} bf16 burst / 2"}


def bench_vae_out(b: int, h: int, w: int, warmup: int, iters: int, flush) -> list[dict]:
    """The decoder's norm_out + conv_out (128 -> 3 channels): the fused kernel against GroupNorm then the
    tensor-core conv."""
    from .vae import _rows, conv_raw

    dev = torch.device("cuda")
    c = 128
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(b, h, w, c, device=dev, generator=g)
    gamma, beta = torch.ones(c, device=dev), torch.zeros(c, device=dev)
    wr = _rows(torch.randn(3, c, 3, 3, device=dev, generator=g) * 0.03)
    bias = torch.zeros(3, device=dev)
    work = torch.empty(_lib.lib().fb_vae_group_norm_work_doubles(b), dtype=torch.float64, device=dev)
    out = torch.empty(b, 3, h, w, device=dev)
    t = torch.empty_like(x)

    def fused():
        _lib.check(_lib.lib().fb_vae_norm_out_conv(x.data_ptr(), b, h, w, c, gamma.data_ptr(), beta.data_ptr(), 1e-6,
                                                   wr.data_ptr(), bias.data_ptr(), 3, out.data_ptr(),
                                                   work.data_ptr(), ops._stream()), "norm_out_conv")

    def two():
        _lib.check(_lib.lib().fb_vae_group_norm(x.data_ptr(), c, b, h * w, c, gamma.data_ptr(), beta.data_ptr(), 1e-6,
                                                1, 1, t.data_ptr(), c, work.data_ptr(), ops._stream()), "gn")
        conv_raw(t, c, wr, 3, 3, bias, None, out, 3, _lib.FB_VAE_OUT_NCHW_CLAMP, b, h, w)

    flops = 2.0 * b * h * w * 3 * 9 * c
    res = []
    for name, fn in (("vae_norm_out_conv_fused", fused), ("vae_norm_out_then_conv", two)):
        ms = _time(fn, warmup, iters, flush)
        res.append({"kernel": name, "shape": [b, h, w, c], "ms": ms, "gbs": b * h * w * c * 4 / (ms * 1e-3) / 1e9,
                    "tflops": flops / (ms * 1e-3) / 1e12})
    return res


def bench_vae_conv(b: int, h: int, w: int, cin: int, cout: int, k: int, warmup: int, iters: int, flush) -> dict:
    from .vae import _rows, conv_raw

    x = torch.randn(b, h, w, cin, device="cuda")
    wt = _rows(torch.randn(cout, cin, k, k, device="cuda") * (1.0 / (cin * k * k)) ** 0.5)
    bias = torch.zeros(cout, device="cuda")
    out = torch.empty(b, h, w, cout, device="cuda")
    ms = _time(lambda: conv_raw(x, cin, wt, cout, k, bias, None, out, cout, 0, b, h, w), warmup, iters, flush)
    flops = 2.0 * b * h * w * cout * cin * k * k
    tf = flops / (ms * 1e-3) / 1e12
    pk = peaks()
    return {"kernel": "vae_conv", "shape": f"{b}x{h}x{w}x{cin}->{cout} k{k}", "ms": ms, "tflops": tf,
            "frac_of_tf32_peak": tf / (pk["bf16"] / 2), "peak_source": f"{pk['source']} bf16 burst / 2"}


def bench_stepcache(rows: int, d: int, warmup: int, iters: int, flush) -> list[dict]:
    """The step-cache streams over a [rows, d] fp32 hidden state: probe distance (reads x, x_in, ref;
    writes the residual), prediction + add (reads x, r1, r0 in bf16; writes fp32), residual capture."""
    dev = torch.device("cuda")
    x, x_in, ref = (torch.randn(rows, d, device=dev) for _ in range(3))
    resid = torch.empty_like(x)
    r1, r0 = torch.randn(rows, d, device=dev).to(BF16), torch.randn(rows, d, device=dev).to(BF16)
    out = torch.empty_like(x)
    n = rows * d
    hbm = peaks()["hbm"]
    cases = [("probe_distance", lambda: ops.probe_distance(x, x_in, ref, resid), 16 * n),
             ("residual_predict_bf16", lambda: ops.residual_predict(x, r1, r0, -0.5, out), 12 * n),
             ("residual_diff_bf16", lambda: ops.residual_diff(x, x_in, BF16), 10 * n)]
    res = []
    for name, fn, nbytes in cases:
        ms = _time(fn, warmup, iters, flush)
        gbs = nbytes / (ms * 1e-3) / 1e9
        res.append({"kernel": name, "shape": [rows, d], "ms": ms, "gbs": gbs, "frac": gbs / hbm})
    return res


def bench_encode(n: int, k: int, warmup: int, iters: int, flush) -> list[dict]:
    """The weight encoders on an [n, k] bf16 weight: NF4 (reads 2 B, writes 0.5 B + absmax per value) and
    int8_row (reads 2 B twice: absmax pass and quantise pass, writes 1 B)."""
    from . import codec

    w = (torch.randn(n, k, device="cuda") * 0.02).to(BF16)
    hbm = peaks()["hbm"]
    res = []
    for name, fn, nbytes in (("nf4_encode", lambda: codec.encode_device(w, 64), n * k * (2 + 0.5 + 4 / 64)),
                             ("int8_row_encode", lambda: codec.encode_int8_row_device(w), n * k * (2 + 1))):
        ms = _time(fn, warmup, iters, flush)
        gbs = nbytes / (ms * 1e-3) / 1e9
        res.append({"kernel": name, "shape": [n, k], "ms": ms, "gbs": gbs, "frac": gbs / hbm})
    return res


def run(kernel: str, shape: str, epi: str | None, warmup: int, iters: int, flush) -> dict:
    s = _shape(shape)
    if kernel == "gemm":
        return bench_gemm(s, epi or "bf16", warmup, iters, flush)
    if kernel == "gemm_cublas":
        return bench_gemm_cublas(s, warmup, iters, flush)
    if kernel == "gemm_nf4":
        return bench_gemm_nf4(*s[0], warmup, iters, flush, fused=True, epi=epi or "bf16")
    if kernel == "gemm_f8":
        return bench_gemm_f8(*s[0], warmup, iters, flush)
    if kernel == "gemm_i8":
        return bench_gemm_i8(*s[0], warmup, iters, flush)
    if kernel == "gemm_nf4_decode":
        return bench_gemm_nf4(*s[0], warmup, iters, flush, fused=False)
    if kernel == "attention":
        return bench_attention(*s[0], warmup, iters, flush)
    if kernel == "attention_cudnn":
        return bench_attention_cudnn(*s[0], warmup, iters, flush)
    if kernel == "block":
        return bench_block(*s[0], warmup, iters, flush)
    if kernel == "ln_mod":
        return bench_ln_mod(*s[0], warmup, iters, flush)
    if kernel == "step_yardstick":
        return bench_step_yardstick(*s[0], warmup, iters, flush)
    if kernel == "nf4":
        return bench_nf4(*s[0], warmup, iters, flush)
    if kernel == "vae":
        return bench_vae(*s[0], warmup, iters, flush)
    if kernel == "vae_out":
        return bench_vae_out(*s[0], warmup, iters, flush)
    if kernel == "vae_conv":
        return bench_vae_conv(*s[0], warmup, iters, flush)
    if kernel == "stepcache":
        return bench_stepcache(*s[0], warmup, iters, flush)
    if kernel == "encode":
        return bench_encode(*s[0], warmup, iters, flush)
    raise SystemExit(f"unknown kernel {kernel}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel", default="gemm")
    ap.add_argument("--shape", default="4608x3072x15360")
    ap.add_argument("--epi", default=None)
    ap.add_argument("--suite", default=None, choices=[None, "c4", "c4_cublas"])
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--no-flush", action="store_true")
    args = ap.parse_args()
    _lib.lib()
    flush = None if args.no_flush else torch.empty(64 * 2 ** 20, device="cuda")
    if args.suite == "c4":
        cases = C4_SUITE
    elif args.suite == "c4_cublas":  # each C4 GEMM shape on this library's kernel, then on cuBLAS
        cases = [c for g_ in C4_SUITE if g_[0] == "gemm" for c in (g_, ("gemm_cublas", g_[1], None))]
        cases += [("attention", "1x24x4608", None), ("attention_cudnn", "1x24x4608", None),
                  ("attention", "4x24x1536", None), ("attention_cudnn", "4x24x1536", None)]
    else:
        cases = [(args.kernel, args.shape, args.epi)]
    for kernel, shape, epi in cases:
        r = run(kernel, shape, epi, args.warmup, args.iters, flush)
        for line in r if isinstance(r, list) else [r]:
            print(json.dumps(line), flush=True)
    torch.cuda.synchronize()
    _lib.raise_on_device_error()


if __name__ == "__main__":
    main()
