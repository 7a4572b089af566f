"""FLUX blocks on the B200 kernels, behind selas's block API.

``double_block``, ``single_block`` and ``final_layer`` have the signatures of
``selas/models/flux.py:300``, ``:327`` and ``:341``; ``B200Kernels`` has the attributes of
``selas.models.flux.Kernels`` (``flux.py:206-212``: ``compiled`` plus the seven segments) and, in
addition, the three block functions, so a runner can dispatch whole blocks to it.

Per double block (B images, Lt text + Li image tokens) the fused path launches seven kernels:
  ln_mod(img), ln_mod(txt)                      LayerNorm + adaLN shift/scale -> bf16
  QKV Linear (txt + img in one launch)          epilogue: bias, QK-RMSNorm, RoPE, heads -> q/k/v [B,H,L,128]
  attention                                     writes the txt rows and the img rows to per-stream buffers
  proj Linear (txt + img)                       epilogue: fp32 gated residual -> img1 / txt1
  ln_mod(img1), ln_mod(txt1)
  MLP-in Linear (txt + img)                     epilogue: GELU-tanh -> bf16
  MLP-out Linear (txt + img)                    epilogue: fp32 gated residual -> img2 / txt2
Per single block: ln_mod, linear1 (epilogue: QKV part -> q/k/v, MLP part -> GELU into the right-hand
columns of linear2's input), attention (into the left-hand columns), linear2 (gated residual).

Weights come from any object with selas's ``UnitView`` interface (``store.py:242-293``): ``get(name,
dtype)`` for raw tensors (a zero-copy view when stored in bf16) and, for NF4 tensors,
``codec(name)``, ``parts(name)`` and ``spec.tensors[name]``. NF4 weights (blocksize 64, K % 256 == 0)
run through the fused NF4 GEMM, which decodes the packed bytes bit-exactly inside its mainloop and never
writes a bf16 weight; other NF4 layouts are decoded by the NF4 kernel into a bf16 temporary per Linear
(selas's own JIT-decode point, ``store.py:265-281``).

Inputs are never modified; every output is a new tensor from torch's caching allocator.
"""

from __future__ import annotations

import torch

from . import _lib, ops
from ._lib import FluxB200Error

BF16, F32 = torch.bfloat16, torch.float32


# ------------------------------------------------------------------------------------------ weights


def _has(w, name: str) -> bool:
    if hasattr(w, "has"):
        return bool(w.has(name))
    shapes = getattr(w, "shapes", None)  # selas's _ShapeOnly stand-in (flux.py:263-273)
    if shapes is not None:
        return name in shapes
    return name in getattr(w, "spec").tensors


def weight(w, name: str) -> torch.Tensor:
    """The [N, K] bf16 weight of one Linear, decoding NF4 on the device when stored that way."""
    codec = w.codec(name) if hasattr(w, "codec") and hasattr(w, "spec") else "raw"
    if codec == "nf4":
        ts = w.spec.tensors[name]
        parts = w.parts(name)
        return ops.nf4_dequant(parts["packed"], parts["absmax"], int(ts.meta["blocksize"]), ts.meta["code"],
                               tuple(ts.shape), BF16)
    if codec == "int8_row":
        raise FluxB200Error(f"{name}: int8_row weights run only through the decoding GEMM (K a multiple of 64)")
    if codec != "raw":
        raise FluxB200Error(f"{name}: codec {codec!r} is not supported by the B200 blocks (raw bf16, nf4 and "
                            "int8_row are)")
    t = w.get(name, BF16)
    if t.stride(-1) != 1:
        t = t.contiguous()
    return t


def bias(w, prefix: str) -> torch.Tensor | None:
    name = prefix + ".bias"
    return w.get(name, BF16).contiguous() if _has(w, name) else None


def norm_scale(w, name: str) -> torch.Tensor:
    return w.get(name, F32).contiguous()


# ------------------------------------------------------------------------------------------ helpers


def _check_dtype(dt) -> None:
    if dt != BF16:
        raise FluxB200Error(f"the B200 blocks compute in bfloat16 (got {dt}); use selas's eager path for {dt}")


def _bf16_rows(mod: torch.Tensor) -> torch.Tensor:
    mod = mod.reshape(mod.shape[0], -1)
    if mod.dtype != BF16:
        mod = mod.to(BF16)
    return mod.contiguous()


def _f32(x: torch.Tensor) -> torch.Tensor:
    if x.dtype != F32:
        x = x.float()
    return x.contiguous()


def _operands(w, prefix: str, keep: list) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Weight and bias of one Linear, kept alive in ``keep`` until the launch that reads them is queued
    (an NF4 weight is a fresh temporary that the caching allocator could otherwise hand out again)."""
    wt, bt = weight(w, prefix + ".weight"), bias(w, prefix)
    keep += [wt, bt]
    return wt, bt


_CODE_CACHE: dict = {}


def _nf4_parts(w, name: str):
    """(packed, absmax, code tensor, shape) when ``name`` is an NF4 weight the fused decode GEMM takes
    (blocksize 64, K % 256 == 0, 16-byte aligned parts), else None."""
    if not (hasattr(w, "codec") and hasattr(w, "spec")) or w.codec(name) != "nf4":
        return None
    ts = w.spec.tensors[name]
    n, k = int(ts.shape[0]), int(ts.shape[-1])
    if int(ts.meta["blocksize"]) != 64 or k % 256:
        return None
    parts = w.parts(name)
    if parts["packed"].data_ptr() % 16 or parts["absmax"].data_ptr() % 16:
        return None
    dev = parts["packed"].device
    key = (tuple(float(c) for c in ts.meta["code"]), str(dev))
    code = _CODE_CACHE.get(key)
    if code is None:
        code = torch.tensor(key[0], dtype=F32, device=dev)
        _CODE_CACHE[key] = code
    return parts["packed"], parts["absmax"], code, (n, k)


def _int8_parts(w, name: str):
    """(q, scale) when ``name`` is an int8_row weight the decoding GEMM takes (K % 64 == 0, 16-byte
    aligned q), else None."""
    if not (hasattr(w, "codec") and hasattr(w, "spec")) or w.codec(name) != "int8_row":
        return None
    parts = w.parts(name)
    q, scale = parts["q"], parts["scale"]
    if q.dim() != 2 or q.shape[1] % 64 or q.data_ptr() % 16:
        return None
    return q, scale.float().contiguous()


def _fp8_weight(w, name: str):
    """The raw fp8 [N, K] weight when ``name`` is stored that way and the decoding GEMM takes it
    (K % 64 == 0, 16-byte aligned), else None."""
    if not (hasattr(w, "codec") and hasattr(w, "parts")) or w.codec(name) != "raw":
        return None
    t = w.parts(name).get("data")
    if t is None or t.dtype not in ops.FP8_DTYPES or t.dim() != 2 or t.shape[1] % 64 or t.data_ptr() % 16:
        return None
    return t.contiguous()


def _problem(w, prefix: str, a: torch.Tensor, rows: int, keep: list) -> _lib.FbLinear:
    """The fb_linear of one Linear of unit ``w`` on activations ``a``: NF4, int8_row and raw fp8 weights go
    to the fused decode GEMM (stored bytes read in the mainloop, no bf16 weight in memory); raw bf16
    weights, and layouts that kernel does not take, to the bf16 GEMM."""
    f8 = _fp8_weight(w, prefix + ".weight")
    if f8 is not None:
        bt = bias(w, prefix)
        keep += [f8, bt]
        return ops.make_linear_f8(a, f8, bt, rows)
    i8 = _int8_parts(w, prefix + ".weight")
    if i8 is not None:
        q, scale = i8
        bt = bias(w, prefix)
        keep += [q, scale, bt]
        return ops.make_linear_i8(a, q, scale, bt, rows)
    nf4 = _nf4_parts(w, prefix + ".weight")
    if nf4 is not None:
        packed, absmax, code, (n, _) = nf4
        bt = bias(w, prefix)
        keep += [packed, absmax, code, bt]
        return ops.make_linear_nf4(a, packed.reshape(-1), absmax.reshape(-1), code, 64, n, bt, rows)
    return ops.make_linear(a, *_operands(w, prefix, keep), rows)


def _run(problems: list, epilogue: int) -> None:
    """One grouped launch when every problem has the same weight kind, else one launch each."""
    kinds = {(bool(p.w_nf4), bool(p.w_i8), bool(p.w_f8), int(p.w_f8_e5m2)) for p in problems}
    if len(kinds) == 1:
        ops.run_linears(problems, epilogue)
    else:
        for p in problems:
            ops.run_linears([p], epilogue)


def _gate(p: _lib.FbLinear, g: torch.Tensor) -> None:
    p.gate = g.data_ptr()
    p.gate_batch_stride = g.stride(0) if g.shape[0] > 1 else 0


def _qkv_fields(p, q, k, v, qs, ks, cos, sin, heads, hd, seq_total, seq_offset, qkv_cols):
    p.q, p.k_out, p.v = q.data_ptr(), k.data_ptr(), v.data_ptr()
    p.q_scale, p.k_scale = qs.data_ptr(), ks.data_ptr()
    p.rope_cos, p.rope_sin = cos.data_ptr(), sin.data_ptr()
    p.heads, p.head_dim, p.seq_total, p.seq_offset, p.qkv_cols = heads, hd, seq_total, seq_offset, qkv_cols


def _rope(cos: torch.Tensor, sin: torch.Tensor, length: int, hd: int):
    cos, sin = cos.float().contiguous(), sin.float().contiguous()
    if tuple(cos.shape) != (length, hd // 2) or tuple(sin.shape) != (length, hd // 2):
        raise FluxB200Error(f"RoPE tables must be [{length}, {hd // 2}], got {tuple(cos.shape)}")
    return cos, sin


def _p2p(sp, b: int, seq: int) -> bool:
    """Whether ``sp`` exchanges through peer memory (sp.UlyssesP2P), checking its buffers fit this block."""
    if sp is None or not getattr(sp, "p2p", False):
        return False
    if b != 1 or seq != sp.ll:
        raise FluxB200Error(f"UlyssesP2P buffers hold one image of {sp.ll} local tokens, got batch {b} x {seq}")
    return True


# ------------------------------------------------------------------------------------------ blocks


@torch.no_grad()
def double_block(w, img, txt, mod, cos, sin, cfg, dt, guard: bool, k=None, sp=None):
    """img [B, Li, D] fp32, txt [B, Lt, D] fp32, mod [B, 12D] (img 6D | txt 6D) -> (img, txt) fp32
    (selas/models/flux.py:300-324). With ``sp`` (a ``selas_b200.sp.Ulysses``), img/txt/cos/sin are this
    rank's tokens and attention runs over the whole sequence of the group; with a ``UlyssesP2P`` the QKV
    epilogue and the attention kernel store straight into the peers' buffers (no all-to-all)."""
    _check_dtype(dt)
    img, txt = _f32(img), _f32(txt)
    b, li, d = img.shape
    lt = txt.shape[1]
    seq = li + lt
    heads = cfg.heads
    hd = d // heads
    dev = img.device
    mod = _bf16_rows(mod)
    m = [mod[:, i * d:(i + 1) * d] for i in range(12)]  # img: sh1 sc1 g1 sh2 sc2 g2 | txt: same
    cos, sin = _rope(cos, sin, seq, hd)
    streams = [s for s in (("txt", txt, lt, 0, m[6:]), ("img", img, li, lt, m[:6])) if s[2] > 0]
    p2p = _p2p(sp, b, seq)

    # LayerNorm + modulation, then QKV with RMSNorm/RoPE/head split in the epilogue.
    if p2p:
        q = kk = v = sp.qkv[0]  # the epilogue stores into the head-group owners' buffers instead
    else:
        q, kk, v = torch.empty(3, b, heads, seq, hd, dtype=BF16, device=dev)  # one buffer (see sp.Ulysses)
    probs = []
    keep = []
    xms = ops.ln_mod_grouped([(x, mm[0], mm[1]) for _, x, _, _, mm in streams])
    for (name, x, rows, off, mm), xm in zip(streams, xms):
        p = _problem(w, f"{name}_attn.qkv", xm.view(b * rows, d), rows, keep)
        qs = norm_scale(w, f"{name}_attn.norm.query_norm.scale")
        ks = norm_scale(w, f"{name}_attn.norm.key_norm.scale")
        _qkv_fields(p, q, kk, v, qs, ks, cos, sin, heads, hd, seq, off, 3 * d)
        if p2p:
            sp.qkv_fields(p)
        probs.append(p)
        keep += [xm, qs, ks]
    _run(probs, _lib.FB_EPI_QKV)

    # Joint attention; the txt rows and the img rows land in separate buffers.
    if p2p:
        sp.barrier()
        sp.attention_into(sp.att_peers, d)
        sp.barrier()
        attn = {"txt": sp.att[:lt].view(1, lt, d), "img": sp.att[lt:].view(1, li, d)}
    else:
        a_txt = torch.empty(b, lt, d, dtype=BF16, device=dev)
        a_img = torch.empty(b, li, d, dtype=BF16, device=dev)
        if sp is not None:
            sp.attention(q, kk, v, out=a_img, split=lt, out_first=a_txt)
        elif lt and li:
            ops.attention(q, kk, v, out=a_img, split=lt, out_first=a_txt)
        else:
            ops.attention(q, kk, v, out=a_img if li else a_txt)
        attn = {"txt": a_txt, "img": a_img}

    # proj + gated residual
    out1 = {"txt": torch.empty_like(txt), "img": torch.empty_like(img)}
    probs = []
    for name, x, rows, off, mm in streams:
        p = _problem(w, f"{name}_attn.proj", attn[name].view(b * rows, d), rows, keep)
        p.resid, p.ld_resid = x.data_ptr(), d
        _gate(p, mm[2])
        p.out, p.ld_out, p.guard = out1[name].data_ptr(), d, int(bool(guard))
        probs.append(p)
    _run(probs, _lib.FB_EPI_GATED_RESIDUAL)

    # LayerNorm + modulation, MLP-in with GELU in the epilogue
    mlp = cfg.mlp_hidden
    hidden = {}
    probs = []
    hms = ops.ln_mod_grouped([(out1[name], mm[3], mm[4]) for name, _, _, _, mm in streams])
    for (name, x, rows, off, mm), hm in zip(streams, hms):
        hidden[name] = torch.empty(b * rows, mlp, dtype=BF16, device=dev)
        p = _problem(w, f"{name}_mlp.0", hm.view(b * rows, d), rows, keep)
        p.out, p.ld_out = hidden[name].data_ptr(), mlp
        probs.append(p)
        keep.append(hm)
    _run(probs, _lib.FB_EPI_GELU)

    # MLP-out + gated residual
    out2 = {"txt": torch.empty_like(txt), "img": torch.empty_like(img)}
    probs = []
    for name, x, rows, off, mm in streams:
        p = _problem(w, f"{name}_mlp.2", hidden[name], rows, keep)
        p.resid, p.ld_resid = out1[name].data_ptr(), d
        _gate(p, mm[5])
        p.out, p.ld_out, p.guard = out2[name].data_ptr(), d, int(bool(guard))
        probs.append(p)
    _run(probs, _lib.FB_EPI_GATED_RESIDUAL)
    del keep
    return out2["img"], out2["txt"]


@torch.no_grad()
def single_block(w, x, mod, cos, sin, cfg, dt, guard: bool, k=None, sp=None):
    """x [B, Lt+Li, D] fp32, mod [B, 3D] -> x fp32 (selas/models/flux.py:327-338). With ``sp``, x and
    cos/sin are this rank's tokens (its txt, then its img) and attention spans the group."""
    _check_dtype(dt)
    x = _f32(x)
    b, seq, d = x.shape
    heads = cfg.heads
    hd = d // heads
    mlp = cfg.mlp_hidden
    dev = x.device
    mod = _bf16_rows(mod)
    sh, sc, g = mod[:, :d], mod[:, d:2 * d], mod[:, 2 * d:3 * d]
    cos, sin = _rope(cos, sin, seq, hd)

    p2p = _p2p(sp, b, seq)

    h = ops.ln_mod(x, sh, sc)
    if p2p:
        cat = sp.cat  # the peers' attention kernels fill its first d columns
        q = kk = v = sp.qkv[0]
    else:
        cat = torch.empty(b * seq, d + mlp, dtype=BF16, device=dev)  # linear2 input: [attn | gelu(mlp)]
        q, kk, v = torch.empty(3, b, heads, seq, hd, dtype=BF16, device=dev)  # one buffer (see sp.Ulysses)
    qs, ks = norm_scale(w, "norm.query_norm.scale"), norm_scale(w, "norm.key_norm.scale")
    keep: list = []
    p = _problem(w, "linear1", h.view(b * seq, d), seq, keep)
    _qkv_fields(p, q, kk, v, qs, ks, cos, sin, heads, hd, seq, 0, 3 * d)
    if p2p:
        sp.qkv_fields(p)
    p.out, p.ld_out, p.gelu_col0 = cat.data_ptr(), d + mlp, d
    _run([p], _lib.FB_EPI_QKV)

    if p2p:
        sp.barrier()
        sp.attention_into(sp.cat_peers, d + mlp)
        sp.barrier()
    elif sp is not None:
        sp.attention(q, kk, v, out=cat.view(b, seq, d + mlp)[:, :, :d])
    else:
        ops.attention(q, kk, v, out=cat.view(b, seq, d + mlp)[:, :, :d])

    out = torch.empty_like(x)
    p = _problem(w, "linear2", cat, seq, keep)
    p.resid, p.ld_resid = x.data_ptr(), d
    _gate(p, g)
    p.out, p.ld_out, p.guard = out.data_ptr(), d, int(bool(guard))
    _run([p], _lib.FB_EPI_GATED_RESIDUAL)
    del keep
    return out


@torch.no_grad()
def final_layer(w, img, fmod, dt, k=None):
    """LN-mod then Linear D -> in_channels, fp32 out (selas/models/flux.py:341-343)."""
    _check_dtype(dt)
    img = _f32(img)
    d = img.shape[-1]
    fmod = _bf16_rows(fmod)
    h = ops.ln_mod(img, fmod[:, :d], fmod[:, d:2 * d])
    return ops.linear(h, weight(w, "final_layer.linear.weight"), bias(w, "final_layer.linear"), out_dtype=F32)


# ------------------------------------------------------------------------------------------ segments


def _mod_bf16(t: torch.Tensor) -> torch.Tensor:
    """A [B, 1, D] / [B, D] modulation chunk as bf16 rows (exact for values that came from a bf16 mod)."""
    t = t.reshape(t.shape[0], -1)
    return t.to(BF16) if t.dtype != BF16 else t


def _mod_in(x, shift, scale, dt):
    _check_dtype(dt)
    return ops.ln_mod(_f32(x), _mod_bf16(shift), _mod_bf16(scale))


def _gated_add(x, g, y, guard: bool):
    return ops.gated_add(_f32(x), _mod_bf16(g), y.to(BF16).contiguous(), guard)


def _gated_add_mod(x, g, y, shift, scale, dt, guard: bool):
    x = _gated_add(x, g, y, guard)
    return x, _mod_in(x, shift, scale, dt)


def _qkv_double(tqkv, iqkv, tqs, tks, iqs, iks, cos, sin, heads: int, dt):
    _check_dtype(dt)
    b, lt, c = tqkv.shape
    li = iqkv.shape[1]
    hd = c // (3 * heads)
    seq = lt + li
    cos, sin = _rope(cos, sin, seq, hd)
    q = torch.empty(b, heads, seq, hd, dtype=BF16, device=tqkv.device)
    k, v = torch.empty_like(q), torch.empty_like(q)
    for t, qs, ks, off in ((tqkv, tqs, tks, 0), (iqkv, iqs, iks, lt)):
        if t.shape[1]:
            ops.qk_norm_rope(t.contiguous(), heads, qs.float().contiguous(), ks.float().contiguous(), cos, sin, q, k, v, off)
    return q, k, v


def _qkv_single(qkv, qs, ks, cos, sin, heads: int, dt):
    _check_dtype(dt)
    b, seq, c = qkv.shape
    hd = c // (3 * heads)
    cos, sin = _rope(cos, sin, seq, hd)
    q = torch.empty(b, heads, seq, hd, dtype=BF16, device=qkv.device)
    k, v = torch.empty_like(q), torch.empty_like(q)
    ops.qk_norm_rope(qkv, heads, qs.float().contiguous(), ks.float().contiguous(), cos, sin, q, k, v, 0)
    return q, k, v


def _gelu(h):
    return ops.gelu_tanh(h.contiguous())


def _attn_mlp(attn, mlp):
    return torch.cat((attn, _gelu(mlp)), dim=2)


class B200Kernels:
    """Drop-in for ``selas.models.flux.Kernels`` (flux.py:206-212), backed by libflux_b200.

    ``compiled`` is True (the segments are fused kernels, like the torch.compile variant). The seven
    segment attributes keep the eager signatures; ``double_block`` / ``single_block`` /
    ``final_layer`` run a whole block on the fused path.
    """

    def __init__(self):
        _lib.lib()  # load + fb_init now: a missing or broken library fails here, loudly
        self.compiled = True
        self.mod_in = _mod_in
        self.gated_add = _gated_add
        self.gated_add_mod = _gated_add_mod
        self.qkv_double = _qkv_double
        self.qkv_single = _qkv_single
        self.gelu = _gelu
        self.attn_mlp = _attn_mlp
        self.double_block = double_block
        self.single_block = single_block
        self.final_layer = final_layer
