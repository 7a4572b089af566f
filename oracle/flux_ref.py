"""FLUX block math restated on the CPU — TEST INFRASTRUCTURE ONLY (the checker for the CUDA path).

A restatement of selas's eager path (tcox-coding/selas ``selas/models/flux.py``), written against
plain dicts (or any mapping) of weights instead of ``UnitView``. Device-agnostic: with the weights and
inputs on a GPU, the same arithmetic runs there through torch (the full-size checks of the GPU tests). ``dt`` is the compute dtype exactly as in the
reference: Linear layers and attention run in ``dt`` (``selas/store.py:289-293``, ``flux.py:135-138``),
while the residual streams, LayerNorm, QK-RMSNorm, RoPE and modulation arithmetic stay fp32
(``flux.py:7-11``). ``dt=torch.float32`` gives the fp32 reference; ``dt=torch.bfloat16`` reproduces the
reference's bf16 numerics on the CPU.

Pinned against the reference itself by ``tests/test_oracle_golden.py`` (golden vectors written by
``tests/golden/make_golden.py``, which imports selas).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

FP16_MAX = 65504.0


# ----------------------------------------------------------------------------- primitives


def rope_tables(ids: torch.Tensor, axes_dim, theta: float = 10000.0):
    """cos/sin [L, sum(axes)/2] fp32 from position ids [L, n_axes]; angles in fp64 (flux.py:106-114)."""
    cols = []
    for axis, dim in enumerate(axes_dim):
        omega = theta ** (-(torch.arange(0, dim, 2, dtype=torch.float64, device=ids.device) / dim))
        cols.append(ids[:, axis].double().unsqueeze(1) * omega.unsqueeze(0))
    angle = torch.cat(cols, dim=1)
    return torch.cos(angle).float(), torch.sin(angle).float()


def apply_rope(x, cos, sin):
    """Rotate interleaved pairs (x[2i], x[2i+1]) by the angle of pair i (flux.py:117-121)."""
    even, odd = x[..., 0::2], x[..., 1::2]
    out = torch.empty_like(x)
    out[..., 0::2] = even * cos - odd * sin
    out[..., 1::2] = even * sin + odd * cos
    return out


def qk_rms(x, scale, eps: float = 1e-6):
    """RMSNorm over the head dim with an fp32 scale (flux.py:124-126)."""
    xf = x.float()
    return xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps) * scale


def layer_norm(x):
    """LayerNorm without affine parameters, eps 1e-6 (flux.py:146-147)."""
    return F.layer_norm(x, (x.shape[-1],), eps=1e-6)


def mod_in(x, shift, scale, dt):
    """LN(x) * (1 + scale) + shift, cast to the compute dtype (flux.py:164-166)."""
    return (layer_norm(x) * (1 + scale) + shift).to(dt)


def residual(y, guard: bool):
    """Linear output promoted to fp32, clamped to the fp16 range when guarding (flux.py:141-143)."""
    y = y.float()
    return y.clamp(-FP16_MAX, FP16_MAX) if guard else y


def gated_add(x, g, y, guard: bool):
    """x + g * y in fp32 (flux.py:169-171)."""
    return x + g * residual(y, guard)


def gelu_tanh(h):
    return F.gelu(h, approximate="tanh")


def linear(W: dict, x, prefix: str, dt):
    """F.linear in the compute dtype with the unit's weight and optional bias (store.py:289-293)."""
    w = W[prefix + ".weight"].to(dt)
    b = W.get(prefix + ".bias")
    return F.linear(x.to(dt), w, None if b is None else b.to(dt))


def split_heads(qkv, heads: int):
    """[B, L, 3*H*Dh] -> three [B, H, L, Dh] views (flux.py:129-132)."""
    b, l, _ = qkv.shape
    t = qkv.reshape(b, l, 3, heads, -1).permute(2, 0, 3, 1, 4)
    return t[0], t[1], t[2]


def attention(q, k, v):
    """softmax(q k^T / sqrt(Dh)) v, then [B, L, H*Dh] (flux.py:135-138)."""
    b, h, l, d = q.shape
    o = F.scaled_dot_product_attention(q, k, v)
    return o.transpose(1, 2).reshape(b, l, h * d)


def _chunks(mod, n):
    return mod.float().unsqueeze(1).chunk(n, dim=-1)


# ----------------------------------------------------------------------------- blocks


def double_block(W: dict, img, txt, mod, cos, sin, heads: int, dt, guard: bool = False):
    """Two-stream MMDiT block (flux.py:300-324). mod [B, 12D] = img (6D) | txt (6D)."""
    m = _chunks(mod, 12)
    i_sh1, i_sc1, i_g1, i_sh2, i_sc2, i_g2 = m[:6]
    t_sh1, t_sc1, t_g1, t_sh2, t_sc2, t_g2 = m[6:]
    lt = txt.shape[1]

    iqkv = linear(W, mod_in(img, i_sh1, i_sc1, dt), "img_attn.qkv", dt)
    tqkv = linear(W, mod_in(txt, t_sh1, t_sc1, dt), "txt_attn.qkv", dt)
    tq, tk, tv = split_heads(tqkv, heads)
    iq, ik, iv = split_heads(iqkv, heads)
    f32 = lambda n: W[n].float()  # noqa: E731
    q = torch.cat((qk_rms(tq, f32("txt_attn.norm.query_norm.scale")), qk_rms(iq, f32("img_attn.norm.query_norm.scale"))), 2)
    k = torch.cat((qk_rms(tk, f32("txt_attn.norm.key_norm.scale")), qk_rms(ik, f32("img_attn.norm.key_norm.scale"))), 2)
    q = apply_rope(q, cos, sin).to(dt)
    k = apply_rope(k, cos, sin).to(dt)
    v = torch.cat((tv, iv), dim=2)
    attn = attention(q, k, v)
    t_attn, i_attn = attn[:, :lt], attn[:, lt:]

    img = gated_add(img, i_g1, linear(W, i_attn, "img_attn.proj", dt), guard)
    h = linear(W, mod_in(img, i_sh2, i_sc2, dt), "img_mlp.0", dt)
    img = gated_add(img, i_g2, linear(W, gelu_tanh(h), "img_mlp.2", dt), guard)
    txt = gated_add(txt, t_g1, linear(W, t_attn, "txt_attn.proj", dt), guard)
    h = linear(W, mod_in(txt, t_sh2, t_sc2, dt), "txt_mlp.0", dt)
    txt = gated_add(txt, t_g2, linear(W, gelu_tanh(h), "txt_mlp.2", dt), guard)
    return img, txt


def single_block(W: dict, x, mod, cos, sin, heads: int, mlp_hidden: int, dt, guard: bool = False):
    """Parallel attention + MLP block on the joint sequence (flux.py:327-338). mod [B, 3D]."""
    sh, sc, g = _chunks(mod, 3)
    d = x.shape[-1]
    h = linear(W, mod_in(x, sh, sc, dt), "linear1", dt)
    qkv, mlp = h.split([3 * d, mlp_hidden], dim=-1)
    q, k, v = split_heads(qkv, heads)
    q = apply_rope(qk_rms(q, W["norm.query_norm.scale"].float()), cos, sin).to(dt)
    k = apply_rope(qk_rms(k, W["norm.key_norm.scale"].float()), cos, sin).to(dt)
    attn = attention(q, k, v.contiguous())
    out = linear(W, torch.cat((attn, gelu_tanh(mlp)), dim=2), "linear2", dt)
    return gated_add(x, g, out, guard)


def final_layer(W: dict, img, fmod, dt):
    """LN-mod then Linear D -> in_channels, returned in fp32 (flux.py:341-343)."""
    sh, sc = _chunks(fmod, 2)
    return linear(W, mod_in(img, sh, sc, dt), "final_layer.linear", dt).float()


# ----------------------------------------------------------------------------- prologue + runner


def timestep_embedding(t, dim: int = 256, max_period: float = 10000.0, time_factor: float = 1000.0):
    """Sinusoidal embedding [cos | sin] (flux.py:95-103)."""
    t = time_factor * t.float()
    half = dim // 2
    freqs = torch.exp(-math.log(max_period) * torch.arange(half, dtype=torch.float32, device=t.device) / half)
    args = t[:, None] * freqs[None]
    emb = torch.cat([torch.cos(args), torch.sin(args)], dim=-1)
    if dim % 2:
        emb = torch.cat([emb, torch.zeros_like(emb[:, :1])], dim=-1)
    return emb


def mlp_embed(W: dict, prefix: str, x, dt):
    return linear(W, F.silu(linear(W, x, prefix + ".in_layer", dt)), prefix + ".out_layer", dt)


def svec(G: dict, sigmas, guidance: float, pooled, dt, guidance_embed: bool = True):
    """silu(vec) [S, 1, D] for one image (flux.py:411-425)."""
    t = torch.tensor(list(sigmas[:-1]), dtype=torch.float32, device=pooled.device)
    vec = mlp_embed(G, "time_in", timestep_embedding(t, 256).to(dt), dt).float()[:, None, :]
    if guidance_embed:
        gv = torch.full((1,), float(guidance), dtype=torch.float32, device=pooled.device)
        vec = vec + mlp_embed(G, "guidance_in", timestep_embedding(gv, 256).to(dt), dt).float()[None]
    vec = vec + mlp_embed(G, "vector_in", pooled.to(dt), dt).float()[None]
    return F.silu(vec).to(dt)


def prepare(units: dict, a, sigmas, guidance: float, pooled, txt, img_ids, txt_ids, dt):
    """Per-batch conditioning (flux.py:448-465): per-step modulations, txt_in, RoPE tables."""
    G = units["globals"]
    svecs = [svec(G, sigmas, guidance, pooled[i:i + 1], dt, a.guidance_embed) for i in range(pooled.shape[0])]
    mods = {}
    for i in range(a.depth_double):
        M = units[f"double.{i}.mod"]
        mods[f"double.{i}"] = torch.cat(
            [torch.cat((linear(M, sv, "img_mod.lin", dt), linear(M, sv, "txt_mod.lin", dt)), dim=-1) for sv in svecs], dim=1)
    for i in range(a.depth_single):
        M = units[f"single.{i}.mod"]
        mods[f"single.{i}"] = torch.cat([linear(M, sv, "modulation.lin", dt) for sv in svecs], dim=1)
    final_mod = torch.cat([linear(G, sv, "final_layer.adaLN_modulation.1", dt) for sv in svecs], dim=1)
    txt_h = linear(G, txt, "txt_in", dt).float()
    cos, sin = rope_tables(torch.cat((txt_ids, img_ids), dim=0), a.axes_dim, a.theta)
    return {"sigmas": list(sigmas), "mods": mods, "final_mod": final_mod, "txt": txt_h, "cos": cos, "sin": sin,
            "l_txt": txt.shape[1]}


def step(units: dict, a, s: int, latents, cond: dict, dt):
    """Velocity prediction for step s (flux.py:527-582, without the step cache)."""
    guard = dt == torch.float16
    G = units["globals"]
    img = linear(G, latents, "img_in", dt).float()
    txt = cond["txt"]
    lt = cond["l_txt"]
    for i in range(a.depth_double):
        img, txt = double_block(units[f"double.{i}"], img, txt, cond["mods"][f"double.{i}"][s], cond["cos"], cond["sin"],
                                a.heads, dt, guard)
    x = torch.cat((txt, img), dim=1)
    for i in range(a.depth_single):
        x = single_block(units[f"single.{i}"], x, cond["mods"][f"single.{i}"][s], cond["cos"], cond["sin"], a.heads,
                         a.mlp_hidden, dt, guard)
    return final_layer(G, x[:, lt:], cond["final_mod"][s], dt)


def denoise(units: dict, a, x, cond: dict, dt):
    """Euler flow-matching loop (pipeline.py:483-489): x <- x + (sigma[s+1] - sigma[s]) * v."""
    sig = cond["sigmas"]
    preds = []
    for s in range(len(sig) - 1):
        v = step(units, a, s, x, cond, dt)
        preds.append(v)
        x = x + (sig[s + 1] - sig[s]) * v
    return x, preds


# ----------------------------------------------------------------------------- sampling helpers


def get_schedule(num_steps: int, image_seq_len: int, base_shift: float = 0.5, max_shift: float = 1.15):
    """num_steps + 1 sigmas from 1 to 0 with the resolution-dependent shift (sampling.py:10-29)."""
    x1, x2 = 256, 4096
    slope = (max_shift - base_shift) / (x2 - x1)
    mu = slope * image_seq_len + (base_shift - slope * x1)
    out = []
    for i in range(num_steps + 1):
        t = 1.0 - i / num_steps
        if t <= 0.0:
            out.append(0.0)
        elif t >= 1.0:
            out.append(1.0)
        else:
            out.append(math.exp(mu) / (math.exp(mu) + (1.0 / t - 1.0)))
    return out


def get_noise(seed: int, height: int, width: int, channels: int = 16):
    """CPU-seeded fp32 latent noise (sampling.py:37-41)."""
    h, w = 2 * math.ceil(height / 16), 2 * math.ceil(width / 16)
    g = torch.Generator(device="cpu").manual_seed(int(seed))
    return torch.randn(1, channels, h, w, generator=g, dtype=torch.float32)


def pack(x):
    """[B, C, H, W] -> [B, (H/2)(W/2), 4C] (sampling.py:44-47)."""
    b, c, h, w = x.shape
    return x.view(b, c, h // 2, 2, w // 2, 2).permute(0, 2, 4, 1, 3, 5).reshape(b, (h // 2) * (w // 2), c * 4)


def image_ids(height: int, width: int):
    """(0, row, col) position ids of the packed latent grid (sampling.py:58-65)."""
    h, w = math.ceil(height / 16), math.ceil(width / 16)
    ids = torch.zeros(h, w, 3)
    ids[..., 1] = torch.arange(h)[:, None]
    ids[..., 2] = torch.arange(w)[None, :]
    return ids.reshape(h * w, 3)


def text_ids(length: int):
    return torch.zeros(length, 3)
