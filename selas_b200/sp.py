"""Ulysses sequence parallelism: one image's denoise step on P GPUs, for single-image latency.

Each of the P ranks holds a full weight replica and 1/P of the tokens of each stream: txt tokens
``rank*Lt/P .. (rank+1)*Lt/P`` and img tokens ``rank*Li/P .. (rank+1)*Li/P``, in that order (txt then
img) in its local sequence. Every part of a block is token-local except attention, which needs every
key. Around it, two all-to-alls over NCCL (NVLink) switch the layout:

* q, k, v leave the QKV GEMM as [B, H, L/P, 128] (local tokens, all heads); the first all-to-all sends
  head group g (heads g*H/P .. (g+1)*H/P) to rank g, which then holds [B, H/P, L, 128] (all tokens,
  its heads; tokens ordered rank by rank). Softmax is over all keys, whose order does not matter.
* The attention output [B, L, H/P*128] goes back by the second all-to-all: rank r receives its own
  tokens' rows from every head group and lays them out as [B, L/P, H*128] (heads in order).

selas has no sequence-parallel path; this is the optional exchange for the single-image 1024^2
latency case. The math is that of ``_attention`` (selas/models/flux.py:135-138) on the full sequence.
"""

from __future__ import annotations

from dataclasses import replace

import torch
import torch.distributed as dist

from . import ops
from ._lib import FluxB200Error


class Ulysses:
    """The all-to-all attention of one sequence-parallel group. ``attention_fn(q, k, v, out=...)`` is the
    single-GPU attention (the tcgen05 kernel by default; tests pass a CPU reference)."""

    def __init__(self, group=None, attention_fn=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.attention_fn = attention_fn or ops.attention

    def span(self, n: int) -> slice:
        """This rank's slice of a stream of n tokens."""
        if n % self.world:
            raise FluxB200Error(f"sequence parallelism over {self.world} ranks needs a token count divisible by it, got {n}")
        per = n // self.world
        return slice(self.rank * per, (self.rank + 1) * per)

    def attention(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor, split: int = 0,
                  out_first: torch.Tensor | None = None) -> None:
        """q/k/v [B, H, Ll, D] for this rank's Ll tokens; writes out [B, Ll - split, H*D] (and out_first
        [B, split, H*D] for the first ``split`` local tokens), like ops.attention on the full sequence."""
        p = self.world
        b, h, ll, d = q.shape
        if h % p:
            raise FluxB200Error(f"sequence parallelism over {p} ranks needs heads divisible by it, got {h}")
        hp = h // p
        # (local tokens, all heads) -> (all tokens, my head group): one exchange for q, k and v together.
        # The blocks allocate q, k, v as consecutive slices of one [3, B, H, Ll, D] buffer, which is then
        # used as is (no stacking copy).
        n, es = q.numel(), q.element_size()
        if k.data_ptr() == q.data_ptr() + es * n and v.data_ptr() == q.data_ptr() + 2 * es * n and q.is_contiguous():
            qkv = q.as_strided((3, b, h, ll, d), (n, h * ll * d, ll * d, d, 1))
        else:
            qkv = torch.stack((q, k, v))
        send = qkv.view(3, b, p, hp, ll, d).permute(2, 0, 1, 3, 4, 5).contiguous()
        recv = torch.empty_like(send)  # [source rank, 3, B, hp, Ll, D]
        dist.all_to_all_single(recv, send, group=self.group)
        g = recv.permute(1, 2, 3, 0, 4, 5).reshape(3, b, hp, p * ll, d)  # one copy; g[i] are contiguous
        og = torch.empty(b, p * ll, hp * d, dtype=q.dtype, device=q.device)
        self.attention_fn(g[0], g[1], g[2], out=og)
        # (all tokens, my head group) -> (local tokens, all heads)
        send2 = og.view(b, p, ll, hp * d).permute(1, 0, 2, 3).contiguous()  # [destination rank, B, Ll, hp*D]
        recv2 = torch.empty_like(send2)  # [source head group, B, Ll, hp*D]
        dist.all_to_all_single(recv2, send2, group=self.group)
        full = recv2.permute(1, 2, 0, 3).reshape(b, ll, h * d)
        if split:
            out_first.copy_(full[:, :split])
            out.copy_(full[:, split:])
        else:
            out.copy_(full)

    def localize(self, cond, l_img: int):
        """The Conditioning of this rank: its txt tokens, and the RoPE rows of its local sequence
        (its txt tokens, then its img tokens)."""
        lt = cond.l_txt
        ts, is_ = self.span(lt), self.span(l_img)
        rows = torch.cat((torch.arange(ts.start, ts.stop), lt + torch.arange(is_.start, is_.stop))).to(cond.cos.device)
        return replace(cond, txt=cond.txt[:, ts].contiguous(), cos=cond.cos[rows].contiguous(),
                       sin=cond.sin[rows].contiguous(), l_txt=ts.stop - ts.start)
