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

import ctypes
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


class UlyssesP2P(Ulysses):
    """Ulysses attention with the two all-to-alls done by the kernels' own stores over NVLink (one image).

    Each rank allocates, once, the buffers the other ranks write into (one device allocation, so one
    CUDA IPC handle per rank, exchanged through the process group and opened with fb_ipc_open):

    * ``qkv`` [3, H/P, P*Ll, 128] bf16 — q, k, v of this rank's head group for every token; the QKV GEMM
      epilogue of every rank stores its tokens' rows of each head group into that group's owner;
    * ``att`` [Ll, D] bf16 — the double blocks' attention rows of this rank's tokens (the proj input);
    * ``cat`` [Ll, D + Mm] bf16 — the single blocks' linear2 input, whose first D columns the peers'
      attention kernels fill and whose GELU columns this rank's linear1 epilogue fills;
    * ``flags`` [8] int32 — the peer barrier's flags.

    A block then runs: QKV GEMM (scattering) -> barrier -> attention (scattering its rows back) ->
    barrier -> proj / linear2 on the local buffer. Each buffer is reused block after block, and a rank
    stores into a peer's buffer only after a barrier that the peer reaches after its last read of it:
    qkv is rewritten by QKV(n+1), which follows barrier 2 of block n, which the owner passes after its
    attention(n); att/cat are rewritten by attention(n+1), which follows barrier 1 of block n+1, which
    the owner passes after its proj/linear2(n).
    """

    def __init__(self, arch, l_local: int, group=None, timeout_ms: int = 20000):
        super().__init__(group)
        from . import _lib

        p, h = self.world, arch.heads
        if h % p or p > 8:
            raise FluxB200Error(f"UlyssesP2P: {p} ranks must divide {h} heads (at most 8 ranks)")
        if arch.hidden // h != 128:
            raise FluxB200Error("UlyssesP2P: head_dim must be 128")
        self.p2p = True
        self.hp = h // p
        self.ll = int(l_local)
        self.timeout_ms = int(timeout_ms)
        d, mm = arch.hidden, arch.mlp_hidden
        sizes = [3 * self.hp * p * self.ll * 128 * 2, self.ll * d * 2, self.ll * (d + mm) * 2, 8 * 4]
        offs, tot = [], 0
        for n in sizes:
            offs.append(tot)
            tot += (n + 255) // 256 * 256
        dev = torch.device("cuda", torch.cuda.current_device())
        self._mem = torch.zeros(tot, dtype=torch.uint8, device=dev)
        view = lambda i, dt: self._mem[offs[i]:offs[i] + sizes[i]].view(dt)  # noqa: E731
        self.qkv = view(0, torch.bfloat16).view(3, self.hp, p * self.ll, 128)
        self.att = view(1, torch.bfloat16).view(self.ll, d)
        self.cat = view(2, torch.bfloat16).view(self.ll, d + mm)
        self.flags = view(3, torch.int32)
        torch.cuda.synchronize()
        L = _lib.lib()
        h64 = (ctypes.c_char * 64)()
        off = ctypes.c_int64(0)
        _lib.check(L.fb_ipc_export(self._mem.data_ptr(), h64, ctypes.byref(off)), "fb_ipc_export")
        everyone = [None] * p
        dist.all_gather_object(everyone, (bytes(h64), int(off.value)), group=group)
        self._opened = []
        bases = []
        for r in range(p):
            if r == self.rank:
                bases.append(self._mem.data_ptr())
                continue
            ptr, base = ctypes.c_void_p(), ctypes.c_void_p()
            _lib.check(L.fb_ipc_open(everyone[r][0], everyone[r][1], ctypes.byref(ptr), ctypes.byref(base)),
                       "fb_ipc_open")
            self._opened.append(base.value)
            bases.append(ptr.value)
        self.qkv_peers, self.att_peers, self.cat_peers, self.flag_peers = ([b + offs[i] for b in bases]
                                                                           for i in range(4))
        self.epoch = 0
        self.barrier()  # every rank has mapped every buffer before anyone stores into one

    def barrier(self) -> None:
        self.epoch += 1
        ops.peer_barrier(self.flag_peers, self.rank, self.epoch, self.timeout_ms)

    def qkv_fields(self, p) -> None:
        """Point a QKV-epilogue fb_linear at the head-group owners' qkv buffers."""
        for g in range(self.world):
            p.sp_qkv_dst[g] = self.qkv_peers[g]
        p.sp_world, p.sp_rank = self.world, self.rank

    def attention_into(self, peers: list[int], ld: int) -> None:
        """Attention of this rank's head group over all tokens, rows stored into each token owner's
        buffer (``peers`` = att_peers or cat_peers) at this group's columns."""
        ops.attention_sp(self.qkv[0], self.qkv[1], self.qkv[2], peers, ld, self.rank * self.hp * 128, self.ll)

    def close(self) -> None:
        """Unmap the peers' buffers, after a final barrier so that no rank still stores into them."""
        from . import _lib

        if not getattr(self, "_opened", None):
            return
        self.barrier()
        torch.cuda.synchronize()
        for base in self._opened:
            _lib.check(_lib.lib().fb_ipc_close(base), "fb_ipc_close")
        self._opened = []
