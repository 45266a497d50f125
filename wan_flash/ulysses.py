"""Sequence-parallel (Ulysses) attention over heads for multi-GPU Wan blocks.

The reference has no distributed code; this is the multi-GPU layer asked of
the B200 build.  Attention is independent per head, so a sequence-sharded
activation (b, S/P, H, D) on each of P ranks is turned into a head-sharded
one (b, S, H/P, D) with one all-to-all, attention runs locally on H/P heads
at full sequence length, and a second all-to-all returns the output to
sequence-sharded layout.  The backward mirrors it (the gradient of an
all-to-all is the inverse all-to-all).  Cross-attention context (text or
image tokens) is replicated on every rank, so each rank slices its heads
with no communication; the context gradient is all-gathered over heads in
the backward so every rank holds the full gradient of its replica.

All exchanges are ``torch.distributed.all_to_all_single`` / ``all_gather``
on contiguous, destination-major packed buffers (NCCL over NVLink on GPUs,
gloo on CPU for tests); remote data always lands in local memory before a
kernel reads it.  ``attn_fn`` defaults to ``wan_flash_attn``; tests inject a
CPU reference.
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist


def _world(group) -> int:
    return dist.get_world_size(group)


def _rank(group) -> int:
    return dist.get_rank(group)


def seq_to_head(x: torch.Tensor, group=None) -> torch.Tensor:
    """(b, S/P, H, D) sequence shard -> (b, S, H/P, D) head shard (no autograd)."""
    P = _world(group)
    b, s_loc, H, D = x.shape
    assert H % P == 0, f"heads {H} not divisible by {P} ranks"
    hp = H // P
    # destination-major: chunk p holds this rank's rows of head group p
    send = x.reshape(b, s_loc, P, hp, D).permute(2, 0, 1, 3, 4).contiguous()
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    # chunk p came from rank p = sequence shard p
    return recv.permute(1, 0, 2, 3, 4).reshape(b, P * s_loc, hp, D)


def head_to_seq(x: torch.Tensor, group=None) -> torch.Tensor:
    """(b, S, H/P, D) head shard -> (b, S/P, H, D) sequence shard (no autograd)."""
    P = _world(group)
    b, S, hp, D = x.shape
    assert S % P == 0, f"sequence {S} not divisible by {P} ranks"
    s_loc = S // P
    send = x.reshape(b, P, s_loc, hp, D).permute(1, 0, 2, 3, 4).contiguous()
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    # chunk p came from rank p = head group p
    return recv.permute(1, 2, 0, 3, 4).reshape(b, s_loc, P * hp, D)


class _SeqToHead(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return seq_to_head(x, group)

    @staticmethod
    def backward(ctx, g):
        return head_to_seq(g.contiguous(), ctx.group), None


class _HeadToSeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return head_to_seq(x, group)

    @staticmethod
    def backward(ctx, g):
        return seq_to_head(g.contiguous(), ctx.group), None


class _HeadSlice(torch.autograd.Function):
    """This rank's head group of a replicated (b, S, H, D) tensor; backward
    all-gathers the per-group gradients so the replica gets the full gradient."""

    @staticmethod
    def forward(ctx, x, group):
        P, r = _world(group), _rank(group)
        H = x.shape[2]
        assert H % P == 0
        hp = H // P
        ctx.group, ctx.hp = group, hp
        return x[:, :, r * hp:(r + 1) * hp].contiguous()

    @staticmethod
    def backward(ctx, g):
        P = _world(ctx.group)
        g = g.contiguous()
        parts = [torch.empty_like(g) for _ in range(P)]
        dist.all_gather(parts, g, group=ctx.group)
        return torch.cat(parts, dim=2), None


def _default_attn():
    from wan_flash.interface import wan_flash_attn

    return wan_flash_attn


def ulysses_self_attention(q, k, v, group=None, attn_fn: Callable | None = None):
    """Self-attention over sequence-sharded (b, S/P, H, D) q/k/v; returns
    the sequence-sharded output.  Differentiable."""
    attn_fn = attn_fn or _default_attn()
    qh = _SeqToHead.apply(q, group)
    kh = _SeqToHead.apply(k, group)
    vh = _SeqToHead.apply(v, group)
    return _HeadToSeq.apply(attn_fn(qh, kh, vh), group)


def ulysses_cross_attention(q, ctx_k, ctx_v, group=None, attn_fn: Callable | None = None):
    """Cross-attention of sequence-sharded q (b, S/P, H, D) against a context
    (b, L, H, D) replicated on every rank.  Differentiable."""
    attn_fn = attn_fn or _default_attn()
    qh = _SeqToHead.apply(q, group)
    kh = _HeadSlice.apply(ctx_k, group)
    vh = _HeadSlice.apply(ctx_v, group)
    return _HeadToSeq.apply(attn_fn(qh, kh, vh), group)


def shard_heads(x: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Head slice of a (b, S, H, D) tensor for replica-style head sharding (no communication)."""
    H = x.shape[2]
    assert H % world == 0
    hp = H // world
    return x[:, :, rank * hp:(rank + 1) * hp]
