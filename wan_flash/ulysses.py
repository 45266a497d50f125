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


# --------------------------------------------------------------------------
# A whole sequence-parallel attention block (self + cross) with overlapped
# exchanges.
# --------------------------------------------------------------------------
def _pack_s2h(x: torch.Tensor, P: int) -> torch.Tensor:
    b, s_loc, H, D = x.shape
    return x.reshape(b, s_loc, P, H // P, D).permute(2, 0, 1, 3, 4).contiguous()


def _unpack_s2h(recv: torch.Tensor) -> torch.Tensor:
    P, b, s_loc, hp, D = recv.shape
    return recv.permute(1, 0, 2, 3, 4).reshape(b, P * s_loc, hp, D)


def _pack_h2s(x: torch.Tensor, P: int) -> torch.Tensor:
    b, S, hp, D = x.shape
    return x.reshape(b, P, S // P, hp, D).permute(1, 0, 2, 3, 4).contiguous()


def _unpack_h2s(recv: torch.Tensor) -> torch.Tensor:
    P, b, s_loc, hp, D = recv.shape
    return recv.permute(1, 2, 0, 3, 4).reshape(b, s_loc, P * hp, D)


def _a2a_start(send: torch.Tensor, group):
    recv = torch.empty_like(send)
    work = dist.all_to_all_single(recv, send, group=group, async_op=True)
    return recv, work


def _default_fwd_bwd():
    from wan_flash.interface import wan_flash_bwd, wan_flash_fwd

    return wan_flash_fwd, wan_flash_bwd


class _UlyssesBlock(torch.autograd.Function):
    """Self-attention over sequence-sharded q/k/v and cross-attention of the
    same q against a replicated context, with the exchanges issued
    asynchronously and ordered so that each runs under attention work that
    does not need it:

    forward   q, k, v out -> [wait q]   cross fwd        (k, v still moving)
                             [wait k,v] self fwd         (o_cross moving back)
                             o_self back
    backward  dO_self in  -> [wait]     self bwd         (dO_cross moving in)
                             dk, dv back; [wait dO_cross] cross bwd (dk, dv moving)
                             dq = dq_self + dq_cross back (q was exchanged once)

    The two attention calls share one exchanged q, and their dq
    contributions are summed before a single return exchange: 10 all-to-alls
    per forward + backward instead of 12."""

    @staticmethod
    def forward(ctx, q, k, v, ck, cv, group, fwd, bwd):
        P, r = _world(group), _rank(group)
        H = q.shape[2]
        assert H % P == 0, f"heads {H} not divisible by {P} ranks"
        hp = H // P
        rq, wq = _a2a_start(_pack_s2h(q, P), group)
        rk, wk = _a2a_start(_pack_s2h(k, P), group)
        rv, wv = _a2a_start(_pack_s2h(v, P), group)
        ckh = ck[:, :, r * hp:(r + 1) * hp].contiguous()
        cvh = cv[:, :, r * hp:(r + 1) * hp].contiguous()
        wq.wait()
        qh = _unpack_s2h(rq)
        o_ch, lse_c = fwd(qh, ckh, cvh)
        roc, woc = _a2a_start(_pack_h2s(o_ch, P), group)
        wk.wait()
        wv.wait()
        kh, vh = _unpack_s2h(rk), _unpack_s2h(rv)
        o_sh, lse_s = fwd(qh, kh, vh)
        ros, wos = _a2a_start(_pack_h2s(o_sh, P), group)
        woc.wait()
        o_c = _unpack_h2s(roc)
        wos.wait()
        o_s = _unpack_h2s(ros)
        ctx.save_for_backward(qh, kh, vh, ckh, cvh, o_sh, lse_s, o_ch, lse_c)
        ctx.group, ctx.P, ctx.hp, ctx.bwd = group, P, hp, bwd
        ctx.out_shape = o_s.shape  # sequence-sharded (b, S/P, H, D), both outputs
        # an output unused by the loss arrives as None (no zeros materialised
        # by autograd); backward makes the zeros it exchanges itself
        ctx.set_materialize_grads(False)
        return o_s, o_c

    @staticmethod
    def backward(ctx, g_s, g_c):
        qh, kh, vh, ckh, cvh, o_sh, lse_s, o_ch, lse_c = ctx.saved_tensors
        group, P, bwd = ctx.group, ctx.P, ctx.bwd
        # an output that did not reach the loss has no gradient: zeros of the
        # sequence-sharded output shape (not the head-sharded o_sh / o_ch)
        if g_s is None:
            g_s = torch.zeros(ctx.out_shape, dtype=o_sh.dtype, device=o_sh.device)
        if g_c is None:
            g_c = torch.zeros(ctx.out_shape, dtype=o_ch.dtype, device=o_ch.device)
        rgs, wgs = _a2a_start(_pack_s2h(g_s.contiguous(), P), group)
        rgc, wgc = _a2a_start(_pack_s2h(g_c.contiguous(), P), group)
        wgs.wait()
        dq_s, dk_h, dv_h = bwd(qh, kh, vh, o_sh, lse_s, _unpack_s2h(rgs))
        rdk, wdk = _a2a_start(_pack_h2s(dk_h, P), group)
        rdv, wdv = _a2a_start(_pack_h2s(dv_h, P), group)
        wgc.wait()
        dq_c, dck_h, dcv_h = bwd(qh, ckh, cvh, o_ch, lse_c, _unpack_s2h(rgc))
        dq_h = (dq_s.float() + dq_c.float()).to(dq_s.dtype)
        rdq, wdq = _a2a_start(_pack_h2s(dq_h, P), group)
        # the replicated context's gradient: every rank's head group, gathered
        parts_k = [torch.empty_like(dck_h) for _ in range(P)]
        parts_v = [torch.empty_like(dcv_h) for _ in range(P)]
        wck = dist.all_gather(parts_k, dck_h.contiguous(), group=group, async_op=True)
        wcv = dist.all_gather(parts_v, dcv_h.contiguous(), group=group, async_op=True)
        wdk.wait()
        wdv.wait()
        wdq.wait()
        wck.wait()
        wcv.wait()
        dq, dk, dv = _unpack_h2s(rdq), _unpack_h2s(rdk), _unpack_h2s(rdv)
        return dq, dk, dv, torch.cat(parts_k, dim=2), torch.cat(parts_v, dim=2), None, None, None


def ulysses_attention_block(q, k, v, ctx_k, ctx_v, group=None, fwd: Callable | None = None,
                            bwd: Callable | None = None):
    """The attention of a sequence-parallel Wan block: self-attention of the
    sequence-sharded q/k/v (b, S/P, H, D) and cross-attention of the same q
    against a context (b, L, H, D) replicated on every rank.  Returns the two
    sequence-sharded outputs; differentiable.  ``fwd``/``bwd`` default to
    ``wan_flash_fwd``/``wan_flash_bwd`` (tests inject a CPU reference)."""
    if fwd is None or bwd is None:
        f0, b0 = _default_fwd_bwd()
        fwd, bwd = fwd or f0, bwd or b0
    return _UlyssesBlock.apply(q, k, v, ctx_k, ctx_v, group, fwd, bwd)
