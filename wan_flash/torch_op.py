"""The attention as ``torch.library`` custom ops, for callers that trace.

The reference exposes a ``torch.autograd.Function`` (``interface.py:199-215``);
its consumer, the external ``wan_attention`` op, wants a registered operator
with a fake (meta) implementation so that graphs holding it can be traced
with fake tensors (``torch.compile``, export, activation checkpointing
replays) without running the kernels.  This module registers

    wan_flash::attn_fwd(q, k, v) -> (o, lse)
    wan_flash::attn_bwd(q, k, v, o, lse, do) -> (dq, dk, dv)

with fake implementations that only produce the contract's shapes and
dtypes -- o like q (bf16), lse (b, h, sq) fp32, gradients like their inputs --
and ties them together with ``register_autograd``.  The real
implementations are ``wan_flash_fwd`` / ``wan_flash_bwd`` (the sm_100a
kernels); nothing here computes on the CPU.

``wan_attention(q, k, v) -> o`` is the op-based counterpart of
``wan_flash_attn``.  The two-context path (Wan I2V text + image cross
attention) has the same treatment:

    wan_flash::attn_fwd_dual(q, k0, v0, k1, v1) -> (o0, lse0, o1, lse1)
    wan_flash::attn_bwd_dual(q, k0, v0, k1, v1, o0, lse0, o1, lse1, do0, do1)
        -> (dq, dk0, dv0, dk1, dv1)

and ``wan_attention_dual(q, k0, v0, k1, v1) -> o0 + o1``.
"""

from __future__ import annotations

import torch

from wan_flash.interface import wan_flash_bwd, wan_flash_bwd_dual, wan_flash_fwd, wan_flash_fwd_dual


@torch.library.custom_op("wan_flash::attn_fwd", mutates_args=())
def attn_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    o, lse = wan_flash_fwd(q, k, v)
    return o, lse


def _like(t: torch.Tensor) -> torch.Tensor:
    """A contiguous tensor of t's shape, dtype and device: the real ops write
    contiguous (b, s, h, 128) outputs whatever the inputs' strides, so the fake
    outputs must not inherit a permuted input's strides."""
    return torch.empty(t.shape, dtype=t.dtype, device=t.device)


@attn_fwd.register_fake
def _attn_fwd_fake(q, k, v):
    b, sq, h, d = q.shape
    torch._check(d == 128, lambda: "specialized for head_dim=128")
    return _like(q), q.new_empty((b, h, sq), dtype=torch.float32)


@torch.library.custom_op("wan_flash::attn_bwd", mutates_args=())
def attn_bwd(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, o: torch.Tensor, lse: torch.Tensor, do: torch.Tensor
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    dq, dk, dv = wan_flash_bwd(q, k, v, o, lse, do)
    return dq, dk, dv


@attn_bwd.register_fake
def _attn_bwd_fake(q, k, v, o, lse, do):
    return _like(q), _like(k), _like(v)


def _setup_context(ctx, inputs, output):
    q, k, v = inputs
    o, lse = output
    # The LSE output carries no gradient (the reference's autograd function
    # returns o only): it is marked non-differentiable, so a loss that uses
    # it gets no gradient through it instead of a silently wrong one.
    ctx.mark_non_differentiable(lse)
    ctx.save_for_backward(q, k, v, o, lse)


def _backward(ctx, do, dlse):
    q, k, v, o, lse = ctx.saved_tensors
    dq, dk, dv = attn_bwd(q, k, v, o, lse, do.contiguous())
    return dq, dk, dv


attn_fwd.register_autograd(_backward, setup_context=_setup_context)


def wan_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """o = softmax(q k^T / sqrt(128)) v through the registered operator (differentiable)."""
    return attn_fwd(q, k, v)[0]


@torch.library.custom_op("wan_flash::attn_fwd_dual", mutates_args=())
def attn_fwd_dual(q: torch.Tensor, k0: torch.Tensor, v0: torch.Tensor, k1: torch.Tensor,
                  v1: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    o0, lse0, o1, lse1 = wan_flash_fwd_dual(q, k0, v0, k1, v1)
    return o0, lse0, o1, lse1


@attn_fwd_dual.register_fake
def _attn_fwd_dual_fake(q, k0, v0, k1, v1):
    b, sq, h, d = q.shape
    torch._check(d == 128, lambda: "specialized for head_dim=128")
    return _like(q), q.new_empty((b, h, sq), dtype=torch.float32), _like(q), q.new_empty((b, h, sq), dtype=torch.float32)


@torch.library.custom_op("wan_flash::attn_bwd_dual", mutates_args=())
def attn_bwd_dual(
    q: torch.Tensor, k0: torch.Tensor, v0: torch.Tensor, k1: torch.Tensor, v1: torch.Tensor, o0: torch.Tensor,
    lse0: torch.Tensor, o1: torch.Tensor, lse1: torch.Tensor, do0: torch.Tensor, do1: torch.Tensor
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    return wan_flash_bwd_dual(q, k0, v0, k1, v1, o0, lse0, o1, lse1, do0, do1)


@attn_bwd_dual.register_fake
def _attn_bwd_dual_fake(q, k0, v0, k1, v1, o0, lse0, o1, lse1, do0, do1):
    return _like(q), _like(k0), _like(v0), _like(k1), _like(v1)


def _setup_context_dual(ctx, inputs, output):
    o0, lse0, o1, lse1 = output
    ctx.mark_non_differentiable(lse0, lse1)  # as in the one-context op
    ctx.save_for_backward(*inputs, o0, lse0, o1, lse1)


def _backward_dual(ctx, do0, dlse0, do1, dlse1):
    q, k0, v0, k1, v1, o0, lse0, o1, lse1 = ctx.saved_tensors
    return attn_bwd_dual(q, k0, v0, k1, v1, o0, lse0, o1, lse1, do0.contiguous(), do1.contiguous())


attn_fwd_dual.register_autograd(_backward_dual, setup_context=_setup_context_dual)


def wan_attention_dual(q: torch.Tensor, k0: torch.Tensor, v0: torch.Tensor, k1: torch.Tensor,
                       v1: torch.Tensor) -> torch.Tensor:
    """attention(q, k0, v0) + attention(q, k1, v1) through the registered operators (differentiable)."""
    o0, _, o1, _ = attn_fwd_dual(q, k0, v0, k1, v1)
    return o0 + o1
