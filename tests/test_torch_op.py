"""The attention as torch.library custom ops (wan_flash.torch_op).

CPU: the fake implementations trace forward and backward under
FakeTensorMode with the contract's shapes and dtypes (no kernel runs).
GPU: the ops return exactly what wan_flash_fwd / wan_flash_bwd return, pass
torch.library.opcheck, and the op-based autograd matches wan_flash_attn.
"""

import pytest
import torch


def _fake_inputs(sq=300, skv=200, h=2):
    q = torch.empty(1, sq, h, 128, dtype=torch.bfloat16, device="cuda")
    k = torch.empty(1, skv, h, 128, dtype=torch.bfloat16, device="cuda")
    v = torch.empty(1, skv, h, 128, dtype=torch.bfloat16, device="cuda")
    return q, k, v


def test_fake_forward_backward_shapes():
    from torch._subclasses.fake_tensor import FakeTensorMode

    import wan_flash.torch_op as op

    with FakeTensorMode():
        q, k, v = _fake_inputs()
        o, lse = torch.ops.wan_flash.attn_fwd(q, k, v)
        assert o.shape == q.shape and o.dtype == torch.bfloat16
        assert lse.shape == (1, 2, 300) and lse.dtype == torch.float32
        dq, dk, dv = torch.ops.wan_flash.attn_bwd(q, k, v, o, lse, o)
        assert (dq.shape, dk.shape, dv.shape) == (q.shape, k.shape, v.shape)
    # the registered autograd formula, on meta tensors (the autograd engine
    # wants a real CUDA device for fake CUDA tensors)
    qg, kg, vg = (torch.empty(1, s, 2, 128, dtype=torch.bfloat16, device="meta", requires_grad=True)
                  for s in (300, 200, 200))
    out = op.wan_attention(qg, kg, vg)
    out.backward(torch.empty_like(out))
    assert out.shape == qg.shape
    assert (qg.grad.shape, kg.grad.shape, vg.grad.shape) == (qg.shape, kg.shape, vg.shape)
    assert qg.grad.dtype == torch.bfloat16


def test_fake_outputs_contiguous_for_permuted_inputs():
    """The kernels write contiguous (b, s, h, 128) outputs whatever the
    inputs' strides; the fakes must report the same strides, or a traced
    graph would index the real outputs wrongly."""
    from torch._subclasses.fake_tensor import FakeTensorMode

    import wan_flash.torch_op  # noqa: F401  (registers the ops)

    def permuted(t):  # dense (b, s, h, d) view of a (b, h, s, d) tensor
        return t.transpose(1, 2).contiguous().transpose(1, 2)

    with FakeTensorMode():
        q, k, v = (permuted(t) for t in _fake_inputs())
        assert not q.is_contiguous()
        o, lse = torch.ops.wan_flash.attn_fwd(q, k, v)
        assert o.is_contiguous() and lse.is_contiguous()
        for g in torch.ops.wan_flash.attn_bwd(q, k, v, permuted(o), lse, permuted(o)):
            assert g.is_contiguous()
        _, k1, v1 = (permuted(t) for t in _fake_inputs(skv=257))
        outs = torch.ops.wan_flash.attn_fwd_dual(q, k, v, k1, v1)
        assert all(t.is_contiguous() for t in outs)
        g = torch.ops.wan_flash.attn_bwd_dual(q, k, v, k1, v1, outs[0], outs[1], outs[2], outs[3], outs[0], outs[2])
        assert all(t.is_contiguous() for t in g)


def test_lse_outputs_not_differentiable():
    """LSE carries no gradient (the reference's autograd returns o only): the
    op marks it non-differentiable instead of dropping its gradient silently."""
    import wan_flash.torch_op  # noqa: F401

    leaves = [torch.empty(1, s, 2, 128, dtype=torch.bfloat16, device="meta", requires_grad=True)
              for s in (300, 200, 200, 257, 257)]
    o, lse = torch.ops.wan_flash.attn_fwd(*leaves[:3])
    assert o.requires_grad and not lse.requires_grad
    o0, lse0, o1, lse1 = torch.ops.wan_flash.attn_fwd_dual(*leaves)
    assert o0.requires_grad and o1.requires_grad and not lse0.requires_grad and not lse1.requires_grad
    with pytest.raises(RuntimeError):
        lse.sum().backward()


@pytest.mark.gpu
def test_ops_match_interface_and_opcheck():
    import wan_flash.torch_op as op
    from tests.gpu_util import seeded
    from wan_flash.interface import wan_flash_attn, wan_flash_bwd, wan_flash_fwd

    q, k, v, do = (t.cuda() for t in seeded(1, 700, 300, 2, seed=23))
    o, lse = torch.ops.wan_flash.attn_fwd(q, k, v)
    o2, lse2 = wan_flash_fwd(q, k, v)
    assert torch.equal(o, o2) and torch.equal(lse, lse2)
    g = torch.ops.wan_flash.attn_bwd(q, k, v, o, lse, do)
    g2 = wan_flash_bwd(q, k, v, o, lse, do)
    # same kernels; only the fp32 reduction order (dq, and dk/dv under split-M) may differ
    for a, b in zip(g, g2):
        assert ((a.float() - b.float()).norm() / b.float().norm()).item() < 1e-3
    torch.library.opcheck(torch.ops.wan_flash.attn_fwd.default, (q, k, v), test_utils=("test_schema", "test_faketensor"))

    qa, ka, va = (t.clone().requires_grad_(True) for t in (q, k, v))
    qb, kb, vb = (t.clone().requires_grad_(True) for t in (q, k, v))
    op.wan_attention(qa, ka, va).backward(do)
    wan_flash_attn(qb, kb, vb).backward(do)
    for a, b in zip((qa.grad, ka.grad, va.grad), (qb.grad, kb.grad, vb.grad)):
        assert ((a.float() - b.float()).norm() / b.float().norm()).item() < 1e-3


def test_fake_dual_forward_backward_shapes():
    from torch._subclasses.fake_tensor import FakeTensorMode

    import wan_flash.torch_op as op

    with FakeTensorMode():
        q, k0, v0 = _fake_inputs(sq=300, skv=512)
        _, k1, v1 = _fake_inputs(sq=300, skv=257)
        o0, lse0, o1, lse1 = torch.ops.wan_flash.attn_fwd_dual(q, k0, v0, k1, v1)
        assert o0.shape == o1.shape == q.shape and o0.dtype == torch.bfloat16
        assert lse0.shape == lse1.shape == (1, 2, 300) and lse1.dtype == torch.float32
        g = torch.ops.wan_flash.attn_bwd_dual(q, k0, v0, k1, v1, o0, lse0, o1, lse1, o0, o1)
        assert [t.shape for t in g] == [q.shape, k0.shape, v0.shape, k1.shape, v1.shape]
    leaves = [torch.empty(1, s, 2, 128, dtype=torch.bfloat16, device="meta", requires_grad=True)
              for s in (300, 512, 512, 257, 257)]
    out = op.wan_attention_dual(*leaves)
    out.backward(torch.empty_like(out))
    assert out.shape == leaves[0].shape
    assert [t.grad.shape for t in leaves] == [t.shape for t in leaves]


@pytest.mark.gpu
def test_dual_ops_match_interface():
    import wan_flash.torch_op as op
    from tests.gpu_util import seeded
    from wan_flash.interface import wan_flash_attn_dual, wan_flash_fwd_dual

    q, k0, v0, do = (t.cuda() for t in seeded(1, 700, 300, 2, seed=29))
    _, k1, v1, _ = (t.cuda() for t in seeded(1, 700, 130, 2, seed=31))
    outs = torch.ops.wan_flash.attn_fwd_dual(q, k0, v0, k1, v1)
    for a, b in zip(outs, wan_flash_fwd_dual(q, k0, v0, k1, v1)):
        assert torch.equal(a, b)
    torch.library.opcheck(torch.ops.wan_flash.attn_fwd_dual.default, (q, k0, v0, k1, v1),
                          test_utils=("test_schema", "test_faketensor"))
    la = [t.clone().requires_grad_(True) for t in (q, k0, v0, k1, v1)]
    lb = [t.clone().requires_grad_(True) for t in (q, k0, v0, k1, v1)]
    oa = op.wan_attention_dual(*la)
    ob = wan_flash_attn_dual(*lb)
    assert torch.equal(oa, ob)
    oa.backward(do)
    ob.backward(do)
    for x, y in zip(la, lb):
        assert ((x.grad.float() - y.grad.float()).norm() / y.grad.float().norm()).item() < 1e-3


@pytest.mark.gpu
def test_op_under_activation_checkpointing():
    """The op inside torch.utils.checkpoint (full recompute) and under a
    selective-checkpoint policy that saves the attention outputs (the
    forward is then not re-run in the backward): gradients match the plain
    run up to the fp32 reduction order."""
    from torch.utils.checkpoint import CheckpointPolicy, checkpoint, create_selective_checkpoint_contexts

    import wan_flash.torch_op as op
    from tests.gpu_util import seeded

    q, k, v, do = (t.cuda() for t in seeded(1, 640, 384, 2, seed=37))
    w = torch.randn(128, 128, device="cuda", dtype=torch.bfloat16) * 0.05

    def block(q, k, v):
        return op.wan_attention(q @ w, k, v) @ w

    def policy(ctx, fn, *args, **kwargs):
        if fn == torch.ops.wan_flash.attn_fwd.default:
            return CheckpointPolicy.MUST_SAVE
        return CheckpointPolicy.PREFER_RECOMPUTE

    # count the forward kernel launches through the op's implementation
    launches = {"n": 0}
    real_fwd = op.wan_flash_fwd

    def counting_fwd(*a):
        launches["n"] += 1
        return real_fwd(*a)

    results, counts = [], []
    op.wan_flash_fwd = counting_fwd
    try:
        for mode in ("plain", "checkpoint", "selective"):
            launches["n"] = 0
            leaves = [t.clone().requires_grad_(True) for t in (q, k, v)]
            if mode == "plain":
                out = block(*leaves)
            elif mode == "checkpoint":
                out = checkpoint(block, *leaves, use_reentrant=False)
            else:
                out = checkpoint(block, *leaves, use_reentrant=False,
                                 context_fn=lambda: create_selective_checkpoint_contexts(policy))
            out.backward(do)
            results.append((out.detach(), [t.grad for t in leaves]))
            counts.append(launches["n"])
    finally:
        op.wan_flash_fwd = real_fwd
    # full checkpointing re-runs the attention forward in the backward; the
    # selective policy keeps its outputs, so it runs once
    assert counts == [1, 2, 1], counts
    base_out, base_grads = results[0]
    for out, grads in results[1:]:
        assert torch.equal(out, base_out)
        for g, g0 in zip(grads, base_grads):
            assert ((g.float() - g0.float()).norm() / g0.float().norm()).item() < 1e-3


@pytest.mark.gpu
def test_op_under_torch_compile():
    """torch.compile traces the op through its fake implementation and runs
    the kernels; forward and gradients match the eager op."""
    import wan_flash.torch_op as op
    from tests.gpu_util import seeded

    q, k, v, do = (t.cuda() for t in seeded(1, 512, 300, 2, seed=41))

    def fn(q, k, v):
        return op.wan_attention(q, k, v) * 2.0

    compiled = torch.compile(fn, backend="aot_eager", fullgraph=True)
    la = [t.clone().requires_grad_(True) for t in (q, k, v)]
    lb = [t.clone().requires_grad_(True) for t in (q, k, v)]
    oa, ob = fn(*la), compiled(*lb)
    assert torch.equal(oa, ob)
    oa.backward(do)
    ob.backward(do)
    for x, y in zip(la, lb):
        assert ((x.grad.float() - y.grad.float()).norm() / x.grad.float().norm()).item() < 1e-3


@pytest.mark.gpu
def test_op_under_torch_compile_permuted_inputs():
    """torch.compile over the op fed permuted views ((b, h, s, d) leaves
    transposed to (b, s, h, d)): the fake strides agree with the real
    contiguous outputs, so compiled and eager results and gradients match."""
    import wan_flash.torch_op as op
    from tests.gpu_util import seeded

    q, k, v, do = (t.cuda() for t in seeded(1, 512, 300, 2, seed=43))

    def fn(qh, kh, vh):
        return op.wan_attention(qh.transpose(1, 2), kh.transpose(1, 2), vh.transpose(1, 2)) * 2.0

    compiled = torch.compile(fn, backend="aot_eager", fullgraph=True)
    la = [t.transpose(1, 2).contiguous().requires_grad_(True) for t in (q, k, v)]
    lb = [t.detach().clone().requires_grad_(True) for t in la]
    oa, ob = fn(*la), compiled(*lb)
    assert torch.equal(oa, ob) and oa.stride() == ob.stride()
    oa.backward(do)
    ob.backward(do)
    for x, y in zip(la, lb):
        assert ((x.grad.float() - y.grad.float()).norm() / x.grad.float().norm()).item() < 1e-3
