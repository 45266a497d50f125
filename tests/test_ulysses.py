"""Ulysses sequence<->head resharding on CPU ranks (gloo, world_size 2 and 4).

Each rank holds a sequence shard; the distributed self/cross attention (with
a CPU reference attention injected for the local part) must equal the
single-process result on the full tensors, forward and backward."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ref_attn(q, k, v):
    # (b, s, h, d) -> SDPA over (b, h, s, d), fp32 on CPU
    o = torch.nn.functional.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2))
    return o.transpose(1, 2)


def _ref_fwd(q, k, v):
    """(o, lse) of the CPU reference: lse (b, h, s) natural log."""
    scale = q.shape[-1] ** -0.5
    s = torch.einsum("bqhd,bkhd->bhqk", q, k) * scale
    lse = torch.logsumexp(s, dim=-1)
    o = torch.einsum("bhqk,bkhd->bqhd", torch.softmax(s, dim=-1), v)
    return o, lse


def _ref_bwd(q, k, v, o, lse, do):
    qq, kk, vv = (t.detach().clone().requires_grad_(True) for t in (q, k, v))
    with torch.enable_grad():
        oo, _ = _ref_fwd(qq, kk, vv)
        oo.backward(do)
    return qq.grad, kk.grad, vv.grad


def _worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from wan_flash import ulysses

        torch.manual_seed(0)
        b, S, H, D, L = 1, 24, 8, 16, 10
        q = torch.randn(b, S, H, D)
        k = torch.randn(b, S, H, D)
        v = torch.randn(b, S, H, D)
        ck = torch.randn(b, L, H, D)
        cv = torch.randn(b, L, H, D)
        go = torch.randn(b, S, H, D)
        go2 = torch.randn(b, S, H, D)
        s_loc = S // world
        sl = slice(rank * s_loc, (rank + 1) * s_loc)

        # raw resharding round trip
        x = q[:, sl].contiguous()
        xh = ulysses.seq_to_head(x)
        assert xh.shape == (b, S, H // world, D)
        assert torch.equal(xh, q[:, :, rank * (H // world):(rank + 1) * (H // world)])
        assert torch.equal(ulysses.head_to_seq(xh), x)

        # self attention, forward + backward
        ql, kl, vl = (t[:, sl].clone().requires_grad_(True) for t in (q, k, v))
        o = ulysses.ulysses_self_attention(ql, kl, vl, attn_fn=_ref_attn)
        o.backward(go[:, sl])
        qf, kf, vf = (t.clone().requires_grad_(True) for t in (q, k, v))
        of = _ref_attn(qf, kf, vf)
        of.backward(go)
        torch.testing.assert_close(o, of[:, sl].detach(), rtol=1e-5, atol=1e-5)
        for g, gf in zip((ql.grad, kl.grad, vl.grad), (qf.grad, kf.grad, vf.grad)):
            torch.testing.assert_close(g, gf[:, sl], rtol=1e-5, atol=1e-5)

        # cross attention against a replicated context
        ql2 = q[:, sl].clone().requires_grad_(True)
        ckl, cvl = ck.clone().requires_grad_(True), cv.clone().requires_grad_(True)
        o2 = ulysses.ulysses_cross_attention(ql2, ckl, cvl, attn_fn=_ref_attn)
        o2.backward(go2[:, sl])
        qf2, ckf, cvf = (t.clone().requires_grad_(True) for t in (q, ck, cv))
        of2 = _ref_attn(qf2, ckf, cvf)
        of2.backward(go2)
        torch.testing.assert_close(o2, of2[:, sl].detach(), rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(ql2.grad, qf2.grad[:, sl], rtol=1e-5, atol=1e-5)
        # every replica of the context receives the full gradient (all heads, all queries)
        torch.testing.assert_close(ckl.grad, ckf.grad, rtol=1e-4, atol=1e-5)
        torch.testing.assert_close(cvl.grad, cvf.grad, rtol=1e-4, atol=1e-5)

        # the whole block (self + cross sharing one exchanged q, overlapped exchanges)
        qb, kb, vb = (t[:, sl].clone().requires_grad_(True) for t in (q, k, v))
        ckb, cvb = ck.clone().requires_grad_(True), cv.clone().requires_grad_(True)
        o_s, o_c = ulysses.ulysses_attention_block(qb, kb, vb, ckb, cvb, fwd=_ref_fwd, bwd=_ref_bwd)
        torch.autograd.backward((o_s, o_c), (go[:, sl], go2[:, sl]))
        qf3, kf3, vf3, ckf3, cvf3 = (t.clone().requires_grad_(True) for t in (q, k, v, ck, cv))
        os_f, oc_f = _ref_attn(qf3, kf3, vf3), _ref_attn(qf3, ckf3, cvf3)
        torch.autograd.backward((os_f, oc_f), (go, go2))
        torch.testing.assert_close(o_s, os_f[:, sl].detach(), rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(o_c, oc_f[:, sl].detach(), rtol=1e-5, atol=1e-5)
        for g, gf in zip((qb.grad, kb.grad, vb.grad), (qf3.grad, kf3.grad, vf3.grad)):
            torch.testing.assert_close(g, gf[:, sl], rtol=1e-4, atol=1e-5)
        torch.testing.assert_close(ckb.grad, ckf3.grad, rtol=1e-4, atol=1e-5)
        torch.testing.assert_close(cvb.grad, cvf3.grad, rtol=1e-4, atol=1e-5)

        # only the self output reaches the loss: the cross output's gradient
        # arrives as None and is exchanged as zeros of its (b, S/P, H, D) shape
        qb, kb, vb = (t[:, sl].clone().requires_grad_(True) for t in (q, k, v))
        ckb, cvb = ck.clone().requires_grad_(True), cv.clone().requires_grad_(True)
        o_s, _ = ulysses.ulysses_attention_block(qb, kb, vb, ckb, cvb, fwd=_ref_fwd, bwd=_ref_bwd)
        o_s.backward(go[:, sl])
        qf4, kf4, vf4 = (t.clone().requires_grad_(True) for t in (q, k, v))
        _ref_attn(qf4, kf4, vf4).backward(go)
        for g, gf in zip((qb.grad, kb.grad, vb.grad), (qf4.grad, kf4.grad, vf4.grad)):
            torch.testing.assert_close(g, gf[:, sl], rtol=1e-4, atol=1e-5)
        assert float(ckb.grad.abs().max()) == 0.0 and float(cvb.grad.abs().max()) == 0.0
        result_q.put((rank, "ok"))
    except Exception as e:  # report to the parent
        result_q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_ulysses_matches_single_process(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=180) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert all(v == "ok" for v in results.values()), results
