"""Ulysses sequence-parallel attention over NCCL with the sm_100a kernels.

Needs >= 2 GPUs (skipped otherwise).  Two ranks hold sequence shards of
q/k/v; wan_flash_attn runs on head shards after the all-to-all; the
sequence-sharded output and gradients must match a single-GPU
wan_flash_attn on the full tensors (same kernels, so the comparison is at
bf16 output rounding: rel_l2 <= 1e-2 leaves room for the different fp32
reduction order of dq).
"""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q_):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    from datetime import timedelta

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from wan_flash import ulysses
        from wan_flash.interface import wan_flash_attn

        torch.manual_seed(0)
        b, S, H, D, L = 1, 2048, 4, 128, 512
        q, k, v, go = (torch.randn(b, S, H, D, dtype=torch.float32).to(torch.bfloat16) for _ in range(4))
        ck, cv = (torch.randn(b, L, H, D, dtype=torch.float32).to(torch.bfloat16) for _ in range(2))
        dev = torch.device("cuda", rank)
        s_loc = S // world
        sl = slice(rank * s_loc, (rank + 1) * s_loc)

        def rel(x, y):
            return ((x.float() - y.float()).norm() / y.float().norm()).item()

        # self attention
        ql, kl, vl = (t[:, sl].to(dev).requires_grad_(True) for t in (q, k, v))
        o = ulysses.ulysses_self_attention(ql, kl, vl)
        o.backward(go[:, sl].to(dev))
        qf, kf, vf = (t.to(dev).requires_grad_(True) for t in (q, k, v))
        of = wan_flash_attn(qf, kf, vf)
        of.backward(go.to(dev))
        errs = [rel(o, of[:, sl].detach())] + [rel(g, gf[:, sl]) for g, gf in zip((ql.grad, kl.grad, vl.grad),
                                                                                   (qf.grad, kf.grad, vf.grad))]
        # cross attention against a replicated context
        ql2 = q[:, sl].to(dev).requires_grad_(True)
        ckl, cvl = ck.to(dev).requires_grad_(True), cv.to(dev).requires_grad_(True)
        o2 = ulysses.ulysses_cross_attention(ql2, ckl, cvl)
        o2.backward(go[:, sl].to(dev))
        qf2, ckf, cvf = q.to(dev).requires_grad_(True), ck.to(dev).requires_grad_(True), cv.to(dev).requires_grad_(True)
        of2 = wan_flash_attn(qf2, ckf, cvf)
        of2.backward(go.to(dev))
        errs += [rel(o2, of2[:, sl].detach()), rel(ql2.grad, qf2.grad[:, sl]), rel(ckl.grad, ckf.grad),
                 rel(cvl.grad, cvf.grad)]
        # the whole block: one exchanged q for both attentions, overlapped exchanges
        go2 = torch.randn(b, S, H, D, dtype=torch.float32).to(torch.bfloat16)
        qb, kb, vb = (t[:, sl].to(dev).requires_grad_(True) for t in (q, k, v))
        ckb, cvb = ck.to(dev).requires_grad_(True), cv.to(dev).requires_grad_(True)
        o_s, o_c = ulysses.ulysses_attention_block(qb, kb, vb, ckb, cvb)
        torch.autograd.backward((o_s, o_c), (go[:, sl].to(dev), go2[:, sl].to(dev)))
        qf3, kf3, vf3, ckf3, cvf3 = (t.to(dev).requires_grad_(True) for t in (q, k, v, ck, cv))
        os_f, oc_f = wan_flash_attn(qf3, kf3, vf3), wan_flash_attn(qf3, ckf3, cvf3)
        torch.autograd.backward((os_f, oc_f), (go.to(dev), go2.to(dev)))
        errs += [rel(o_s, os_f[:, sl].detach()), rel(o_c, oc_f[:, sl].detach())]
        errs += [rel(g, gf[:, sl]) for g, gf in zip((qb.grad, kb.grad, vb.grad), (qf3.grad, kf3.grad, vf3.grad))]
        errs += [rel(ckb.grad, ckf3.grad), rel(cvb.grad, cvf3.grad)]
        q_.put((rank, errs))
    except Exception as e:  # report to the parent
        q_.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ulysses_nccl_matches_single_gpu():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q_ = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q_)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q_.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
    for rank, errs in results.items():
        assert isinstance(errs, list), errs
        assert all(e <= 1e-2 for e in errs), (rank, errs)
