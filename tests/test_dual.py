"""Two-context attention (the Wan I2V cross attention: the same query rows
attend a text context and an image context and the model adds the outputs):
``wan_flash_fwd_dual`` / ``wan_flash_bwd_dual`` / ``wan_flash_attn_dual``.

The forward gives each context exactly what a one-context call gives
(bitwise: same arithmetic per segment, one launch, Q loaded once).  The
backward adds both contexts' dQ into one accumulator, so dq matches the sum
of the one-context dq's up to the fp32 reduction order; dk/dv of each
context are its own kernel's, bitwise at nsplit = 1.  Against the oracle:
the north star's gates on every output and gradient.
"""

import numpy as np
import pytest
import torch

from oracle.oracle import error_metrics, oracle_bwd, oracle_fwd
from tests.gpu_util import LSE_ABS_TOL, REL_L2_TOL, seeded
from tests.helpers import to_bhsd_f32

pytestmark = pytest.mark.gpu

# (b, h, sq, skv0, skv1)
DUAL_SHAPES = [(1, 2, 2048, 512, 257), (2, 3, 700, 520, 33), (1, 1, 300, 1, 130), (1, 2, 1, 64, 200),
               (1, 2, 1500, 257, 512)]


def _inputs(b, h, sq, skv0, skv1, seed):
    q, k0, v0, do = seeded(b, sq, skv0, h, seed)
    _, k1, v1, _ = seeded(b, sq, skv1, h, seed + 1)
    return [t.cuda() for t in (q, k0, v0, k1, v1, do)]


@pytest.mark.parametrize("shape", DUAL_SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("scheduler,num_sms", [("auto", 0), ("single", 0), ("persistent", 3)])
def test_fwd_dual_matches_two_calls(shape, scheduler, num_sms):
    from wan_flash import _lib, features
    from wan_flash.interface import wan_flash_fwd, wan_flash_fwd_dual

    q, k0, v0, k1, v1, _ = _inputs(*shape, seed=41)
    try:
        features.set_overrides(scheduler=scheduler, num_sms=num_sms)
        o0, lse0, o1, lse1 = wan_flash_fwd_dual(q, k0, v0, k1, v1)
        _lib.check_device()
        r0, rl0 = wan_flash_fwd(q, k0, v0)
        r1, rl1 = wan_flash_fwd(q, k1, v1)
    finally:
        features.reset()
    for x, y in ((o0, r0), (lse0, rl0), (o1, r1), (lse1, rl1)):
        assert torch.equal(x, y)


# a 1-key context has dK = dQ = 0 exactly (rel_l2 against fp32 noise is
# meaningless; test_bwd_single_key covers it), so the oracle cases use 3 keys
@pytest.mark.parametrize("shape", [(1, 2, 2048, 512, 257), (2, 3, 700, 520, 33), (1, 1, 300, 3, 130)],
                         ids=lambda s: "x".join(map(str, s)))
def test_dual_vs_oracle(shape):
    """Forward outputs and the gradients of o0 + o1 against the oracle."""
    from wan_flash import _lib
    from wan_flash.interface import wan_flash_bwd_dual, wan_flash_fwd_dual

    q, k0, v0, k1, v1, do = _inputs(*shape, seed=43)
    o0, lse0, o1, lse1 = wan_flash_fwd_dual(q, k0, v0, k1, v1)
    dq, dk0, dv0, dk1, dv1 = wan_flash_bwd_dual(q, k0, v0, k1, v1, o0, lse0, o1, lse1, do)
    _lib.check_device()
    Q, K0, V0, K1, V1, DO = (to_bhsd_f32(t.cpu()) for t in (q, k0, v0, k1, v1, do))
    refs = []
    for K, V, o, lse in ((K0, V0, o0, lse0), (K1, V1, o1, lse1)):
        ro, rlse = oracle_fwd(Q, K, V)
        e = error_metrics(to_bhsd_f32(o.cpu()), ro)
        assert e["finite"] and e["rel_l2"] <= REL_L2_TOL, e
        assert float(np.abs(lse.cpu().numpy().astype(np.float64) - rlse).max()) <= LSE_ABS_TOL
        refs.append(oracle_bwd(Q, K, V, to_bhsd_f32(o.cpu()), lse.cpu().numpy(), DO))
    checks = {"dq": (dq, refs[0][0] + refs[1][0]), "dk0": (dk0, refs[0][1]), "dv0": (dv0, refs[0][2]),
              "dk1": (dk1, refs[1][1]), "dv1": (dv1, refs[1][2])}
    for name, (g, r) in checks.items():
        e = error_metrics(to_bhsd_f32(g.cpu()), r)
        assert e["finite"] and e["rel_l2"] <= REL_L2_TOL, (name, e)


def test_bwd_dual_matches_two_calls():
    from wan_flash import features
    from wan_flash.interface import wan_flash_bwd, wan_flash_bwd_dual, wan_flash_fwd_dual

    q, k0, v0, k1, v1, do = _inputs(1, 2, 2048, 512, 257, seed=47)
    o0, lse0, o1, lse1 = wan_flash_fwd_dual(q, k0, v0, k1, v1)
    features.set_bwd_overrides(nsplit=1)
    try:
        dq, dk0, dv0, dk1, dv1 = wan_flash_bwd_dual(q, k0, v0, k1, v1, o0, lse0, o1, lse1, do)
        a = wan_flash_bwd(q, k0, v0, o0, lse0, do)
        b = wan_flash_bwd(q, k1, v1, o1, lse1, do)
    finally:
        features.reset()
    for x, y in ((dk0, a[1]), (dv0, a[2]), (dk1, b[1]), (dv1, b[2])):
        assert torch.equal(x, y)
    ref = a[0].float() + b[0].float()
    assert ((dq.float() - ref).norm() / ref.norm()).item() < 4e-3


def test_attn_dual_autograd():
    """wan_flash_attn_dual = attention(q, k0, v0) + attention(q, k1, v1), with
    gradients, against fp32 torch SDPA."""
    from wan_flash.interface import wan_flash_attn_dual

    q, k0, v0, k1, v1, do = _inputs(1, 2, 640, 384, 257, seed=53)
    leaves = [t.clone().requires_grad_(True) for t in (q, k0, v0, k1, v1)]
    out = wan_flash_attn_dual(*leaves)
    out.backward(do)
    ref_leaves = [t.float().clone().requires_grad_(True) for t in (q, k0, v0, k1, v1)]
    Q, K0, V0, K1, V1 = (t.transpose(1, 2) for t in ref_leaves)
    ref = (torch.nn.functional.scaled_dot_product_attention(Q, K0, V0)
           + torch.nn.functional.scaled_dot_product_attention(Q, K1, V1)).transpose(1, 2)
    ref.backward(do.float())
    rel = lambda x, y: ((x.float() - y).norm() / y.norm()).item()  # noqa: E731
    assert rel(out, ref.detach()) <= REL_L2_TOL
    for x, y in zip(leaves, ref_leaves):
        assert rel(x.grad, y.grad) <= REL_L2_TOL


def test_bwd_dual_deterministic_bitwise():
    """deterministic=True: the shared-accumulator backward is bitwise
    reproducible (each context's main kernel adds in KV-block order; the
    contexts run one after the other)."""
    from wan_flash import _lib, features
    from wan_flash.interface import wan_flash_bwd_dual, wan_flash_fwd_dual

    q, k0, v0, k1, v1, do = _inputs(1, 2, 1500, 512, 257, seed=59)
    o0, lse0, o1, lse1 = wan_flash_fwd_dual(q, k0, v0, k1, v1)
    features.set_bwd_overrides(deterministic=True, nsplit=3)
    try:
        runs = [wan_flash_bwd_dual(q, k0, v0, k1, v1, o0, lse0, o1, lse1, do) for _ in range(3)]
        _lib.check_device()
    finally:
        features.reset()
    for g in runs[1:]:
        for a, b in zip(runs[0], g):
            assert torch.equal(a, b)
