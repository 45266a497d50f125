"""Empty and degenerate problems through the public API on the GPU: no
kernel work, outputs of the contract's shapes, zero gradients where the
sum is empty, and the contract's AssertionError for attention over an
empty key set."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _t(b, s, h):
    return torch.randn(b, s, h, 128, device="cuda").to(torch.bfloat16)


@pytest.mark.parametrize("b,sq,skv,h", [(0, 64, 64, 2), (1, 0, 64, 2), (1, 64, 64, 0), (2, 0, 130, 3)])
def test_fwd_bwd_empty(b, sq, skv, h):
    from wan_flash import _lib
    from wan_flash.interface import wan_flash_bwd, wan_flash_fwd

    q, k, v, do = _t(b, sq, h), _t(b, skv, h), _t(b, skv, h), _t(b, sq, h)
    o, lse = wan_flash_fwd(q, k, v)
    assert o.shape == q.shape and o.dtype == torch.bfloat16
    assert lse.shape == (b, h, sq) and lse.dtype == torch.float32
    dq, dk, dv = wan_flash_bwd(q, k, v, o, lse, do)
    _lib.check_device()
    assert (dq.shape, dk.shape, dv.shape) == (q.shape, k.shape, v.shape)
    # no query rows: the sums over queries are empty
    assert dk.float().abs().sum().item() == 0.0 and dv.float().abs().sum().item() == 0.0


def test_fwd_empty_key_set_is_an_error():
    from wan_flash.interface import wan_flash_fwd

    q, k = _t(1, 64, 2), _t(1, 0, 2)
    with pytest.raises(AssertionError):
        wan_flash_fwd(q, k, k)


def test_bwd_empty_key_set_gives_zero_dq():
    from wan_flash import _lib
    from wan_flash.interface import wan_flash_bwd

    q, k, do = _t(1, 64, 2), _t(1, 0, 2), _t(1, 64, 2)
    lse = torch.zeros(1, 2, 64, device="cuda")
    dq, dk, dv = wan_flash_bwd(q, k, k, q, lse, do)
    _lib.check_device()
    assert dq.float().abs().sum().item() == 0.0 and dk.numel() == 0 and dv.numel() == 0


def test_dual_empty_queries():
    from wan_flash import _lib
    from wan_flash.interface import wan_flash_bwd_dual, wan_flash_fwd_dual

    q, k0, k1, do = _t(1, 0, 2), _t(1, 512, 2), _t(1, 257, 2), _t(1, 0, 2)
    o0, lse0, o1, lse1 = wan_flash_fwd_dual(q, k0, k0, k1, k1)
    assert o0.shape == o1.shape == q.shape and lse0.shape == lse1.shape == (1, 2, 0)
    dq, dk0, dv0, dk1, dv1 = wan_flash_bwd_dual(q, k0, k0, k1, k1, o0, lse0, o1, lse1, do)
    _lib.check_device()
    assert all(t.float().abs().sum().item() == 0.0 for t in (dk0, dv0, dk1, dv1))
