"""wf_bwd_noalloc: the backward for callers that cannot allocate device memory.

Some callers can pass this library their tensors but cannot allocate device
memory when they call it -- a plugin host that owns every allocation and
hands over only inputs and outputs, or a latency-critical caller that cannot
take cudaMalloc's implicit synchronisation.  wf_bwd_noalloc runs the same
backward chain as the regular entry points with its workspaces in a fixed
array inside the library.  This test calls it through the C ABI and checks
it against the regular path (wan_flash_bwd, whose workspaces the Python
driver allocates) on two calls in a row with different inputs, so the
second call also shows that the shared array's leftover contents do not leak
into a result.  Collected last on purpose (file name), so a failure here
comes after every other test has run.
"""

import ctypes

import pytest
import torch

from tests.gpu_util import REL_L2_TOL, seeded

pytestmark = pytest.mark.gpu


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _noalloc_bwd(lib, q, k, v, o, lse, do):
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    b, sq, h, _ = q.shape
    skv = k.shape[1]
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.wf_bwd_noalloc(_ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(lse), _ptr(do), _ptr(dq), _ptr(dk), _ptr(dv),
                            b, sq, skv, h, stream)
    return rc, (dq, dk, dv)


def _rel(x, ref):
    return ((x.float() - ref.float()).norm() / ref.float().norm().clamp_min(1e-12)).item()


def test_noalloc_matches_regular_backward_twice():
    from wan_flash import _lib, features
    from wan_flash.interface import wan_flash_bwd, wan_flash_fwd

    lib = _lib.lib()
    features.set_bwd_overrides(nsplit=1)  # the no-alloc path does not split M
    try:
        for b, sq, skv, h, seed in ((1, 1024, 1024, 2, 21), (1, 700, 300, 3, 22)):
            q, k, v, do = (t.cuda() for t in seeded(b, sq, skv, h, seed))
            o, lse = wan_flash_fwd(q, k, v)
            ref = wan_flash_bwd(q, k, v, o, lse, do)
            rc, got = _noalloc_bwd(lib, q, k, v, o, lse, do)
            torch.cuda.synchronize()
            assert rc == 0, _lib.last_error()
            _lib.check_device()
            for name, g, r in zip(("dq", "dk", "dv"), got, ref):
                assert torch.isfinite(g.float()).all(), name
                assert _rel(g, r) <= REL_L2_TOL, (name, _rel(g, r))
            # dk / dv take the identical deterministic path at nsplit = 1
            assert torch.equal(got[1], ref[1]) and torch.equal(got[2], ref[2])
    finally:
        features.reset()


def test_noalloc_rejects_sizes_beyond_its_scratch():
    from wan_flash import _lib

    lib = _lib.lib()
    # 1 x 32768 x 4 heads -> 131072 query rows > 129024: rejected before any work
    null = ctypes.c_void_p(0)
    rc = lib.wf_bwd_noalloc(null, null, null, null, null, null, null, null, null, 1, 32768, 128, 4, null)
    assert rc == -2 and "scratch limit" in _lib.last_error()
