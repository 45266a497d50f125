"""Device-side failure detection without a GPU fault.

Every mbarrier wait in the kernels is bounded; on expiry the kernel records
(code, block, role, barrier) in a device error word and returns instead of
trapping.  The self-test launches a wait that nothing satisfies under a short
limit: the host must read WF_ERR_WAIT_TIMEOUT with the recorded role/tag,
the word must be cleared by the read, and the context must stay usable (a
forward afterwards still matches the oracle).
"""

import ctypes

import pytest

from tests.gpu_util import assert_fwd_ok, fwd_vs_oracle, seeded

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives():
    from wan_flash import _lib

    lib = _lib.lib()
    info = (ctypes.c_uint * 4)()
    rc = lib.wf_selftest_wait_timeout(2_000_000, info)  # 2 ms limit
    assert rc == -6, (rc, _lib.last_error())
    assert info[2] == 99 and info[3] == 99  # role / barrier tag recorded by the kernel
    assert "device error -6" in _lib.last_error()
    code, _ = _lib.device_status()
    assert code == 0  # the read cleared the word
    q, k, v, _ = seeded(1, 512, 512, 2, seed=13)
    _, _, e, lse_err = fwd_vs_oracle(q, k, v)
    assert_fwd_ok(e, lse_err, "after timeout self-test")
