"""Helpers shared by the GPU parity tests: run the CUDA path on seeded
inputs and compare with the numpy oracle (oracle/oracle.py)."""

from __future__ import annotations

import numpy as np
import torch

from oracle.oracle import error_metrics, oracle_bwd, oracle_fwd
from tests.helpers import make_inputs, to_bhsd_f32

# Tolerances stated by the north star: O/dQ/dK/dV rel_l2 <= 2x the bf16
# floor (~4.5e-3); natural-log LSE max abs error <= 1e-5.
REL_L2_TOL = 4.5e-3
LSE_ABS_TOL = 1e-5


def to_cuda(*ts):
    return tuple(t.to("cuda") for t in ts)


def fwd_vs_oracle(q, k, v):
    """Run wan_flash_fwd on cuda copies of (q, k, v); return (o, lse, o_err, lse_err, oracle)."""
    from wan_flash import _lib
    from wan_flash.interface import wan_flash_fwd

    qc, kc, vc = to_cuda(q, k, v)
    o, lse = wan_flash_fwd(qc, kc, vc)
    _lib.check_device()
    ro, rlse = oracle_fwd(to_bhsd_f32(q), to_bhsd_f32(k), to_bhsd_f32(v))
    e = error_metrics(to_bhsd_f32(o), ro)
    lse_err = float(np.abs(lse.cpu().numpy().astype(np.float64) - rlse).max()) if lse.numel() else 0.0
    return o, lse, e, lse_err


def bwd_vs_oracle(q, k, v, do, o=None, lse=None):
    """Run wan_flash_bwd with the given (or our own forward's) o/lse; compare each grad."""
    from wan_flash import _lib
    from wan_flash.interface import wan_flash_bwd, wan_flash_fwd

    qc, kc, vc, doc = to_cuda(q, k, v, do)
    if o is None:
        o, lse = wan_flash_fwd(qc, kc, vc)
    else:
        o, lse = o.to("cuda"), lse.to("cuda")
    grads = wan_flash_bwd(qc, kc, vc, o, lse, doc)
    _lib.check_device()
    refs = oracle_bwd(to_bhsd_f32(q), to_bhsd_f32(k), to_bhsd_f32(v), to_bhsd_f32(o),
                      lse.float().cpu().numpy(), to_bhsd_f32(do))
    errs = {name: error_metrics(to_bhsd_f32(g), r) for name, g, r in zip(("dq", "dk", "dv"), grads, refs)}
    return grads, errs


def seeded(b, sq, skv, h, seed=0, std=1.0):
    return make_inputs(b, sq, skv, h, seed, std)


def assert_fwd_ok(e, lse_err, tag=""):
    assert e["finite"], f"{tag}: non-finite O"
    assert e["rel_l2"] <= REL_L2_TOL, f"{tag}: O rel_l2 {e['rel_l2']:.3e}"
    assert lse_err <= LSE_ABS_TOL, f"{tag}: LSE abs err {lse_err:.3e}"


def assert_bwd_ok(errs, tag=""):
    for name, e in errs.items():
        assert e["finite"], f"{tag}: non-finite {name}"
        assert e["rel_l2"] <= REL_L2_TOL, f"{tag}: {name} rel_l2 {e['rel_l2']:.3e}"


def cuda_ok() -> bool:
    return torch.cuda.is_available()
