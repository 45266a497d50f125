"""Pin the numpy oracle (oracle/oracle.py) to the reference's own torch oracle.

The fixtures under tests/golden/ were produced by running the reference's
``tests/oracle.py`` (Quarky93/wan-flash) on seeded inputs; see
tests/golden/make_golden.py.  Both sides compute in fp32, so agreement is
at fp32 rounding level (only matmul summation order differs).
"""

import numpy as np
import pytest

from oracle.oracle import (
    bf16_bits_to_f32, error_metrics, f32_to_bf16_bits, oracle_bwd, oracle_fwd, round_bf16,
)
from tests.helpers import NPZ_CASE_NAMES, load_checksums, load_npz_case, make_inputs, to_bhsd_f32

FP32_REL = 2e-6


def _run_oracle(ins):
    q, k, v, do = (to_bhsd_f32(ins[n]) for n in ("q", "k", "v", "do"))
    o, lse = oracle_fwd(q, k, v)
    dq, dk, dv = oracle_bwd(q, k, v, o, lse, do)
    return {"o": o, "lse": lse, "dq": dq, "dk": dk, "dv": dv}


@pytest.mark.parametrize("name", NPZ_CASE_NAMES)
def test_oracle_matches_reference_fixture(name):
    ins, ref, _ = load_npz_case(name)
    got = _run_oracle(ins)
    for key in ("o", "dq", "dk", "dv"):
        e = error_metrics(got[key], ref[key])
        assert e["finite"] and e["rel_l2"] < FP32_REL, (name, key, e)
    assert np.abs(got["lse"] - ref["lse"]).max() < 1e-5


@pytest.mark.parametrize("name", ["tiny_c1_s2048_h2", "chunked_s2100_kv96_h1"])
def test_oracle_matches_reference_checksums(name):
    spec = load_checksums()[name]
    b, sq, skv, h = spec["shape"]
    ins = dict(zip(("q", "k", "v", "do"), make_inputs(b, sq, skv, h, spec["seed"], spec["std"])))
    # the inputs themselves must be the ones the fixture was made from
    for n, t in ins.items():
        assert abs(float(t.float().norm()) - spec["input_l2"][n]) <= 1e-4 * spec["input_l2"][n]
    got = _run_oracle(ins)
    for key in ("o", "lse", "dq", "dk", "dv"):
        s = spec[key]
        arr = got[key].astype(np.float64)
        assert list(arr.shape) == s["shape"]
        assert abs(np.linalg.norm(arr) - s["l2"]) <= 1e-5 * s["l2"], key
        assert abs(np.abs(arr).sum() - s["abs_sum"]) <= 1e-5 * s["abs_sum"], key
        sample = arr.ravel()[s["sample_idx"]]
        scale = max(1.0, np.abs(s["sample"]).max())
        assert np.allclose(sample, s["sample"], rtol=1e-4, atol=1e-5 * scale), key


def test_bf16_roundtrip_matches_torch():
    import torch

    x = torch.randn(4096, dtype=torch.float32) * 7.0
    x[:4] = torch.tensor([0.0, -0.0, 1e-40, 3.4e38])
    ours = f32_to_bf16_bits(x.numpy())
    theirs = x.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(ours, theirs)
    assert np.array_equal(bf16_bits_to_f32(ours), x.to(torch.bfloat16).float().numpy())
    assert np.array_equal(round_bf16(x.numpy()), x.to(torch.bfloat16).float().numpy())


def test_oracle_lse_is_natural_log_and_softmax_normalised():
    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal((1, 1, 64, 128)).astype(np.float32) for _ in range(3))
    o, lse = oracle_fwd(q, k, v)
    s = q[0, 0] @ k[0, 0].T / np.sqrt(128)
    p = np.exp(s - lse[0, 0][:, None])
    assert np.allclose(p.sum(-1), 1.0, atol=1e-5)
    assert np.allclose(o[0, 0], p @ v[0, 0], atol=1e-5)


def test_oracle_on_row_and_key_slices():
    """The oracle called on a slice of query rows returns exactly those rows
    of O, LSE and dQ, and called on a slice of keys (every query row, the
    given o / lse) exactly those rows of dK and dV: the 75600-token parity
    test checks the GPU result on such slices."""
    q, k, v, do = make_inputs(1, 3000, 3000, 1, seed=3)
    Q, K, V, DO = (to_bhsd_f32(t) for t in (q, k, v, do))
    O, LSE = oracle_fwd(Q, K, V)
    fdq, fdk, fdv = oracle_bwd(Q, K, V, O, LSE, DO)
    for sl in (slice(0, 512), slice(1536 + 64, 2112), slice(2488, 3000)):
        ro, rl = oracle_fwd(Q[:, :, sl], K, V)
        assert np.allclose(ro, O[:, :, sl], rtol=1e-5, atol=1e-6) and np.allclose(rl, LSE[:, :, sl], atol=1e-6)
        rdq, _, _ = oracle_bwd(Q[:, :, sl], K, V, O[:, :, sl], LSE[:, :, sl], DO[:, :, sl])
        assert np.allclose(rdq, fdq[:, :, sl], rtol=1e-4, atol=1e-6)
        _, rdk, rdv = oracle_bwd(Q, K[:, :, sl], V[:, :, sl], O, LSE, DO)
        assert np.allclose(rdk, fdk[:, :, sl], rtol=1e-4, atol=1e-6)
        assert np.allclose(rdv, fdv[:, :, sl], rtol=1e-4, atol=1e-6)
