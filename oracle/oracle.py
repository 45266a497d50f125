"""CPU oracle for the Wan attention hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this module, and only as the checker.  The product path
(``wan_flash.interface``) never calls it and has no CPU fallback.

This is a numpy restatement of the reference's chunked-fp32 oracle
(``tests/oracle.py`` of Quarky93/wan-flash):

* ``oracle_fwd``  follows ``tests/oracle.py:14-31``: per (batch, head) and per
  2048-row chunk of queries, ``s = (q @ k.T) * scale``, ``lse = logsumexp(s)``
  (natural log), ``o = exp(s - lse) @ v``; everything in fp32.
* ``oracle_bwd``  follows ``tests/oracle.py:34-52``: P is recomputed from the
  *given* lse, ``D = rowsum(dO * O)`` from the *given* o,
  ``dS = P * (dO @ v.T - D) * scale``, ``dq = dS @ k``, ``dk += dS.T @ q``,
  ``dv += P.T @ dO``.
* ``error_metrics`` follows ``tests/oracle.py:55-61`` (max_abs, rel_l2,
  finite).

Layout convention is the reference oracle's: tensors are (b, h, s, d) and
lse is (b, h, s).  Inputs may be any float dtype (bf16 arrives as float32
values that are exactly representable in bf16).

Parity pin: ``tests/golden/make_golden.py`` runs the reference's own torch
oracle on seeded inputs and stores the results under ``tests/golden/``;
``tests/test_oracle.py`` checks this restatement against them.
"""

from __future__ import annotations

import math

import numpy as np

CHUNK = 2048  # rows of q per step, as tests/oracle.py:11


def _f32(x):
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32))


def _logsumexp_rows(s: np.ndarray) -> np.ndarray:
    m = s.max(axis=-1)
    # rows of all -inf give -inf, like torch.logsumexp
    m_safe = np.where(np.isfinite(m), m, 0.0).astype(np.float32)
    return (np.log(np.exp(s - m_safe[:, None]).sum(axis=-1, dtype=np.float32)) + m_safe).astype(np.float32)


def oracle_fwd(q, k, v, scale: float | None = None):
    """q (b,h,sq,d), k/v (b,h,skv,d) -> (o (b,h,sq,d) fp32, lse (b,h,sq) fp32, natural log)."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    b, h, sq, d = q.shape
    scale = np.float32(scale if scale is not None else 1.0 / math.sqrt(d))
    o = np.empty((b, h, sq, d), dtype=np.float32)
    lse = np.empty((b, h, sq), dtype=np.float32)
    for bi in range(b):
        for hi in range(h):
            kq, kk, kv = q[bi, hi], k[bi, hi], v[bi, hi]
            for i0 in range(0, sq, CHUNK):
                i1 = min(i0 + CHUNK, sq)
                s = (kq[i0:i1] @ kk.T) * scale
                l = _logsumexp_rows(s)
                o[bi, hi, i0:i1] = np.exp(s - l[:, None]) @ kv
                lse[bi, hi, i0:i1] = l
    return o, lse


def oracle_bwd(q, k, v, o, lse, do, scale: float | None = None):
    """Analytic backward from the given (o, lse): returns (dq, dk, dv) fp32 in (b,h,s,d)."""
    q, k, v, o, lse, do = (_f32(t) for t in (q, k, v, o, lse, do))
    b, h, sq, d = q.shape
    scale = np.float32(scale if scale is not None else 1.0 / math.sqrt(d))
    dq = np.zeros_like(q)
    dk = np.zeros_like(k)
    dv = np.zeros_like(v)
    for bi in range(b):
        for hi in range(h):
            kq, kk, kv = q[bi, hi], k[bi, hi], v[bi, hi]
            ko, kl, kdo = o[bi, hi], lse[bi, hi], do[bi, hi]
            D = (kdo * ko).sum(-1, dtype=np.float32)
            for i0 in range(0, sq, CHUNK):
                i1 = min(i0 + CHUNK, sq)
                p = np.exp((kq[i0:i1] @ kk.T) * scale - kl[i0:i1, None])
                ds = p * (kdo[i0:i1] @ kv.T - D[i0:i1, None]) * scale
                dq[bi, hi, i0:i1] = ds @ kk
                dk[bi, hi] += ds.T @ kq[i0:i1]
                dv[bi, hi] += p.T @ kdo[i0:i1]
    return dq, dk, dv


def error_metrics(x, ref) -> dict:
    """max_abs, rel_l2 and finiteness of ``x`` against ``ref`` (tests/oracle.py:55-61)."""
    x = np.asarray(x, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    diff = x - ref
    return {
        "max_abs": float(np.abs(diff).max()) if diff.size else 0.0,
        "rel_l2": float(np.linalg.norm(diff) / max(np.linalg.norm(ref), 1e-12)),
        "finite": bool(np.isfinite(x).all()),
    }


# ---------------------------------------------------------------------------
# bf16 helpers (inputs are bf16 on the GPU; the oracle works on their exact
# fp32 values).  Round-to-nearest-even, like torch's float->bfloat16 cast.
# ---------------------------------------------------------------------------

def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns -> float32 values."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> uint16 bf16 bit patterns, round to nearest even (NaN kept quiet)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    out = rounded.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bf16 value (returned as float32)."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))
