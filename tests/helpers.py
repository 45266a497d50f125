"""Shared test helpers: seeded inputs and golden-fixture loaders.

Inputs are drawn on torch's CPU generator so that the same seed gives the
same bf16 tensors here and on a GPU box (same image, same torch build).
"""

from __future__ import annotations

import json
import pathlib

import numpy as np
import torch

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"


def make_inputs(b, sq, skv, h, seed, std=1.0, d=128):
    """Seeded bf16 (q, k, v, dO) in (b, s, h, d).

    Draw order q, k, v, dO follows the reference tests (``tests/test_bwd.py:46-50``
    of Quarky93/wan-flash).  Values are drawn in fp32, q and k are multiplied
    by ``std`` (the N(0, 2^2) rescale-stress variant uses 2.0), then cast to
    bf16 with round-to-nearest-even.
    """
    torch.manual_seed(seed)
    q = torch.randn(b, sq, h, d, dtype=torch.float32)
    k = torch.randn(b, skv, h, d, dtype=torch.float32)
    v = torch.randn(b, skv, h, d, dtype=torch.float32)
    do = torch.randn(b, sq, h, d, dtype=torch.float32)
    q, k = q * std, k * std
    return tuple(t.to(torch.bfloat16) for t in (q, k, v, do))


def load_npz_case(name):
    """-> (inputs dict of bf16 torch tensors in (b,s,h,d), outputs dict of fp32 numpy, meta)."""
    z = np.load(GOLDEN / f"{name}.npz")
    ins = {
        key: torch.from_numpy(z[key].astype(np.int16)).view(torch.bfloat16)
        for key in ("q", "k", "v", "do")
    }
    outs = {key: z[key] for key in ("o", "lse", "dq", "dk", "dv")}
    return ins, outs, z["meta"].tolist()


def load_checksums():
    return json.loads((GOLDEN / "checksums.json").read_text())


NPZ_CASE_NAMES = ["self_s160_h1", "cross_s136_kv77_h2", "self_s130_h1_std2"]


def to_bhsd_f32(t: torch.Tensor) -> np.ndarray:
    """(b,s,h,d) torch tensor -> (b,h,s,d) float32 numpy (oracle layout)."""
    return t.detach().float().cpu().transpose(1, 2).contiguous().numpy()
