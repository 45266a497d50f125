"""Generate the golden fixtures that pin ``oracle/oracle.py`` to the reference.

Run in a container where the reference checkout is readable::

    python tests/golden/make_golden.py --reference <path-to-wan-flash-checkout>

It imports the reference's own chunked-fp32 torch oracle
(``tests/oracle.py`` of Quarky93/wan-flash, functions ``oracle_fwd`` at
lines 14-31 and ``oracle_bwd`` at lines 34-52) by file path, feeds it seeded
bf16 inputs drawn in the reference tests' order (``torch.manual_seed(seed)``,
then q, k, v, dO from ``torch.randn`` in (b, s, h, d) -- ``tests/test_bwd.py:46-50``;
drawn in fp32 on the CPU generator, q/k scaled by the case's std, then cast
to bf16; see ``tests/helpers.make_inputs``), and writes

* ``<case>.npz`` for small cases: bf16 input bit patterns plus the oracle's
  fp32 o / lse / dq / dk / dv, and
* ``checksums.json`` for the larger cases (the C1 tiny config and a case that
  crosses the oracle's 2048-row chunk boundary): norms, sums and sampled
  elements of every output.

The fixtures are consumed by ``tests/test_oracle.py`` (oracle pinning, CPU)
and by the GPU parity tests.  Nothing at run time reads the reference.
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import pathlib
import sys

import numpy as np
import torch

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))
from tests.helpers import make_inputs  # noqa: E402

# name, (b, sq, skv, h), seed, q/k std
NPZ_CASES = [
    ("self_s160_h1", (1, 160, 160, 1), 0, 1.0),
    ("cross_s136_kv77_h2", (1, 136, 77, 2), 0, 1.0),
    ("self_s130_h1_std2", (1, 130, 130, 1), 1, 2.0),
]
SUM_CASES = [
    ("tiny_c1_s2048_h2", (1, 2048, 2048, 2), 0, 1.0),
    ("chunked_s2100_kv96_h1", (1, 2100, 96, 1), 3, 1.0),
]


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _load_ref_oracle(ref_root: pathlib.Path):
    spec = importlib.util.spec_from_file_location("_ref_oracle", ref_root / "tests" / "oracle.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _run_ref(mod, q, k, v, do):
    qh, kh, vh, doh = (t.transpose(1, 2) for t in (q, k, v, do))
    o, lse = mod.oracle_fwd(qh, kh, vh)
    dq, dk, dv = mod.oracle_bwd(qh, kh, vh, o, lse, doh)
    return {"o": o, "lse": lse, "dq": dq, "dk": dk, "dv": dv}


def summarize(arr: np.ndarray) -> dict:
    flat = np.asarray(arr, dtype=np.float64).ravel()
    idx = np.linspace(0, flat.size - 1, num=16).astype(np.int64)
    return {
        "shape": list(arr.shape),
        "sum": float(flat.sum()),
        "abs_sum": float(np.abs(flat).sum()),
        "l2": float(np.linalg.norm(flat)),
        "sample_idx": idx.tolist(),
        "sample": flat[idx].tolist(),
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=pathlib.Path)
    args = ap.parse_args()
    mod = _load_ref_oracle(args.reference)
    torch.set_num_threads(8)

    for name, (b, sq, skv, h), seed, std in NPZ_CASES:
        q, k, v, do = make_inputs(b, sq, skv, h, seed, std)
        out = _run_ref(mod, q, k, v, do)
        np.savez_compressed(
            HERE / f"{name}.npz",
            q=_bits(q), k=_bits(k), v=_bits(v), do=_bits(do),
            meta=np.array([b, sq, skv, h, seed], dtype=np.int64), std=np.float32(std),
            **{key: val.numpy().astype(np.float32) for key, val in out.items()},
        )
        print("wrote", name)

    sums = {}
    for name, (b, sq, skv, h), seed, std in SUM_CASES:
        q, k, v, do = make_inputs(b, sq, skv, h, seed, std)
        out = _run_ref(mod, q, k, v, do)
        sums[name] = {
            "shape": [b, sq, skv, h], "seed": seed, "std": std,
            "input_l2": {n: float(t.float().norm()) for n, t in zip(("q", "k", "v", "do"), (q, k, v, do))},
            **{key: summarize(val.numpy()) for key, val in out.items()},
        }
        print("summed", name)
    (HERE / "checksums.json").write_text(json.dumps(sums, indent=1))


if __name__ == "__main__":
    main()
