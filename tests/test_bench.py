"""Host logic of bench.py (no GPU): the configs, the FLOP formula of the
reference (bench/bench.py:89-93 of Quarky93/wan-flash: forward
4*b*h*sq*skv*128, backward 2.5x), and the CPU sampler of the reference arm,
including the two-context I2V config."""

import importlib.util
import pathlib

ROOT = pathlib.Path(__file__).resolve().parents[1]


def _bench():
    spec = importlib.util.spec_from_file_location("bench_module", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_configs_and_flops():
    bench = _bench()
    assert {"c2", "c3", "c3i2v", "c3dual", "c4", "c5"} <= set(bench.CONFIGS)
    kind, b, sq, skv, h, seed, _ = bench.CONFIGS["c2"]
    assert (kind, b, sq, skv, h, seed) == ("self", 1, 32760, 32760, 12, 1)
    f, fb = bench.flops(b, h, sq, skv)
    assert abs(f - 6.594e12) / 6.594e12 < 1e-3 and abs(fb / f - 2.5) < 1e-12
    f3, _ = bench.flops(1, 12, 75600, 512)
    assert abs(f3 - 237.8e9) / 237.8e9 < 1e-3


def test_cpu_sampler_single_and_dual():
    bench = _bench()
    single = bench.CpuSampler("c3")
    dual = bench.CpuSampler("c3dual")
    assert [k.shape[2] for k, _ in single.kv] == [512]
    assert [k.shape[2] for k, _ in dual.kv] == [512, bench.DUAL_IMAGE_CONTEXT]
    rows = 64
    assert dual.flops(rows) == sum(sum(bench.flops(1, 1, rows, n)) for n in (512, bench.DUAL_IMAGE_CONTEXT))
    assert single.run(rows) > 0.0 and dual.run(rows) > 0.0


def test_heads_layout_and_shared_config():
    """C4 is strong-scaled over the 40 heads (40/20/10/5 per GPU); C2 weak."""
    bench = _bench()
    for n, hp in ((1, 40), (2, 20), (4, 10), (8, 5)):
        assert bench.heads_layout("c4", n) == (hp, 40, "strong")
        cfg = bench.config_dict("c4", n)
        assert (cfg["heads_per_gpu"], cfg["heads_total"], cfg["parallelism"]) == (hp, 40, f"heads/{n}")
    assert bench.heads_layout("c2", 8) == (12, 96, "weak")
    assert bench.heads_layout("c4", 2, heads_override=3) == (3, 6, "weak")


def test_reference_arm_uses_all_cores_and_the_same_config():
    """The CPU reference arm under torchrun's OMP_NUM_THREADS=1 still runs on
    every host core, and prints the GPU arm's config object."""
    import json
    import os
    import subprocess
    import sys

    env = dict(os.environ, OMP_NUM_THREADS="1")  # what torchrun sets for its ranks
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "0", "--cpu-seconds", "0.2"], capture_output=True, text=True, env=env,
                         timeout=300, cwd=str(ROOT))
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    bench = _bench()
    assert line["impl"] == "reference" and line["config"] == bench.config_dict("c4", 1)
    assert line["cpu_baseline"]["cores"] == os.cpu_count()
    assert line["scaling"] == "strong" and line["value"] > 0


def test_timed_output_check_against_the_oracle():
    """The bench's post-timing check of its outputs (fp32 torch attention on
    slices of head 0) accepts the oracle's own outputs and flags a corrupted
    gradient; it runs on the host here."""
    import numpy as np
    import torch

    from oracle.oracle import oracle_bwd, oracle_fwd
    from tests.helpers import make_inputs, to_bhsd_f32

    bench = _bench()
    q, k, v, do = make_inputs(1, 96, 80, 2, seed=11)

    def bshd(x):  # (b, h, s, d) numpy -> (b, s, h, d) bf16 torch
        return torch.from_numpy(np.ascontiguousarray(x)).transpose(1, 2).contiguous().to(torch.bfloat16)

    o, lse = oracle_fwd(to_bhsd_f32(q), to_bhsd_f32(k), to_bhsd_f32(v))
    o_t = bshd(o)
    lse_t = torch.from_numpy(lse).float()
    dq, dk, dv = oracle_bwd(to_bhsd_f32(q), to_bhsd_f32(k), to_bhsd_f32(v), to_bhsd_f32(o_t), lse, to_bhsd_f32(do))
    errs = bench.timed_output_check(q, k, v, do, o_t, bshd(dq), bshd(dk), bshd(dv), lse_t, rows=64)
    assert all(errs[n] <= 4.5e-3 for n in ("o_rel_l2", "dq_rel_l2", "dk_rel_l2", "dv_rel_l2")), errs
    assert errs["lse_max_abs"] <= 1e-5, errs
    bad = bshd(dk) * 1.01
    assert bench.timed_output_check(q, k, v, do, o_t, bshd(dq), bad, bshd(dv), lse_t, rows=64)["dk_rel_l2"] > 4.5e-3
