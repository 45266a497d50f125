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
