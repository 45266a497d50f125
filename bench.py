"""Benchmark of the Wan attention hot path (forward + backward) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2|c3|c3i2v|c4|c5]
                    [--impl ours|reference]

One step = wan_flash_fwd + wan_flash_bwd over one batch of synthetic bf16
inputs of the configured Wan shape (default C4: Wan2.1-14B 720p
self-attention, b=1, s=75600, 40 heads, d=128, q/k/v/dO ~ N(0,1), seed 3,
head-sharded over the GPUs: 40/N heads per rank).
TFLOP/s counts 4*b*h*sq*skv*128 for the forward and 2.5x that for the
backward (the reference's convention, bench/bench.py:89-93).

Multi-GPU (torchrun, one rank per GPU): the work shards by heads with no
data-path collective.  C4 (Wan2.1-14B 720p, 40 heads) runs as strong scaling
(40/N heads per rank); C2 and the cross-attention configs run as weak
scaling (every rank owns the config's heads of an N-times-larger problem).
C5 is the sequence-parallel Wan block: activations sequence-sharded
(1, 75600/N, 40, 128) per rank, Ulysses all-to-all to head shards, self- and
cross-attention forward + backward, all-to-all back; it reports the exposed
communication (step time minus the same attention work without the
exchanges) and checks its outputs and query gradient against attention
computed without the all-to-all (full K/V gathered along the sequence).  At
N > 1 the default C4 run also runs the C5 block in the same invocation and
adds it to the line as ``sp_block``.  Time is the max over ranks of
CUDA-event time.

Printed (rank 0): one JSON line with value (whole-job TFLOP/s, inputs
resident in HBM), e2e (same metric through the public API with every step's
inputs copied from pinned host memory and its o/dq/dk/dv copied back inside
the timed region; copies on a second stream overlap neighbouring steps), the
roofline of the dominant kernel, a CPU baseline (the oracle
port on the host cores, bounded sample), clocks sampled during the timed
region, and the number of our kernel launches.

``--impl reference`` times the reference's algorithm on the host cores: the
reference ships no CPU implementation other than its chunked-fp32 torch
oracle (tests/oracle.py), so this arm runs the numpy port of that oracle
(oracle/oracle.py) with all host threads on a bounded sample of the same
workload.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import pathlib
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CONFIGS = {
    # name: (kind, b, sq, skv, h_total, seed, description)
    "c2": ("self", 1, 32760, 32760, 12, 1, "Wan2.1-1.3B 480p self-attention fwd+bwd (b=1, s=32760, h=12, d=128)"),
    "c3": ("cross", 1, 75600, 512, 12, 2, "Wan2.1 cross-attention fwd+bwd (sq=75600, skv=512, h=12)"),
    "c3i2v": ("cross", 1, 75600, 257, 12, 2, "Wan2.1 I2V image cross-attention fwd+bwd (sq=75600, skv=257, h=12)"),
    # the I2V block's two cross attentions with the same Q (text 512 + image 257), one
    # two-context launch forward and a shared dQ accumulator backward; kv_len is the text context
    "c3dual": ("dual", 1, 75600, 512, 12, 2, "Wan2.1 I2V cross-attention, text (skv=512) + image (skv=257) "
               "contexts of the same Q, fwd+bwd (sq=75600, h=12)"),
    "c4": ("self", 1, 75600, 75600, 40, 3, "Wan2.1-14B 720p self-attention fwd+bwd, head-sharded (b=1, s=75600, h=40)"),
    # the sequence-parallel block: self-attention over 75600 tokens plus cross-attention against
    # a 512-token context, activations sequence-sharded; the CPU arm samples its self-attention part
    "c5": ("self", 1, 75600, 75600, 40, 4, "Wan2.1-14B 720p sequence-parallel block: Ulysses all-to-all, "
           "self (75600) + cross (512) attention fwd+bwd, all-to-all back (b=1, h=40)"),
}
C5_CONTEXT = 512
DUAL_IMAGE_CONTEXT = 257
METRIC = "fwd and bwd TFLOP/s per B200 at Wan shapes; % of bf16 dense peak; 1/2/4/8-GPU"
# DRAM bytes (read + write) per launch per head, from one ncu capture of the
# C2 shape at 4 heads (profiles/wf_bwd_main_c2_h4.md, profiles/wf_fwd2_c2_h4.md);
# traffic grows with the number of heads, so it is scaled by the run's heads.
DRAM_BYTES_PER_HEAD = {("c2", "bwd_main"): (219.57e6 + 102.19e6) / 4, ("c2", "fwd"): (103.67e6 + 16.50e6) / 4,
                       # C4 shape at 4 heads (profiles/dram_c4_h4.md)
                       ("c4", "bwd_main"): (1232.46e6 + 625.67e6) / 4, ("c4", "fwd"): (270.61e6 + 63.98e6) / 4}
NOMINAL_BF16_TFLOPS = 2250.0


STRONG_SCALING = {"c4", "c5"}  # total work fixed as N grows (heads split over the ranks)


def heads_layout(cfg_name: str, world: int, heads_override: int = 0):
    """(heads per rank, heads of the whole job, scaling) of a config at N ranks."""
    h_total = CONFIGS[cfg_name][4]
    if heads_override > 0:
        return heads_override, heads_override * world, "weak"
    if cfg_name in STRONG_SCALING:
        assert h_total % world == 0, f"{h_total} heads must split evenly over {world} ranks"
        return h_total // world, h_total, "strong"
    return h_total, h_total * world, "weak"


def config_dict(cfg_name: str, world: int, heads_override: int = 0) -> dict:
    """The line's ``config`` object; both arms (ours and --impl reference)
    print the same one for the same workload."""
    kind, b, sq, skv, _, _, desc = CONFIGS[cfg_name]
    h, global_h, _ = heads_layout(cfg_name, world, heads_override)
    return {
        "workload": desc, "global_batch": b, "seq_len": sq,
        "kv_len": [skv, DUAL_IMAGE_CONTEXT] if kind == "dual" else skv, "heads_per_gpu": h,
        "heads_total": global_h, "head_dim": 128, "parallelism": f"heads/{world}",
        "l2": "inputs larger than L2 (q/k/v/dO/o/grad working set >> 126 MB); no flush",
    }


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"bf16_tflops": d["bf16_tflops"], "bf16_tflops_sustained": d.get("bf16_tflops_sustained"),
                "hbm_gbs": d["hbm_gbs"], "source": "measured"}
    return {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0, "source": "fallback"}


def flops(b, h, sq, skv):
    f = 4.0 * b * h * sq * skv * 128
    return f, 2.5 * f


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-f", self.path], stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        try:
            for line in pathlib.Path(self.path).read_text().splitlines():
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
            os.unlink(self.path)
        except Exception:
            return None
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        loaded = [x for x in sm if x > 0.5 * max(sm)] if sm else []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# --------------------------------------------------------------------------- CPU arm
def _cpu_threads() -> int:
    try:
        from threadpoolctl import threadpool_info

        return int(max([i.get("num_threads", 1) for i in threadpool_info()] + [1]))
    except Exception:
        return 1


def _use_all_cores() -> int:
    """Give numpy's BLAS every host core (torchrun sets OMP_NUM_THREADS=1 for
    its ranks, which would otherwise leave the CPU arm on one thread) and
    return the thread count actually in use."""
    try:
        import numpy  # noqa: F401  (threadpoolctl only sees BLAS libraries already loaded)
        from threadpoolctl import threadpool_limits

        threadpool_limits(os.cpu_count() or 1)
    except Exception:
        pass
    return _cpu_threads()


class CpuSampler:
    """The oracle port (fp32 numpy, oracle/oracle.py) on a bounded sample of
    the workload: head 0, ``rows`` query rows against the full K/V, forward +
    analytic backward.  Cost is linear in query rows and heads, so TFLOP/s
    over the sample is the workload's rate on these cores."""

    def __init__(self, cfg_name: str):
        import numpy as np

        from oracle.oracle import round_bf16

        self.kind, self.b, self.sq, self.skv, self.h, seed, _ = CONFIGS[cfg_name]
        self.rng = np.random.default_rng(seed)
        lens = [self.skv] + ([DUAL_IMAGE_CONTEXT] if self.kind == "dual" else [])
        self.kv = [tuple(round_bf16(self.rng.standard_normal((1, 1, n, 128), dtype=np.float32)) for _ in range(2))
                   for n in lens]

    def run(self, rows: int) -> float:
        from oracle.oracle import oracle_bwd, oracle_fwd, round_bf16

        import numpy as np

        q = round_bf16(self.rng.standard_normal((1, 1, rows, 128), dtype=np.float32))
        do = round_bf16(self.rng.standard_normal((1, 1, rows, 128), dtype=np.float32))
        t0 = time.perf_counter()
        for k, v in self.kv:
            o, lse = oracle_fwd(q, k, v)
            oracle_bwd(q, k, v, o, lse, do)
        return time.perf_counter() - t0

    def rows_for(self, seconds: float) -> int:
        dt = self.run(256)
        rows = int(256 * seconds / max(dt, 1e-4))
        return max(256, min(self.sq, rows))

    def flops(self, rows: int) -> float:
        return sum(sum(flops(1, 1, rows, k.shape[2])) for k, _ in self.kv)


def cpu_sample(cfg_name: str, target_s: float = 12.0):
    s = CpuSampler(cfg_name)
    rows = s.rows_for(target_s)
    dt = s.run(rows)
    return {
        "value": s.flops(rows) / dt / 1e12,
        "unit": "TFLOP/s",
        "cores": _cpu_threads(),
        "kind": "port",
        "sample": (f"oracle/oracle.py fp32 fwd+bwd on head 0: {rows} of {s.sq} query rows x "
                   f"{' + '.join(str(k.shape[2]) for k, _ in s.kv)} keys ({dt:.1f} s); cost is linear in rows "
                   f"and heads"),
    }


# --------------------------------------------------------------------------- C5 (sequence parallel)
def c5_measure(args, rank, world, dev, group):
    """One step = the attention of a sequence-parallel Wan block, forward and
    backward, through wan_flash.ulysses.ulysses_attention_block: q/k/v/dO
    sequence-sharded per rank, a 512-token context replicated, exchanges
    overlapped with the attention work that does not need them.  Exposed
    communication = step time minus the time of the same local attention on
    head-sharded inputs.  Returns (a dict of timings and parity, the step's
    FLOPs for the whole job, the kernel launches per step); the process
    group, if any, is the caller's."""
    import torch
    import torch.distributed as dist

    from wan_flash import _lib
    from wan_flash.interface import bwd_plan, wan_flash_attn
    from wan_flash.ulysses import shard_heads, ulysses_attention_block

    kind, b, S, _, H, seed, desc = CONFIGS["c5"]
    L = C5_CONTEXT
    assert S % world == 0 and H % world == 0, "75600 tokens and 40 heads must split evenly over the ranks"
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed * 1000 + rank)

    def rnd(*shape, grad=False):
        t = torch.randn(*shape, device=dev, dtype=torch.float32, generator=gen).to(torch.bfloat16)
        return t.requires_grad_(grad)

    s_loc, hp = S // world, H // world
    q, k, v = (rnd(b, s_loc, H, 128, grad=True) for _ in range(3))
    do_self, do_cross = rnd(b, s_loc, H, 128), rnd(b, s_loc, H, 128)
    gctx = torch.Generator(device=dev)
    gctx.manual_seed(seed * 1000 + 999)  # the context is the same on every rank
    ck, cv = (torch.randn(b, L, H, 128, device=dev, generator=gctx).to(torch.bfloat16).requires_grad_(True)
              for _ in range(2))
    # local (head-sharded) inputs of the same attention work, for the no-exchange reference timing
    qh, kh, vh = (rnd(b, S, hp, 128, grad=True) for _ in range(3))
    doh_s, doh_c = rnd(b, S, hp, 128), rnd(b, S, hp, 128)
    ckh, cvh = (shard_heads(t.detach(), rank, world).contiguous().requires_grad_(True) for t in (ck, cv))
    out = {}

    def sp_step():
        for t in (q, k, v, ck, cv):
            t.grad = None
        if world > 1:
            o_s, o_c = ulysses_attention_block(q, k, v, ck, cv, group)
        else:
            o_s, o_c = wan_flash_attn(q, k, v), wan_flash_attn(q, ck, cv)
        torch.autograd.backward((o_s, o_c), (do_self, do_cross))
        out["o_s"], out["o_c"] = o_s.detach(), o_c.detach()

    def local_step():
        for t in (qh, kh, vh, ckh, cvh):
            t.grad = None
        o_s, o_c = wan_flash_attn(qh, kh, vh), wan_flash_attn(qh, ckh, cvh)
        torch.autograd.backward((o_s, o_c), (doh_s, doh_c))

    def barrier():
        if world > 1:
            dist.barrier(group=group)
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        return float(t.item())

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            fn()
        e1.record()
        barrier()
        return max_over_ranks(e0.elapsed_time(e1)) / args.steps

    ms = timed(sp_step)
    local_ms = timed(local_step)
    _lib.check_device()
    parity = c5_parity(q, k, v, ck, cv, do_self, do_cross, out["o_s"], out["o_c"], group, world)
    f_self, fb_self = flops(b, H, S, S)
    f_cross, fb_cross = flops(b, H, S, L)
    step_flops = f_self + fb_self + f_cross + fb_cross  # whole job (all ranks)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    launches = sum(1 + 3 + (2 if bwd_plan(b, S, skv, hp, sms)["nsplit"] > 1 else 0) for skv in (S, L))
    # one all-to-all per tensor: q, k, v in; o out (x2 outputs); dO in (x2); dq, dk, dv back
    a2a_bytes = b * s_loc * H * 128 * 2 * (world - 1) / world
    res = {
        "workload": desc, "ms_per_step": ms, "tflops": step_flops / (ms * 1e-3) / 1e12,
        "attention_only_ms": local_ms,
        "attention_only_tflops_per_gpu": step_flops / world / (local_ms * 1e-3) / 1e12,
        "exposed_comm_ms": max(0.0, ms - local_ms),
        "exposed_comm_frac": max(0.0, ms - local_ms) / ms,
        "all_to_all_bytes_per_tensor_per_rank": a2a_bytes,
        "parity": parity,
    }
    return res, step_flops, launches


def c5_parity(q, k, v, ck, cv, do_self, do_cross, o_s, o_c, group, world):
    """Check the sequence-parallel block's outputs and query gradient against
    attention computed without the all-to-all: K and V are gathered along the
    sequence (all_gather, not the all-to-all under test) and this rank's
    query rows attend them directly with all heads.  o_self and o_cross are
    per-row computations of the same kernels (expected bitwise equal); dq
    differs only by the fp32 reduction order.  Gate: rel_l2 <= 4.5e-3, the
    test suite's tolerance.  Worst over ranks."""
    import torch
    import torch.distributed as dist

    from wan_flash.interface import wan_flash_bwd, wan_flash_fwd

    def gather_seq(t):
        if world == 1:
            return t.detach()
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t.detach().contiguous(), group=group)
        return torch.cat(parts, dim=1)

    def rel(x, y):
        return ((x.float() - y.float()).norm() / y.float().norm().clamp_min(1e-30)).item()

    with torch.no_grad():
        qd = q.detach()
        kf, vf = gather_seq(k), gather_seq(v)
        o_ref, lse_ref = wan_flash_fwd(qd, kf, vf)
        oc_ref, lsec_ref = wan_flash_fwd(qd, ck.detach(), cv.detach())
        dq_s, _, _ = wan_flash_bwd(qd, kf, vf, o_ref, lse_ref, do_self)
        dq_c, _, _ = wan_flash_bwd(qd, ck.detach(), cv.detach(), oc_ref, lsec_ref, do_cross)
        dq_ref = (dq_s.float() + dq_c.float()).to(torch.bfloat16)
        errs = [rel(o_s, o_ref), rel(o_c, oc_ref), rel(q.grad, dq_ref),
                float((o_s.float() - o_ref.float()).abs().max())]
        del kf, vf
    t = torch.tensor(errs, device=q.device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    e = t.tolist()
    return {"o_self_rel_l2": e[0], "o_cross_rel_l2": e[1], "dq_rel_l2": e[2], "o_self_max_abs": e[3],
            "tolerance_rel_l2": 4.5e-3, "ok": all(x <= 4.5e-3 for x in e[:3]),
            "against": "attention of this rank's rows over K/V gathered along the sequence, no all-to-all"}


def run_c5(args, rank, world, local_rank):
    """--config c5: the sequence-parallel block as the line's workload."""
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    group = dist.group.WORLD if world > 1 else None
    clocks = ClockSampler(local_rank)
    clocks.start()
    res, step_flops, launches = c5_measure(args, rank, world, dev, group)
    clk = clocks.stop()
    if rank == 0:
        kind, b, S, _, H, seed, desc = CONFIGS["c5"]
        peaks = load_peaks()
        local_tf = res["attention_only_tflops_per_gpu"]
        line = {
            "metric": METRIC, "value": res["tflops"], "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": res["ms_per_step"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) bf16; no dataset)",
            "config": {"workload": desc, "global_batch": b, "seq_len": S, "kv_len": S, "context_len": C5_CONTEXT,
                       "heads_total": H, "heads_per_gpu": H // world, "head_dim": 128,
                       "parallelism": f"ulysses sp{world}",
                       "l2": "inputs larger than L2 (activations >> 126 MB); no flush"},
            **{k: res[k] for k in ("attention_only_ms", "attention_only_tflops_per_gpu", "exposed_comm_ms",
                                   "exposed_comm_frac", "all_to_all_bytes_per_tensor_per_rank", "parity")},
            "roofline": {"kernel": "attention (fwd+bwd, local)", "bound": "tensor", "achieved": local_tf,
                         "peak": peaks["bf16_tflops"], "unit": "TFLOP/s", "frac": local_tf / peaks["bf16_tflops"],
                         "traffic": None},
            "cpu_baseline": None, "e2e": None, "clocks": clk,
            "gpu_launches": launches * args.steps,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


# --------------------------------------------------------------------------- features A/B
def run_features_ab(args):
    """Re-evaluate the features.py flags on B200: each setting against the
    defaults on the config's shape (1 GPU), forward or backward chain timed
    with CUDA events on the stream, settings interleaved round-robin over
    `--steps` rounds (median reported) so clock drift hits all alike."""
    import torch

    from wan_flash import features, interface

    kind, b, sq, skv, h, seed, desc = CONFIGS[args.config]
    assert kind in ("self", "cross"), "--features-ab runs on c2, c3 or c3i2v"
    if args.heads > 0:
        h = args.heads
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed * 1000)

    def rnd(s):
        return torch.randn(b, s, h, 128, device=dev, dtype=torch.float32, generator=gen).to(torch.bfloat16)

    q, k, v, do = rnd(sq), rnd(skv), rnd(skv), rnd(sq)
    f_fwd, f_bwd = flops(b, h, sq, skv)
    o, lse = interface.wan_flash_fwd(q, k, v)
    settings = [
        ("fwd", "defaults", {}, {}),
        ("fwd", "rescale_skip_threshold=0", {"rescale_skip_threshold": 0.0}, {}),
        ("fwd", "scheduler=single", {"scheduler": "single"}, {}),
        ("fwd", "scheduler=persistent", {"scheduler": "persistent"}, {}),
        ("fwd", "cluster_mn=(1,1)", {"cluster_mn": (1, 1)}, {}),
        ("bwd", "defaults", {}, {}),
        ("bwd", "cluster_n=2", {}, {"cluster_n": 2}),
        ("bwd", "deterministic", {}, {"deterministic": True}),
        ("bwd", "pdl=False", {}, {"pdl": False}),
    ]
    auto_nsplit = interface.bwd_plan(b, sq, skv, h)["nsplit"]
    for n in sorted({1, 2, max(1, auto_nsplit // 2), auto_nsplit * 2} - {auto_nsplit}):
        settings.append(("bwd", f"nsplit={n}", {}, {"nsplit": n}))
    times = {i: [] for i in range(len(settings))}
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    fwd_idx = [i for i, st in enumerate(settings) if st[0] == "fwd"]
    bwd_idx = [i for i, st in enumerate(settings) if st[0] == "bwd"]
    for rnd_i in range(args.warmup + args.steps):
        # each round runs the forward settings, one untimed backward (so the
        # first timed backward does not inherit the forward runs' power and
        # clock state), then the backward settings; both blocks are rotated by
        # the round index so no setting always runs first
        rf, rb = rnd_i % len(fwd_idx), rnd_i % len(bwd_idx)
        order = fwd_idx[rf:] + fwd_idx[:rf] + [None] + bwd_idx[rb:] + bwd_idx[:rb]
        for i in order:
            if i is None:
                features.reset()
                interface.wan_flash_bwd(q, k, v, o, lse, do)
                continue
            what, _, fo, bo = settings[i]
            features.reset()
            features.set_overrides(**fo)
            features.set_bwd_overrides(**bo)
            ev0.record()
            if what == "fwd":
                interface.wan_flash_fwd(q, k, v)
            else:
                interface.wan_flash_bwd(q, k, v, o, lse, do)
            ev1.record()
            torch.cuda.synchronize()
            if rnd_i >= args.warmup:
                times[i].append(ev0.elapsed_time(ev1))
    features.reset()
    base = {}
    for i, (what, name, fo, bo) in enumerate(settings):
        ms = statistics.median(times[i])
        tf = (f_fwd if what == "fwd" else f_bwd) / (ms * 1e-3) / 1e12
        if name == "defaults":
            base[what] = tf
        line = {"features_ab": what, "setting": name, "ms": ms, "tflops": tf,
                "vs_defaults": tf / base[what] if what in base else None,
                "config": {"workload": desc, "heads": h}, "rounds": args.steps}
        print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- output check
def timed_output_check(q, k, v, do, o, dq, dk, dv, lse, rows: int = 1024) -> dict:
    """Compare the last timed step's outputs with plain fp32 attention
    (torch matmuls, TF32 off) on slices of head 0 of batch 0: O, LSE and dQ
    of query rows [0, rows), dK and dV of key rows [0, rows).  The backward
    reference recomputes P from the kernel's own lse and uses its o, as the
    reference's tests do.  Returns rel_l2 errors and the LSE max abs error."""
    import torch

    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        with torch.no_grad():
            scale = 1.0 / math.sqrt(q.shape[-1])
            qh, kh, vh, doh, oh = (t[0, :, 0].float() for t in (q, k, v, do, o))
            lh = lse[0, 0].float()
            rq, rk = min(rows, qh.shape[0]), min(rows, kh.shape[0])

            def rel(x, y):
                return float((x.float() - y).norm() / y.norm().clamp_min(1e-30))

            s_r = (qh[:rq] @ kh.T) * scale
            lse_ref = torch.logsumexp(s_r, dim=-1)
            o_ref = torch.softmax(s_r, dim=-1) @ vh
            p_r = torch.exp(s_r - lh[:rq, None])
            d_r = (doh[:rq] * oh[:rq]).sum(-1)
            dq_ref = (p_r * ((doh[:rq] @ vh.T) - d_r[:, None])) @ kh * scale
            del s_r, p_r
            s_c = (qh @ kh[:rk].T) * scale
            p_c = torch.exp(s_c - lh[:, None])
            dv_ref = p_c.T @ doh
            d_all = (doh * oh).sum(-1)
            dk_ref = (p_c * ((doh @ vh[:rk].T) - d_all[:, None])).T @ qh * scale
            return {"o_rel_l2": rel(o[0, :rq, 0], o_ref), "lse_max_abs": float((lh[:rq] - lse_ref).abs().max()),
                    "dq_rel_l2": rel(dq[0, :rq, 0], dq_ref), "dk_rel_l2": rel(dk[0, :rk, 0], dk_ref),
                    "dv_rel_l2": rel(dv[0, :rk, 0], dv_ref)}
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


# --------------------------------------------------------------------------- GPU arm
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="c4", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=0.0,
                    help="--impl reference: seconds of CPU work per step (0 = sized so the run ends in minutes)")
    ap.add_argument("--no-sp", action="store_true", help="at N > 1, skip the sequence-parallel block (C5) run")
    ap.add_argument("--heads", type=int, default=0, help="override heads per GPU (small profiling cases)")
    ap.add_argument("--features-ab", action="store_true",
                    help="A/B the features.py flags on --config (c2 or c3): one JSON line per setting")
    ap.add_argument("--bwd-cluster-n", type=int, default=0, choices=[0, 1, 2],
                    help="backward kernel form: 1 = single CTAs, 2 = CTA pairs, 0 = the feature default")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    kind, b, sq, skv, h_total, seed, desc = CONFIGS[args.config]

    if args.impl == "reference":
        # rank 0 alone runs the CPU reference arm; other ranks exit without work
        if rank == 0:
            world = world if world > 1 else max(1, args.gpus)  # the arm it stands beside
            cores = _use_all_cores()
            sampler = CpuSampler(args.config)
            per_step_s = args.cpu_seconds or min(20.0, max(1.0, 150.0 / (args.steps + args.warmup)))
            rows = sampler.rows_for(per_step_s)
            for _ in range(args.warmup):
                sampler.run(rows)
            t = sum(sampler.run(rows) for _ in range(args.steps))
            value = sampler.flops(rows) * args.steps / t / 1e12
            cpu = {"value": value, "unit": "TFLOP/s", "cores": cores, "kind": "port",
                   "sample": (f"per step: oracle/oracle.py fp32 fwd+bwd on head 0, {rows} of {sq} query rows x "
                              f"{' + '.join(str(kk.shape[2]) for kk, _ in sampler.kv)} keys; cost is linear in rows "
                              f"and heads")}
            line = {
                "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": 1e3 * t / args.steps, "higher_is_better": True,
                "scaling": heads_layout(args.config, world, args.heads)[2],
                "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1), bf16-rounded)",
                "config": config_dict(args.config, world, args.heads),
                "cpu_baseline": cpu,
                "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            }
            print(json.dumps(line), flush=True)
        return

    import torch
    import torch.distributed as dist

    from wan_flash import _lib, features, interface

    if args.config == "c5":
        return run_c5(args, rank, world, local_rank)
    if args.features_ab:
        return run_features_ab(args)

    if args.bwd_cluster_n:
        features.set_bwd_overrides(cluster_n=args.bwd_cluster_n)

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    h, global_h, scaling = heads_layout(args.config, world, args.heads)

    gen = torch.Generator(device=dev)
    gen.manual_seed(seed * 1000 + rank)

    def rnd(s):
        return torch.randn(b, s, h, 128, device=dev, dtype=torch.float32, generator=gen).to(torch.bfloat16)

    q, k, v, do = rnd(sq), rnd(skv), rnd(skv), rnd(sq)
    f_fwd, f_bwd = flops(b, h, sq, skv)
    dual = kind == "dual"
    if dual:
        # the image context: same Q, separate softmax; FLOPs of both contexts
        k1, v1 = rnd(DUAL_IMAGE_CONTEXT), rnd(DUAL_IMAGE_CONTEXT)
        f1, fb1 = flops(b, h, sq, DUAL_IMAGE_CONTEXT)
        f_fwd, f_bwd = f_fwd + f1, f_bwd + fb1
    step_flops = f_fwd + f_bwd

    def step(marks=None):
        if dual:
            interface._mark(marks, "fwd")
            o0, lse0, o1, lse1 = interface.wan_flash_fwd_dual(q, k, v, k1, v1)
            dq, grads = interface._bwd_multi(q, ((k, v, o0, lse0), (k1, v1, o1, lse1)), do, marks)
            return o0, dq, grads
        o, lse = interface._fwd_impl(q, k, v, marks)
        dq, dk, dv = interface._bwd_impl(q, k, v, o, lse, do, marks)
        return o, dq, dk, dv, lse

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        step()
    _lib.check_device()
    barrier()

    clocks = ClockSampler(local_rank)
    clocks.start()
    # ---- timed region: K steps, inputs resident in HBM (working set >> L2)
    all_marks = []
    barrier()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record()
    last = None
    for _ in range(args.steps):
        marks = []
        last = step(marks)
        all_marks.append(marks)
    t_end.record()
    barrier()
    ms = t_start.elapsed_time(t_end)
    ms = max_over_ranks(ms)
    ms_per_step = ms / args.steps
    # the last timed step's outputs against fp32 attention on slices of head 0
    # (outside the timed region; every rank checks its own heads' slice)
    timed_check = None
    if not dual:
        errs = timed_output_check(q, k, v, do, *last)
        t_err = torch.tensor(list(errs.values()), device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t_err, op=dist.ReduceOp.MAX)
        timed_check = dict(zip(errs.keys(), t_err.tolist()))
        timed_check.update({"tolerance_rel_l2": 4.5e-3, "tolerance_lse_abs": 1e-5,
                            "ok": all(timed_check[n] <= 4.5e-3 for n in ("o_rel_l2", "dq_rel_l2", "dk_rel_l2",
                                                                          "dv_rel_l2"))
                            and timed_check["lse_max_abs"] <= 1e-5,
                            "against": "fp32 torch attention of head 0: query rows [0, 1024) for o/lse/dq, "
                                       "key rows [0, 1024) for dk/dv (o and lse of the kernel given to the "
                                       "backward, as the reference's tests do)"})

    # per-kernel averages from the marks of the timed region
    per = {}
    for marks in all_marks:
        for (name, ev), (_, ev_next) in zip(marks[:-1], marks[1:]):
            if name == "end":
                continue
            per.setdefault(name, []).append(ev.elapsed_time(ev_next))
    kern_ms = {n: sum(x) / len(x) for n, x in per.items()}

    # ---- e2e: public API, host (pinned) inputs copied in and results copied out
    # every step.  Host->device copies and device->host reads run on their own
    # streams (both PCIe directions at once) into two alternating device buffer
    # sets, so step i's inputs and step i-1's results move while step i's
    # kernels run, as in a training input pipeline.
    e2e = None
    if not args.no_e2e:
        from wan_flash.interface import wan_flash_bwd, wan_flash_bwd_dual, wan_flash_fwd, wan_flash_fwd_dual

        ins = (q, k, v, do) + ((k1, v1) if dual else ())
        hins = [t.cpu().pin_memory() for t in ins]
        outs_like = (q, q, k, v) + ((k1, v1) if dual else ())
        n_out = len(outs_like)
        host_out = [[torch.empty(t.shape, dtype=torch.bfloat16, pin_memory=True) for t in outs_like]
                    for _ in range(2)]
        dev_in = [[torch.empty_like(t) for t in ins] for _ in range(2)]
        dev_out = [[None] * n_out for _ in range(2)]
        copy_stream = torch.cuda.Stream(device=dev)  # host -> device
        read_stream = torch.cuda.Stream(device=dev)  # device -> host (the other PCIe direction)
        compute_stream = torch.cuda.current_stream(dev)
        in_ready = [torch.cuda.Event() for _ in range(2)]
        out_ready = [torch.cuda.Event() for _ in range(2)]
        out_read = [torch.cuda.Event() for _ in range(2)]
        for ev in out_read:
            ev.record(read_stream)

        def e2e_step(i):
            sl = i % 2
            with torch.cuda.stream(copy_stream):
                copy_stream.wait_event(out_ready[sl])  # kernels of step i-2 are done with this set
                for dst, src in zip(dev_in[sl], hins):
                    dst.copy_(src, non_blocking=True)
                in_ready[sl].record(copy_stream)
            compute_stream.wait_event(in_ready[sl])
            compute_stream.wait_event(out_read[sl])  # step i-2's results have been read back
            if dual:
                qd, kd, vd, dod, k1d, v1d = dev_in[sl]
                o0_, lse0_, o1_, lse1_ = wan_flash_fwd_dual(qd, kd, vd, k1d, v1d)
                dq_, dk_, dv_, dk1_, dv1_ = wan_flash_bwd_dual(qd, kd, vd, k1d, v1d, o0_, lse0_, o1_, lse1_, dod)
                dev_out[sl] = [o0_ + o1_, dq_, dk_, dv_, dk1_, dv1_]
            else:
                qd, kd, vd, dod = dev_in[sl]
                o_, lse_ = wan_flash_fwd(qd, kd, vd)
                dq_, dk_, dv_ = wan_flash_bwd(qd, kd, vd, o_, lse_, dod)
                dev_out[sl] = [o_, dq_, dk_, dv_]
            out_ready[sl].record(compute_stream)
            with torch.cuda.stream(read_stream):
                read_stream.wait_event(out_ready[sl])
                for dst, src in zip(host_out[sl], dev_out[sl]):
                    dst.copy_(src, non_blocking=True)
                out_read[sl].record(read_stream)

        for i in range(2):
            e2e_step(i)
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(compute_stream)
        for i in range(args.steps):
            e2e_step(i)
        compute_stream.wait_stream(read_stream)  # the last read-back is inside the timed region
        e1.record(compute_stream)
        barrier()
        e_ms = max_over_ranks(e0.elapsed_time(e1)) / args.steps
        h2d = sum(t.numel() * t.element_size() for t in hins)
        d2h = sum(t.numel() * t.element_size() for t in host_out[0])
        e2e = {"value": step_flops * world / (e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
               "ms_per_step": e_ms, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "pipeline": "H2D and D2H on two copy streams, double-buffered, overlapping neighbouring steps"}
    clk = clocks.stop()
    _lib.check_device()

    # At N > 1 the default (C4, head-sharded) run also measures the
    # sequence-parallel block (C5: Ulysses all-to-alls around the same
    # attention) so the collective path is timed and checked in every scaling
    # run; every rank takes part.
    sp_block = None
    if world > 1 and args.config == "c4" and args.heads == 0 and not args.no_sp:
        sp_res, sp_flops, sp_launches = c5_measure(args, rank, world, dev, dist.group.WORLD)
        sp_block = {**sp_res, "n_gpus": world, "gpu_launches": sp_launches * args.steps,
                    "note": "separate timed region after the C4 steps; not part of value or ms_per_step"}

    if rank == 0:
        peaks = load_peaks()
        value = step_flops * world / (ms_per_step * 1e-3) / 1e12
        fwd_tf = f_fwd / (kern_ms["fwd"] * 1e-3) / 1e12
        bwd_chain_ms = sum(kern_ms.get(n, 0.0) for n in ("bwd_pre", "bwd_main", "bwd_convert"))
        bwd_tf = f_bwd / (bwd_chain_ms * 1e-3) / 1e12
        main_tf = f_bwd / (kern_ms["bwd_main"] * 1e-3) / 1e12
        dominant = "bwd_main" if kern_ms["bwd_main"] >= kern_ms["fwd"] else "fwd"
        dom_flops = f_bwd if dominant == "bwd_main" else f_fwd
        dom_ms = kern_ms[dominant]
        achieved = dom_flops / (dom_ms * 1e-3) / 1e12
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        plan = interface.bwd_plan(b, sq, skv, h, sms)
        launches_per_step = 1 + 3 + (2 if plan["nsplit"] > 1 else 0)
        if dual:  # one forward; a second preprocess and main; its own split-M converts
            plan1 = interface.bwd_plan(b, sq, DUAL_IMAGE_CONTEXT, h, sms)
            launches_per_step += 2 + (2 if plan1["nsplit"] > 1 else 0)
        # HBM-side figures: algorithmic bytes per step over the measured time
        # of the memory-bound kernels, and of the forward (for the short-KV
        # cross attention, whose intensity sits near the HBM ridge)
        sq_r = -(-sq // 128) * 128
        ctx_lens = [skv] + ([DUAL_IMAGE_CONTEXT] if dual else [])
        act = 2 * b * h * 128  # bytes per row of a bf16 (b, s, h, 128) tensor
        pre_bytes = sum(2 * sq * act + 4 * b * h * sq + 8 * b * h * sq_r for _ in ctx_lens) + 4 * b * h * sq_r * 128
        conv_bytes = 4 * b * h * sq_r * 128 + sq * act
        for n, pl in zip(ctx_lens, [plan] + ([plan1] if dual else [])):
            if pl["nsplit"] > 1:  # dk and dv accumulators
                conv_bytes += 2 * (4 * b * h * (-(-n // 128) * 128) * 128 + n * act)
        fwd_bytes = sq * act * (1 + len(ctx_lens)) + sum(2 * n * act for n in ctx_lens) + 4 * b * h * sq * len(ctx_lens)

        def gbs(nbytes, name):
            t = kern_ms.get(name)
            if not t:
                return None
            v = nbytes / (t * 1e-3) / 1e9
            return {"bytes_per_step": nbytes, "gbs": v, "frac_of_hbm": v / peaks["hbm_gbs"]}

        hbm = {"bwd_pre": gbs(pre_bytes, "bwd_pre"), "bwd_convert": gbs(conv_bytes, "bwd_convert"),
               "fwd": gbs(fwd_bytes, "fwd"), "hbm_peak_gbs": peaks["hbm_gbs"],
               "note": "algorithmic bytes (each tensor read or written once) over CUDA-event time"}
        cpu = None
        if not args.no_cpu and world == 1:
            cpu = cpu_sample(args.config)
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_per_step,
            "higher_is_better": True,
            "scaling": scaling,
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) bf16; no dataset)",
            "config": config_dict(args.config, world, args.heads),
            "fwd_tflops": fwd_tf,
            "bwd_tflops": bwd_tf,
            "bwd_main_tflops": main_tf,
            "fwd_frac_of_measured_peak": fwd_tf / peaks["bf16_tflops"],
            "bwd_frac_of_measured_peak": bwd_tf / peaks["bf16_tflops"],
            # the step runs for seconds at the 1 kW power cap, as the driver's
            # sustained cuBLAS loop does: the fractions of that figure too
            "frac_of_measured_sustained": ({"fwd": fwd_tf / peaks["bf16_tflops_sustained"],
                                            "bwd": bwd_tf / peaks["bf16_tflops_sustained"],
                                            "peak_sustained": peaks["bf16_tflops_sustained"]}
                                           if peaks.get("bf16_tflops_sustained") else None),
            "frac_of_nominal_2250": {"fwd": fwd_tf / NOMINAL_BF16_TFLOPS, "bwd": bwd_tf / NOMINAL_BF16_TFLOPS},
            "kernel_ms": kern_ms,
            "roofline": {
                "kernel": dominant, "bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"],
                "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"],
                "traffic": (DRAM_BYTES_PER_HEAD[(args.config, dominant)] * h
                            if (args.config, dominant) in DRAM_BYTES_PER_HEAD else None),
                "frac_of_sustained": (achieved / peaks["bf16_tflops_sustained"]
                                      if peaks.get("bf16_tflops_sustained") else None),
                "traffic_unit": "bytes per launch (ncu capture at 4 heads, scaled by heads)",
                "peak_source": f"{peaks['source']} burst bf16 (MEASURED_PEAKS.json)" if peaks["source"] == "measured"
                else "fallback 1.59 PFLOP/s",
            },
            "hbm": hbm,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "clocks": clk,
            "gpu_launches": launches_per_step * args.steps,
            "sp_block": sp_block,
            "timed_outputs_check": timed_check,
            "bwd_nsplit": plan["nsplit"],
            "bwd_cluster_n": plan["cluster_n"],
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
