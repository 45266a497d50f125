"""Host driver: torch tensors -> the sm_100a C ABI (libwanflash.so).

Same API and contract as the reference driver (``wan_flash/interface.py`` of
Quarky93/wan-flash):

wan_flash_fwd(q, k, v) -> (o, lse)                      (interface.py:33-75)
  q: (b, s_q, h, d) bf16, k/v: (b, s_kv, h, d) bf16
  o: (b, s_q, h, d) bf16, lse: (b, h, s_q) fp32, NATURAL log.

wan_flash_bwd(q, k, v, o, lse, do) -> (dq, dk, dv)      (interface.py:98-196)
  lse: natural log, (b, h, s_q) fp32.  dq is accumulated with fp32
  reductions, so it is nondeterministic (as in the reference).

wan_flash_attn(q, k, v) -> o                            (interface.py:199-215)
  autograd.Function chaining the two.

Contract violations raise AssertionError (the reference uses ``assert``);
non-contiguous inputs are made contiguous.  Outputs and workspaces are torch
allocations made here; the kernels run on ``torch.cuda.current_stream()``
and nothing synchronises.  There is no CPU path: the CUDA library must be
built (``python -m wan_flash.build``) and the tensors must live on an
sm_100 GPU.
"""

from __future__ import annotations

import ctypes
import math

import torch

from wan_flash import _lib, features
from wan_flash.shapes import BWD_TILE_M, TILE_N, sm_count

_SM_CACHE: dict = {}


def _sms(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _SM_CACHE:
        _SM_CACHE[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return _SM_CACHE[idx]


def _aligned(t: torch.Tensor) -> torch.Tensor:
    t = t if t.is_contiguous() else t.contiguous()
    if t.data_ptr() % 16 != 0:  # a contiguous view with an odd storage offset
        t = t.clone()
    return t


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: torch.Tensor):
    return ctypes.c_void_p(t.data_ptr())


def _mark(marks, name):
    """Record a CUDA event on the current stream (bench timing only)."""
    if marks is not None:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        marks.append((name, ev))


def _fwd_cfg(f) -> "_lib.FwdCfg":
    """wf_fwd_cfg from the forward feature flags.  cluster_mn (2, 1) maps to
    cluster_m = 0 (auto: CTA pairs where the kernel supports them, single
    CTAs elsewhere), (1, 1) to single CTAs."""
    return _lib.FwdCfg(float(f.rescale_skip_threshold), {"auto": 0, "single": 1, "persistent": 2}[f.scheduler],
                       int(f.num_sms), 0 if tuple(f.cluster_mn) == (2, 1) else 1)


def wan_flash_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
    return _fwd_impl(q, k, v)


def _fwd_impl(q, k, v, marks=None):
    assert q.dtype == torch.bfloat16 and k.dtype == torch.bfloat16 and v.dtype == torch.bfloat16
    assert q.dim() == 4 and k.dim() == 4 and v.dim() == 4
    b, sq, h, d = q.shape
    bk, skv, hk, dk = k.shape
    assert (b, h, d) == (bk, hk, dk) and v.shape == k.shape
    assert d == 128, "specialized for head_dim=128"
    assert q.is_cuda and k.device == q.device and v.device == q.device, "tensors must be on one CUDA device"
    assert skv > 0 or sq == 0 or b == 0 or h == 0, "attention over an empty key set"
    q, k, v = (_aligned(t) for t in (q, k, v))

    o = torch.empty_like(q)
    lse = torch.empty(b, h, sq, device=q.device, dtype=torch.float32)
    if o.numel() == 0:
        return o, lse

    f = features.get()
    cfg = _fwd_cfg(f)
    with torch.cuda.device(q.device):
        _mark(marks, "fwd")
        rc = _lib.lib().wf_fwd(_ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(lse), b, sq, skv, h,
                               ctypes.byref(cfg), ctypes.c_void_p(_stream_ptr(q.device)))
        _mark(marks, "end")
    _lib.check(rc)
    return o, lse


def _auto_nsplit(base_ctas: int, m_blocks: int, sm_count: int = 148) -> int:
    """Split-M factor for the backward main kernel (reference: interface.py:78-95).

    1 when the (n_blocks*h*b) grid fills the GPU well; otherwise the smallest
    split with >= 95% wave efficiency (filling partial waves).  The SM count
    is the device's (148 on B200), not the reference's hard-coded 132.
    """

    def eff(ctas):
        return ctas / (sm_count * -(-ctas // sm_count))

    if eff(base_ctas) >= 0.85:
        return 1
    best_k, best_eff = 1, 0.0
    for cand in range(1, min(m_blocks, 64) + 1):
        e = eff(base_ctas * cand)
        if base_ctas * cand >= sm_count and e >= 0.95:
            return cand
        if e > best_eff:
            best_k, best_eff = cand, e
    return best_k


def bwd_plan(b: int, sq: int, skv: int, h: int, sms: int | None = None) -> dict:
    """Tile / split arithmetic of one backward call (host logic, no device)."""
    f = features.get_bwd()
    sq_rounded = -(-sq // BWD_TILE_M) * BWD_TILE_M
    m_blocks = sq_rounded // BWD_TILE_M
    n_blocks = -(-skv // TILE_N)
    skv_rounded = n_blocks * TILE_N
    sms = sms if sms is not None else sm_count()
    nsplit = f.nsplit if f.nsplit > 0 else _auto_nsplit(n_blocks * h * b, m_blocks, sms)
    nsplit = max(1, min(nsplit, m_blocks))
    return {
        "sq_rounded": sq_rounded, "m_blocks": m_blocks, "n_blocks": n_blocks,
        "skv_rounded": skv_rounded, "nsplit": nsplit, "cluster_n": f.cluster_n,
        "deterministic": bool(f.deterministic), "pdl": bool(f.pdl),
        # deterministic mode: ordered-accumulation counters, (b*h) x (m_blocks + n_blocks) int32
        "sem_len": b * h * (m_blocks + n_blocks) if f.deterministic else 0,
    }


def wan_flash_bwd(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    o: torch.Tensor,
    lse: torch.Tensor,
    do: torch.Tensor,
):
    """(b,s,h,d) bf16 q/k/v/o/do; lse (b,h,s_q) fp32 natural log ->
    (dq, dk, dv) bf16 (b,s,h,d)."""
    return _bwd_impl(q, k, v, o, lse, do)


def _bwd_impl(q, k, v, o, lse, do, marks=None):
    dq, ((dk, dv),) = _bwd_multi(q, ((k, v, o, lse),), do, marks)
    return dq, dk, dv


def _bwd_multi(q, contexts, do, marks=None):
    """Backward of attention(q, k_c, v_c) for one or two KV contexts given
    o_c, lse_c of each and dO (one tensor: the gradient of the sum of the
    outputs, or one per context): the contexts' main kernels add into one
    dQ accumulator (zeroed by the first preprocess), converted once.
    Returns (dq, ((dk_c, dv_c), ...))."""
    dos = list(do) if isinstance(do, (list, tuple)) else [do] * len(contexts)
    assert len(dos) == len(contexts)
    assert q.dtype == torch.bfloat16 and all(x.dtype == torch.bfloat16 and x.shape == q.shape for x in dos)
    b, sq, h, d = q.shape
    assert d == 128, "specialized for head_dim=128"
    for k, v, o, lse in contexts:
        assert all(t.dtype == torch.bfloat16 for t in (k, v, o))
        assert lse.dtype == torch.float32
        bk, skv, hk, dk_ = k.shape
        assert (b, h, d) == (bk, hk, dk_) and v.shape == k.shape
        assert o.shape == q.shape
        assert lse.shape == (b, h, sq)
        assert all(t.is_cuda and t.device == q.device for t in (k, v, o, lse, *dos)), \
            "tensors must be on one CUDA device"
    q = _aligned(q)
    dos = [_aligned(x) for x in dos]
    # the kernels write dq/dk/dv as contiguous (b, s, h, 128): allocate them
    # contiguous whatever the strides of the (possibly permuted) inputs
    dq = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    grads = [(torch.empty(k.shape, dtype=k.dtype, device=k.device),
              torch.empty(v.shape, dtype=v.dtype, device=v.device)) for k, v, _, _ in contexts]
    live = [c for c, (k, _, _, _) in enumerate(contexts) if b > 0 and h > 0 and k.shape[1] > 0]
    if sq == 0:
        for dk, dv in grads:
            dk.zero_(), dv.zero_()
        return dq, tuple(grads)
    if not live:
        return dq.zero_(), tuple(grads)

    dev = q.device
    sq_rounded = -(-sq // BWD_TILE_M) * BWD_TILE_M
    dq_accum = torch.empty(b, h, sq_rounded * d, device=dev, dtype=torch.float32)
    L = _lib.lib()
    stream = ctypes.c_void_p(_stream_ptr(dev))
    # per context: plan, workspaces, preprocess (the first one zeroes dq_accum)
    runs = []
    with torch.cuda.device(dev):
        _mark(marks, "bwd_pre")
        for i, c in enumerate(live):
            k, v, o, lse = contexts[c]
            k, v, o = (_aligned(t) for t in (k, v, o))
            do = dos[c]
            lse = lse if lse.is_contiguous() else lse.contiguous()
            skv = k.shape[1]
            plan = bwd_plan(b, sq, skv, h, _sms(dev))
            dpsum = torch.empty(b, h, sq_rounded, device=dev, dtype=torch.float32)
            neg_lse_log2 = torch.empty(b, h, sq_rounded, device=dev, dtype=torch.float32)
            dk, dv = grads[c]
            if plan["nsplit"] > 1:
                # split-M: dK/dV accumulate in fp32 (must start zeroed)
                dk_accum = torch.zeros(b, h, plan["skv_rounded"] * d, device=dev, dtype=torch.float32)
                dv_accum = torch.zeros_like(dk_accum)
            else:
                dk_accum = dv_accum = None
            cfg = _lib.BwdCfg(plan["nsplit"], plan["cluster_n"])
            cfg.pdl_off = 0 if plan["pdl"] else 1
            sem = None
            if plan["deterministic"]:
                sem = torch.zeros(plan["sem_len"], device=dev, dtype=torch.int32)
                cfg.deterministic, cfg.sem = 1, sem.data_ptr()
            _lib.check(L.wf_bwd_pre(_ptr(o), _ptr(do), _ptr(lse), _ptr(dpsum), _ptr(neg_lse_log2),
                                    _ptr(dq_accum) if i == 0 else None, b, sq, sq_rounded, h, stream))
            runs.append((k, v, skv, dpsum, neg_lse_log2, dk, dv, dk_accum, dv_accum, cfg, sem, do))
        _mark(marks, "bwd_main")
        for k, v, skv, dpsum, neg_lse_log2, dk, dv, dk_accum, dv_accum, cfg, _sem, do in runs:
            main_dk = dk_accum if dk_accum is not None else dk
            main_dv = dv_accum if dv_accum is not None else dv
            _lib.check(L.wf_bwd_main(_ptr(q), _ptr(k), _ptr(v), _ptr(do), _ptr(neg_lse_log2), _ptr(dpsum),
                                     _ptr(dq_accum), _ptr(main_dk), _ptr(main_dv), b, sq, skv, h,
                                     ctypes.byref(cfg), stream))
        _mark(marks, "bwd_convert")
        _lib.check(L.wf_bwd_convert(_ptr(dq_accum), _ptr(dq), ctypes.c_float(1.0 / math.sqrt(d)), b, sq, h, stream))
        for k, v, skv, dpsum, neg_lse_log2, dk, dv, dk_accum, dv_accum, cfg, _sem, _do in runs:
            if dk_accum is not None:
                _lib.check(L.wf_bwd_convert(_ptr(dk_accum), _ptr(dk), ctypes.c_float(1.0), b, skv, h, stream))
                _lib.check(L.wf_bwd_convert(_ptr(dv_accum), _ptr(dv), ctypes.c_float(1.0), b, skv, h, stream))
        _mark(marks, "end")
    return dq, tuple(grads)


def wan_flash_fwd_dual(q: torch.Tensor, k0: torch.Tensor, v0: torch.Tensor, k1: torch.Tensor, v1: torch.Tensor):
    """Two KV contexts attended by the same query rows in one launch (the Wan
    I2V cross attention: a text context and an image context, whose outputs
    the model adds).  Returns (o0, lse0, o1, lse1), each exactly what
    wan_flash_fwd(q, k_c, v_c) returns; every 256-row query block is loaded
    once for both contexts.  No reference counterpart."""
    assert q.dtype == torch.bfloat16 and q.dim() == 4
    b, sq, h, d = q.shape
    assert d == 128, "specialized for head_dim=128"
    for k, v in ((k0, v0), (k1, v1)):
        assert k.dtype == torch.bfloat16 and v.dtype == torch.bfloat16 and k.dim() == 4
        assert (k.shape[0], k.shape[2], k.shape[3]) == (b, h, d) and v.shape == k.shape
        assert q.is_cuda and k.device == q.device and v.device == q.device, "tensors must be on one CUDA device"
        assert k.shape[1] > 0 or sq == 0 or b == 0 or h == 0, "attention over an empty key set"
    q, k0, v0, k1, v1 = (_aligned(t) for t in (q, k0, v0, k1, v1))
    o0, o1 = torch.empty_like(q), torch.empty_like(q)
    lse0 = torch.empty(b, h, sq, device=q.device, dtype=torch.float32)
    lse1 = torch.empty_like(lse0)
    if o0.numel() == 0:
        return o0, lse0, o1, lse1
    f = features.get()
    cfg = _fwd_cfg(f)
    with torch.cuda.device(q.device):
        rc = _lib.lib().wf_fwd_dual(_ptr(q), _ptr(k0), _ptr(v0), _ptr(k1), _ptr(v1), _ptr(o0), _ptr(o1),
                                    _ptr(lse0), _ptr(lse1), b, sq, k0.shape[1], k1.shape[1], h,
                                    ctypes.byref(cfg), ctypes.c_void_p(_stream_ptr(q.device)))
    _lib.check(rc)
    return o0, lse0, o1, lse1


def wan_flash_bwd_dual(q, k0, v0, k1, v1, o0, lse0, o1, lse1, do, do1=None):
    """Backward of wan_flash_fwd_dual: (dq, dk0, dv0, dk1, dv1) given dO of
    o0 + o1 (``do``), or of o0 and o1 separately (``do``, ``do1``).  Both
    contexts add into one dQ accumulator that is zeroed and converted once."""
    dos = do if do1 is None else (do, do1)
    dq, ((dk0, dv0), (dk1, dv1)) = _bwd_multi(q, ((k0, v0, o0, lse0), (k1, v1, o1, lse1)), dos)
    return dq, dk0, dv0, dk1, dv1


class _WanFlashAttnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v):
        o, lse = wan_flash_fwd(q, k, v)
        ctx.save_for_backward(q, k, v, o, lse)
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = wan_flash_bwd(q, k, v, o, lse, do)
        return dq, dk, dv


def wan_flash_attn(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
    """Differentiable attention: our fwd + our bwd. Returns o (b,s,h,d) bf16."""
    return _WanFlashAttnFn.apply(q, k, v)


class _WanFlashAttnDualFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k0, v0, k1, v1):
        o0, lse0, o1, lse1 = wan_flash_fwd_dual(q, k0, v0, k1, v1)
        ctx.save_for_backward(q, k0, v0, k1, v1, o0, lse0, o1, lse1)
        return o0 + o1

    @staticmethod
    def backward(ctx, do):
        return wan_flash_bwd_dual(*ctx.saved_tensors, do.contiguous())


def wan_flash_attn_dual(q: torch.Tensor, k0: torch.Tensor, v0: torch.Tensor, k1: torch.Tensor, v1: torch.Tensor):
    """Differentiable attention(q, k0, v0) + attention(q, k1, v1) (the Wan I2V
    text + image cross attention) with the two-context kernels."""
    return _WanFlashAttnDualFn.apply(q, k0, v0, k1, v1)
