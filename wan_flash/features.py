"""Feature-flag registry (same accessors as the reference's
``wan_flash/features.py:28-100``: ``get``, ``get_bwd``, ``set_overrides``,
``set_bwd_overrides``, ``reset``), with the B200 kernels' options.

Forward flags
  rescale_skip_threshold  skip the O rescale while the running row max grew by
                          at most this many log2 units (exact by max-shift
                          invariance; only rounding differs).  0.0 = always
                          rescale.
  scheduler               "auto" | "single" | "persistent".  "single": one CTA
                          per 256-row work item.  "persistent": one CTA per
                          SM looping over the items, so the next item's Q
                          load and first QK^T overlap the current item's
                          last blocks and epilogue.  "auto": persistent
                          when KV has at most 64 blocks of 128 keys (cross
                          attention and short self attention), else single
                          (the hardware's dynamic CTA placement balances
                          long items better than a static stride).
  num_sms                 persistent grid size; 0 = the device's SM count.
  tile_m / tile_n         fixed at 128 x 128 (two 128-row query tiles per CTA).
  num_stages              K/V ring depth in (K, V) pairs (fixed at 2).
  cluster_mn              (2, 1) (default): pairs of CTAs along the query axis
                          (cluster of 2) issue 2-SM tensor-core MMAs
                          (M = 256): each CTA supplies its own query rows
                          and loads half of every K/V tile, where the
                          reference's cluster (2, 1) multicasts whole K/V
                          tiles into both CTAs.  Used for one KV context on
                          the one-item-per-CTA schedule (long self
                          attention); the persistent and two-context paths
                          run single CTAs.  (1, 1): single CTAs everywhere.
                          No TMA load is multicast in either form.
  intra_wg_overlap        the two query tiles of a CTA ping-pong softmax and
                          tensor work (always on in this design).
  mma_pv_is_rs            P feeds the PV MMA from tensor memory (always on).

Backward flags
  tile_m / tile_n         fixed at 128 x 128.
  num_stages              2 (fixed): Q double-buffered; dO single-buffered,
                          refilled between dV(u) and dP(u+1) (shared
                          memory holds no second dO tile).
  nsplit                  split-M factor; 0 = auto (1 when the
                          (n_blocks*h*b) grid fills the GPU, otherwise the
                          smallest split with >= 95% wave efficiency).  With
                          nsplit > 1 dK/dV go through fp32 reductions and a
                          convert, which makes them nondeterministic.
  cluster_n               1 = one CTA per 128-row KV block; 2 = CTA pairs over
                          adjacent KV blocks of a head (cluster of 2): the
                          pair issues 2-SM tensor-core MMAs over its 256 KV
                          rows, each CTA loading and reading half of every
                          Q / dO tile and the pair reducing one dQ partial
                          per 256 KV rows.  Same purpose as the reference's
                          cluster_n = 2 (halve the Q/dO stream), reached
                          without multicast loads.
  deterministic           False (default): dQ (and split-M dK/dV) are fp32
                          reductions in arrival order.  True: contributions
                          are added in KV-block (split) order behind
                          per-block counters, so every gradient is bitwise
                          reproducible; slower, single-CTA kernel only.
  pdl                     True (default): the main kernel and the converts are
                          launched as programmatic dependents of the kernel
                          before them (the reference's use_pdl=True,
                          bwd_sm90.py:140,498,506): their set-up and the K/V
                          loads overlap the previous kernel's tail, and each
                          waits (griddepcontrol.wait) before reading its
                          results.  False launches the main kernel plainly.
"""

from dataclasses import dataclass, replace


@dataclass(frozen=True)
class FwdFeatures:
    rescale_skip_threshold: float = 8.0
    intra_wg_overlap: bool = True
    mma_pv_is_rs: bool = True
    num_stages: int = 2
    tile_m: int = 128
    tile_n: int = 128
    scheduler: str = "auto"
    cluster_mn: tuple = (2, 1)
    num_sms: int = 0


@dataclass(frozen=True)
class BwdFeatures:
    tile_m: int = 128
    tile_n: int = 128
    num_stages: int = 2
    nsplit: int = 0
    cluster_n: int = 1
    deterministic: bool = False
    pdl: bool = True


_current = FwdFeatures()
_current_bwd = BwdFeatures()


def _validate_fwd(f: FwdFeatures):
    if f.tile_m != 128 or f.tile_n != 128:
        raise ValueError("the sm_100a forward is built for 128x128 tiles")
    if f.num_stages != 2:
        raise ValueError("the forward K/V ring holds 2 (K, V) pairs")
    if tuple(f.cluster_mn) not in ((1, 1), (2, 1)):
        raise ValueError("cluster_mn must be (2, 1) (CTA pairs along the query axis) or (1, 1)")
    if f.scheduler not in ("auto", "single", "persistent"):
        raise ValueError(f"unknown scheduler {f.scheduler!r}")
    if f.num_sms < 0:
        raise ValueError("num_sms must be >= 0 (0 = the device's SM count)")
    if not (f.rescale_skip_threshold >= 0.0):
        raise ValueError("rescale_skip_threshold must be >= 0")
    if not f.intra_wg_overlap or not f.mma_pv_is_rs:
        raise ValueError("intra_wg_overlap and mma_pv_is_rs are structural in this design")


def _validate_bwd(f: BwdFeatures):
    if f.tile_m != 128 or f.tile_n != 128:
        raise ValueError("the sm_100a backward is built for 128x128 tiles")
    if f.num_stages != 2:
        raise ValueError("the backward's Q/dO staging is fixed (num_stages=2)")
    if f.nsplit < 0:
        raise ValueError("nsplit must be >= 0 (0 = auto)")
    if f.cluster_n not in (1, 2):
        raise ValueError("cluster_n must be 1 (single CTAs) or 2 (CTA pairs)")
    if f.deterministic and f.cluster_n != 1:
        raise ValueError("deterministic mode runs on the single-CTA kernel (cluster_n=1)")


def get() -> FwdFeatures:
    return _current


def get_bwd() -> BwdFeatures:
    return _current_bwd


def set_overrides(**kw):
    global _current
    new = replace(_current, **kw)
    _validate_fwd(new)
    _current = new
    return _current


def set_bwd_overrides(**kw):
    global _current_bwd
    new = replace(_current_bwd, **kw)
    _validate_bwd(new)
    _current_bwd = new
    return _current_bwd


def reset():
    global _current, _current_bwd
    _current = FwdFeatures()
    _current_bwd = BwdFeatures()
