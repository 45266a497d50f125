"""Wan2.1 attention shape registry + tile arithmetic.

Same registry as the reference (``wan_flash/shapes.py:10-45`` of
Quarky93/wan-flash): the Wan constants, ``WanShape`` with ``blocks()`` and
``fwd_ctas()``, and the shape lists.  ``SM_COUNT`` is the B200's 148 SMs;
``sm_count()`` asks the current device instead of trusting the constant.
"""

from dataclasses import dataclass

HEAD_DIM = 128
S_480P = 32760   # 21 x 30 x 52
S_720P = 75600   # 21 x 45 x 80
TEXT_LEN = 512
CLIP_LEN = 257
SM_COUNT = 148   # B200 (2 dies x 74 SMs)

FWD_TILE_M = 256  # query rows per forward CTA (two 128-row tiles)
BWD_TILE_M = 128  # query rows per backward m-block
TILE_N = 128      # key/value rows per block


def sm_count() -> int:
    """SM count of the current CUDA device (``SM_COUNT`` without a device)."""
    try:
        import torch

        if torch.cuda.is_available():
            return torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    except Exception:  # pragma: no cover - torch missing or broken driver
        pass
    return SM_COUNT


@dataclass(frozen=True)
class WanShape:
    kind: str      # "self" | "cross"
    b: int
    h: int
    sq: int
    skv: int
    d: int = HEAD_DIM

    @property
    def name(self):
        return f"{self.kind}_h{self.h}_sq{self.sq}_skv{self.skv}"

    def blocks(self, m_block: int, n_block: int):
        """(m_blocks, m_tail, n_blocks, n_tail); only the last n-block needs key predication."""
        mb, mt = -(-self.sq // m_block), self.sq % m_block
        nb, nt = -(-self.skv // n_block), self.skv % n_block
        return mb, mt, nb, nt

    def fwd_ctas(self, m_block: int = FWD_TILE_M):
        return self.b * self.h * self.blocks(m_block, m_block)[0]

    def fwd_flops(self) -> float:
        """4 * b * h * sq * skv * d (two GEMMs of 2*sq*skv*d each)."""
        return 4.0 * self.b * self.h * self.sq * self.skv * self.d

    def bwd_flops(self) -> float:
        """2.5x the forward (five GEMMs), the reference's convention."""
        return 2.5 * self.fwd_flops()


SELF_SHAPES = [WanShape("self", 1, h, s, s) for h in (12, 40) for s in (S_480P, S_720P)]
CROSS_SHAPES = [WanShape("cross", 1, h, s, TEXT_LEN) for h in (12, 40) for s in (S_480P, S_720P)]
ALL_SHAPES = SELF_SHAPES + CROSS_SHAPES
PRIMARY = [s for s in ALL_SHAPES if s.h == 12]  # 1.3B first
