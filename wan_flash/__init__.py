"""wan_flash (B200 / sm_100a): Wan attention forward + backward.

Drop-in for the reference package's public API (Quarky93/wan-flash):
``wan_flash.interface.{wan_flash_fwd, wan_flash_bwd, wan_flash_attn}``,
``wan_flash.features`` and ``wan_flash.shapes``.  The kernels live in
``libwanflash.so`` (built from ``csrc/`` by ``python -m wan_flash.build``).
"""

__version__ = "1.0.0"
