"""Build the sm_100a CUDA library in-tree: ``python -m wan_flash.build``.

One nvcc invocation compiles ``csrc/wf_lib.cu`` (a single translation unit
that includes every kernel and the C ABI) into ``wan_flash/libwanflash.so``
for ``compute_100a``/``sm_100a``.  The CUDA runtime is linked statically and
the driver is reached through ``cudaGetDriverEntryPoint``, so the library
loads on a machine without a GPU (it only fails when a call needs one).
"""

from __future__ import annotations

import os
import pathlib
import shutil
import subprocess
import sys

PKG = pathlib.Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libwanflash.so"
SOURCES = ["wf_lib.cu", "wf_capi.cu", "wf_fwd.cu", "wf_fwd2.cu", "wf_bwd.cu", "wf_bwd2.cu", "wf_aux.cu", "wf_noalloc.cu", "wf_common.cuh",
           "wf_kernels.h"]

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-Xcompiler", "-fPIC",
    "-shared",
    "-cudart", "static",
]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the sm_100a library cannot be built")
    return cand


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + [ROOT / "include" / "wan_flash.h"]
    return any(p.exists() and p.stat().st_mtime > t for p in deps)


def build(force: bool = False, verbose: bool = False) -> pathlib.Path:
    if not force and not needs_build():
        return LIB
    cmd = [nvcc_path(), *NVCC_FLAGS, f"-I{ROOT / 'include'}", "-o", str(LIB) + ".tmp", str(CSRC / "wf_lib.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    res = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or res.returncode != 0:
        sys.stdout.write(res.stdout)
        sys.stderr.write(res.stderr)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed with code {res.returncode}")
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv or "--verbose" in sys.argv)
    print(LIB)
