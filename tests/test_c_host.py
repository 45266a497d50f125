"""The C ABI from a plain C program (tests/c_host/wf_c_host.c): compiled with
gcc against include/wan_flash.h and linked with libwanflash.so, as a C/C++
host or another language's FFI would use it.  CPU: it compiles and links.
GPU: it runs the forward, the backward chain and wf_bwd_noalloc on a small
problem and checks them against its own double-precision reference."""

import pathlib
import shutil
import subprocess

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
SRC = ROOT / "tests" / "c_host" / "wf_c_host.c"
LIB_DIR = ROOT / "wan_flash"
CUDA_LIB = pathlib.Path("/usr/local/cuda/lib64")


def _build(out: pathlib.Path) -> pathlib.Path:
    if shutil.which("gcc") is None or not (CUDA_LIB / "libcudart.so").exists():
        pytest.skip("gcc or the CUDA runtime library is not available")
    if not (LIB_DIR / "libwanflash.so").exists():
        pytest.skip("libwanflash.so is not built")
    exe = out / "wf_c_host"
    cmd = ["gcc", "-O2", "-std=c11", "-Wall", "-Werror", f"-I{ROOT / 'include'}",
           "-I/usr/local/cuda/include", str(SRC), "-o", str(exe), f"-L{LIB_DIR}", "-lwanflash", f"-L{CUDA_LIB}",
           "-lcudart", "-lm", f"-Wl,-rpath,{LIB_DIR}", f"-Wl,-rpath,{CUDA_LIB}"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    return exe


def test_c_host_compiles_and_links(tmp_path):
    _build(tmp_path)


@pytest.mark.gpu
def test_c_host_runs_and_matches_its_reference(tmp_path):
    exe = _build(tmp_path)
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    print(res.stdout)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "C host: OK" in res.stdout
