"""The header-only kl API compiled as a host program: the compile-time checks restating the
reference's unit tests, plus a host main() (tests/native/test_kl_headers.cu)."""

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def nvcc():
    return shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"


def test_headers_compile_and_pass(tmp_path):
    exe = tmp_path / "test_kl_headers"
    cmd = [nvcc(), "-std=c++20", "--expt-relaxed-constexpr", "-gencode", "arch=compute_100a,code=sm_100a",
           "-I", str(ROOT / "include"), str(ROOT / "tests" / "native" / "test_kl_headers.cu"), "-o", str(exe)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failures" in r.stdout


def test_product_headers_pull_in_no_cutlass():
    """The product include graph (kl headers, GEMM kernel, C ABI) reaches no CUTLASS/CuTe header:
    the same kind of allow-list check as kernel_lib/tools/check_includes.py:15-58, stricter."""
    src = "#include <kl/kl.hpp>\n#include <kl/gemm/gemm.hpp>\n#include <kl_gemm.h>\n"
    r = subprocess.run([nvcc(), "-std=c++20", "--expt-relaxed-constexpr", "-arch=sm_100a", "-I", str(ROOT / "include"),
                        "-M", "-x", "cu", "-"], input=src, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    deps = [t for t in r.stdout.replace("\\\n", " ").split() if t.endswith((".h", ".hpp", ".cuh"))]
    assert any("kl/gemm/gemm_kernel.cuh" in d for d in deps)
    bad = [d for d in deps if "/cute/" in d or "/cutlass/" in d or "cublas" in d.lower()]
    assert not bad, bad
