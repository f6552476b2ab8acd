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


def test_cmake_consumer_builds_against_kl_target(tmp_path):
    """A C++ consumer links kl::kl from the repository's CMakeLists.txt (the reference exports the
    same INTERFACE target name) and runs the header checks."""
    import shutil
    import subprocess

    cmake = shutil.which("cmake")
    if cmake is None:
        pytest.skip("cmake not installed")
    build = tmp_path / "build"
    cfg = subprocess.run([cmake, "-S", str(ROOT), "-B", str(build), "-DKL_BUILD_LIBRARY=OFF", "-DKL_BUILD_EXAMPLES=ON",
                          "-DCMAKE_BUILD_TYPE=Release"], capture_output=True, text=True)
    if cfg.returncode != 0 and "CUDA" in (cfg.stderr + cfg.stdout) and "not" in (cfg.stderr + cfg.stdout):
        pytest.skip("CMake found no usable CUDA toolkit here")
    assert cfg.returncode == 0, cfg.stdout + cfg.stderr
    bld = subprocess.run([cmake, "--build", str(build), "--target", "kl_header_example"], capture_output=True, text=True)
    assert bld.returncode == 0, bld.stdout + bld.stderr
    run = subprocess.run([str(build / "kl_header_example")], capture_output=True, text=True)
    assert run.returncode == 0, run.stdout + run.stderr


def test_stream_k_schedule(tmp_path):
    """The tile kernels' work schedule on the host: every (tile, K-block) unit dealt exactly once,
    the split tail before the whole tiles, every K-range of a tail tile once and never empty, and
    tn_schedule's decisions on the N-sharded shapes (tests/native/test_stream_k_schedule.cu)."""
    exe = tmp_path / "test_stream_k_schedule"
    cmd = [nvcc(), "-std=c++20", "--expt-relaxed-constexpr", "-gencode", "arch=compute_100a,code=sm_100a",
           "-I", str(ROOT / "include"), str(ROOT / "tests" / "native" / "test_stream_k_schedule.cu"), "-o", str(exe)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    assert " 0 failures" in r.stdout


def test_library_build_tracks_every_header():
    """The library is rebuilt when any header its sources can include changes, the .cuh kernel
    headers included (an edit to one of them alone must not leave a stale libkl_b200.so)."""
    from maia_b200 import build as b

    tracked = {p.resolve() for p in b.HEADERS}
    for p in (ROOT / "include").rglob("*"):
        if p.suffix in (".h", ".hpp", ".cuh"):
            assert p.resolve() in tracked, p
    assert any(p.name == "gemm_kernel.cuh" for p in tracked)
