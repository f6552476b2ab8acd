"""Build recipe for libkl_b200.so (the CUDA kernels and the C ABI), in-tree, for sm_100a.

Run as a module (``python -m maia_b200.build``) or call :func:`build`. The library is written next
to this file so that it travels with the repository snapshot to a GPU machine.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
LIB = PKG / "libkl_b200.so"
SOURCES = sorted((PKG / "csrc").glob("*.cu"))
# Every header the sources can include: .h / .hpp and the .cuh kernel headers.
HEADERS = sorted(p for p in (ROOT / "include").rglob("*") if p.suffix in (".h", ".hpp", ".cuh")) + \
    sorted((PKG / "csrc").glob("*.cuh"))

NVCC_FLAGS = [
    "-std=c++20",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every .cu under csrc/ and link libkl_b200.so (cudart linked statically)."""
    deps = list(SOURCES) + list(HEADERS) + [Path(__file__)]
    if not force and not _stale(LIB, deps):
        return LIB
    objdir = PKG / "_build"
    objdir.mkdir(exist_ok=True)
    cmds = []
    for src in SOURCES:
        obj = objdir / (src.stem + ".o")
        cmds.append([nvcc(), *NVCC_FLAGS, "-I", str(ROOT / "include"), "-c", str(src), "-o", str(obj)])
    objs = [c[-1] for c in cmds]

    def compile_one(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)

    # The translation units are independent: compile them side by side.
    with ThreadPoolExecutor(max_workers=max(1, min(len(cmds), os.cpu_count() or 1))) as pool:
        list(pool.map(compile_one, cmds))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", str(tmp), *objs,
           "-cudart", "static", "-Xlinker", "--no-undefined", "-ldl", "-lpthread", "-lrt"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
