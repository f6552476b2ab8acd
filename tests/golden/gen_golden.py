"""Regenerate the golden descriptor fixtures from the reference itself.

Run with REF_ROOT naming a checkout of the reference sources (the directory holding kernel_lib/;
there is no default) and the CUTLASS/CuTe headers importable through flashinfer:

    REF_ROOT=<maia checkout> python tests/golden/gen_golden.py

1. ref_host_tables.json: oracle/_ref/ref_host_dump, i.e. the reference's own headers
   (kernel_lib/include/kl) compiled against CuTe 4.5.0, evaluated on the host: smem layouts
   (physical offsets through tile.tensor(), and the un-swizzled layout_b), TmaBox geometry,
   block_offset_16B, the UMMA smem descriptor body at shared address 0, and instruction
   descriptors; plus CuTe's own MN-major operand tiles and make_umma_desc<Major::MN> (the reference
   is K-major only) and CuTe's block-scaled (MXFP8) instruction descriptors, with and without
   scale-factor ids. Large offset arrays are stored as SHA-256 of their little-endian int64 bytes
   plus a 64-entry prefix.
2. ref_test_known_answers.json: the known answers written into the reference's unit tests,
   extracted from the test sources as text (file:line recorded with each).
"""

from __future__ import annotations

import hashlib
import json
import os
import re
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
# The reference checkout (its kernel_lib/ sources); given by the caller, e.g.
#   REF_ROOT=<maia checkout> python tests/golden/gen_golden.py
_REF_ENV = os.environ.get("REF_ROOT")
REF_ROOT = Path(_REF_ENV) if _REF_ENV else None


def sha(values) -> str:
    return hashlib.sha256(np.asarray(values, dtype="<i8").tobytes()).hexdigest()


def require_ref_root() -> Path:
    if REF_ROOT is None or not (REF_ROOT / "kernel_lib" / "include").is_dir():
        sys.exit("gen_golden: set REF_ROOT to a checkout of the reference (the directory holding kernel_lib/); "
                 f"got {_REF_ENV!r}")
    return REF_ROOT


def host_tables() -> list:
    ref = require_ref_root()
    subprocess.run(["make", "-C", str(ROOT / "oracle"), "ref", f"REF={ref / 'kernel_lib' / 'include'}"], check=True)
    with tempfile.TemporaryDirectory() as tmp:
        out = Path(tmp) / "t.json"
        subprocess.run([str(ROOT / "oracle" / "_ref" / "ref_host_dump"), str(out)], check=True,
                       stdout=subprocess.DEVNULL)
        raw = json.loads(out.read_text())
    tables = []
    for e in raw:
        if e["kind"] == "tile":
            t = {k: v for k, v in e.items() if k not in ("layout", "tensor", "layout_b")}
            t["tensor_sha256"] = sha(e["tensor"])
            t["tensor_prefix"] = e["tensor"][:64]
            t["layout_b_sha256"] = sha(e["layout_b"])
            t["layout_b_prefix"] = e["layout_b"][:64]
            tables.append(t)
        elif e["kind"] == "mn_tile":
            t = {k: v for k, v in e.items() if k != "tensor"}
            t["tensor_sha256"] = sha(e["tensor"])
            t["tensor_prefix"] = e["tensor"][:64]
            tables.append(t)
        else:
            tables.append(e)
    return tables


def known_answers() -> list:
    tests = REF_ROOT / "kernel_lib" / "tests" / "unit"
    out = []

    def find(path: Path, pattern: str):
        for i, line in enumerate(path.read_text().splitlines(), 1):
            m = re.search(pattern, line)
            if m:
                return i, m
        raise SystemExit(f"pattern {pattern!r} not found in {path}")

    p = tests / "test_umma_desc.cu"
    ln, m = find(p, r"static_assert\(expected == (0x[0-9a-fA-F]+)u\)")
    out.append({"what": "idesc bf16 x bf16 -> f32, M=128, N=256, K-major", "a": "bf16", "b": "bf16", "acc": "f32",
                "m": 128, "n": 256, "value": m.group(1).lower(), "source": f"kernel_lib/tests/unit/test_umma_desc.cu:{ln}"})
    ln, _ = find(p, r"stride_byte_offset_\), 1024 / 16")
    out.append({"what": "smem desc bf16 128x64 SW128 fields", "type": "bf16", "rows": 128, "cols": 64, "swizzle": 128,
                "layout_type": 2, "version": 1, "stride_byte_offset": 64, "leading_byte_offset": 1, "base_offset": 0,
                "start_step_per_k_block": 2, "source": f"kernel_lib/tests/unit/test_umma_desc.cu:{ln - 2}-{ln + 4}"})
    ln, _ = find(p, r"second.start_address_\), int\(\(d.base \+ 32 \* 1024\) >> 4\)")
    out.append({"what": "bf16 512x64 SW128, row block 256 starts 32 KB in", "type": "bf16", "rows": 512, "cols": 64,
                "swizzle": 128, "row": 256, "start_offset_bytes": 32768, "base_offset": 0,
                "source": f"kernel_lib/tests/unit/test_umma_desc.cu:{ln}"})
    p = tests / "test_smem_tile.cu"
    ln, m = find(p, r"constexpr int expected\[4\]\[3\] = \{(.*)\};")
    rows = [list(map(int, x)) for x in re.findall(r"\{(\d+), (\d+), (\d+)\}", m.group(1))]
    out.append({"what": "TmaBox bf16 512x128 SW128: (row, col, smem byte offset) per box", "type": "bf16", "rows": 512,
                "cols": 128, "swizzle": 128, "boxes": rows, "source": f"kernel_lib/tests/unit/test_smem_tile.cu:{ln}"})
    ln, _ = find(p, r"smem_offset\(1\), 128u \* 64 \* 2")
    out.append({"what": "TmaBox bf16 128x128 SW128: second box 16 KB in", "type": "bf16", "rows": 128, "cols": 128,
                "swizzle": 128, "boxes": [[0, 0, 0], [0, 64, 16384]], "source": f"kernel_lib/tests/unit/test_smem_tile.cu:{ln - 1}-{ln}"})
    ln, _ = find(p, r"static_assert\(A::alignment == 1024\)")
    out.append({"what": "SmemTile<bf16,128,64> sizes", "type": "bf16", "rows": 128, "cols": 64, "swizzle": 128,
                "bytes": 16384, "alignment": 1024, "atom_elems": 64, "source": f"kernel_lib/tests/unit/test_smem_tile.cu:{ln - 1}-{ln + 3}"})
    ln, _ = find(p, r"static_assert\(C::alignment == 512\)")
    out.append({"what": "SmemTile<bf16,128,32,SW64> sizes", "type": "bf16", "rows": 128, "cols": 32, "swizzle": 64,
                "alignment": 512, "atom_elems": 32, "source": f"kernel_lib/tests/unit/test_smem_tile.cu:{ln - 1}-{ln + 1}"})
    ln, _ = find(p, r"static_assert\(W::atom_elems == 128\)")
    out.append({"what": "SmemTile<int8,128,128> sizes", "type": "i8", "rows": 128, "cols": 128, "swizzle": 128,
                "bytes": 16384, "atom_elems": 128, "source": f"kernel_lib/tests/unit/test_smem_tile.cu:{ln - 1}-{ln + 1}"})
    p = tests / "test_tma_desc.cu"
    text = p.read_text().splitlines()
    errs = []
    for i, line in enumerate(text, 1):
        if "EXPECT_THROW(kl::make_tma_load<A>(" in line:
            errs.append({"line": i, "code": line.strip()})
    out.append({"what": "make_tma_load error cases (std::invalid_argument)", "cases": errs,
                "source": f"kernel_lib/tests/unit/test_tma_desc.cu:{errs[0]['line']}-{errs[-1]['line']}"})
    return out


def main() -> int:
    require_ref_root()
    (HERE / "ref_host_tables.json").write_text(json.dumps(host_tables(), indent=1) + "\n")
    (HERE / "ref_test_known_answers.json").write_text(json.dumps(known_answers(), indent=1) + "\n")
    print("wrote", HERE / "ref_host_tables.json", HERE / "ref_test_known_answers.json")
    return 0


if __name__ == "__main__":
    sys.exit(main())
