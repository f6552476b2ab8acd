"""Loaders for the golden fixtures made by tests/golden/gen_golden.py."""

import hashlib
import json
from functools import lru_cache
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"
ELEM_BYTES = {"bf16": 2, "f16": 2, "f32": 4, "i8": 1, "e4m3": 1, "e5m2": 1}


@lru_cache(None)
def host_tables():
    return json.loads((GOLDEN / "ref_host_tables.json").read_text())


@lru_cache(None)
def known_answers():
    return json.loads((GOLDEN / "ref_test_known_answers.json").read_text())


def tiles():
    return [t for t in host_tables() if t["kind"] == "tile"]


def idescs():
    return [t for t in host_tables() if t["kind"] == "idesc"]


def tile_id(t):
    return f"{t['type']}_{t['rows']}x{t['cols']}_sw{t['swizzle']}"


def sha(values) -> str:
    return hashlib.sha256(np.asarray(values, dtype="<i8").tobytes()).hexdigest()


def mn_tiles():
    return [t for t in host_tables() if t["kind"] == "mn_tile"]


def idesc_majors():
    return [t for t in host_tables() if t["kind"] == "idesc_major"]
