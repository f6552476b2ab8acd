"""The plain-Python descriptor oracle (oracle/descriptors.py) against the reference's own outputs:
its compiled headers (golden tables) and the known answers in its unit tests."""

import pytest

from golden_util import ELEM_BYTES, idescs, known_answers, sha, tile_id, tiles
from oracle import descriptors as od


@pytest.mark.parametrize("t", tiles(), ids=tile_id)
def test_layouts_match_reference(t):
    eb, R, C, S = ELEM_BYTES[t["type"]], t["rows"], t["cols"], t["swizzle"]
    phys = [od.physical_offset(R, C, eb, S, r, c) for r in range(R) for c in range(C)]
    plain = [od.tile_offset(R, C, eb, S, r, c) for r in range(R) for c in range(C)]
    assert phys[:64] == t["tensor_prefix"] and sha(phys) == t["tensor_sha256"]
    assert plain[:64] == t["layout_b_prefix"] and sha(plain) == t["layout_b_sha256"]
    assert od.atom_elems(eb, S) == t["atom_elems"]


@pytest.mark.parametrize("t", tiles(), ids=tile_id)
def test_tma_box_matches_reference(t):
    eb, R, C, S = ELEM_BYTES[t["type"]], t["rows"], t["cols"], t["swizzle"]
    box = od.tma_box(R, C, eb, S)
    for k in ("inner", "outer", "col_boxes", "row_boxes", "count", "bytes", "pos"):
        assert box[k] == t["box"][k], k


@pytest.mark.parametrize("t", [t for t in tiles() if "umma_desc_base0" in t], ids=tile_id)
def test_umma_desc_matches_reference(t):
    eb, R, C, S = ELEM_BYTES[t["type"]], t["rows"], t["cols"], t["swizzle"]
    for row, k, off in t["block_offset_16B"]:
        assert od.block_offset_16B(R, C, eb, S, k, row) == off
    for row, k, val in t["umma_desc_base0"]:
        assert od.umma_smem_desc(R, C, eb, S, k, row) == int(val, 16), (row, k)


@pytest.mark.parametrize("d", idescs(), ids=lambda d: f"{d['a']}_{d['acc']}_m{d['m']}_n{d['n']}_{d['source']}")
def test_instr_desc_matches_reference(d):
    assert od.instr_desc(d["a"], d["b"], d["acc"], d["m"], d["n"]) == int(d["value"], 16)


def test_known_answers_from_reference_tests():
    for ka in known_answers():
        if ka["what"].startswith("idesc"):
            assert od.instr_desc(ka["a"], ka["b"], ka["acc"], ka["m"], ka["n"]) == int(ka["value"], 16)
        elif ka["what"].startswith("TmaBox"):
            box = od.tma_box(ka["rows"], ka["cols"], ELEM_BYTES[ka["type"]], ka["swizzle"])
            assert [p for p in box["pos"]][: len(ka["boxes"])] == ka["boxes"]
        elif ka["what"].startswith("smem desc"):
            for k in range(4):
                d = od.umma_smem_desc(128, 64, 2, 128, k, start=0x1000)
                assert d >> 61 == ka["layout_type"] and (d >> 46) & 3 == ka["version"]
                assert (d >> 32) & 0x3FFF == ka["stride_byte_offset"]
                assert (d >> 16) & 0x3FFF == ka["leading_byte_offset"]
                assert (d >> 49) & 7 == ka["base_offset"]
                assert d & 0x3FFF == (0x1000 >> 4) + ka["start_step_per_k_block"] * k
        elif ka["what"].startswith("bf16 512x64"):
            d = od.umma_smem_desc(512, 64, 2, 128, 0, row=ka["row"], start=0x1000)
            assert d & 0x3FFF == (0x1000 + ka["start_offset_bytes"]) >> 4 and (d >> 49) & 7 == 0


def test_tma_args_and_errors():
    # The C2 operand A: 4096 x 4096 bf16, tile 128 x 64, 128-byte swizzle.
    args = od.tma_encode_args(2, 128, 64, 128, 0x10000, [4096, 4096], [4096, 1])
    assert args["dims"] == [4096, 4096] and args["strides"] == [8192] and args["box"] == [64, 128]
    # The error cases of kernel_lib/tests/unit/test_tma_desc.cu:102-107.
    assert "16-byte aligned" in od.tma_encode_args(2, 128, 64, 128, 0x10002, [4096, 4096], [4096, 1])
    assert "rows overlap" in od.tma_encode_args(2, 128, 64, 128, 0x10000, [4096, 4096], [1024, 1])
    assert "multiples of 16 bytes" in od.tma_encode_args(2, 128, 64, 128, 0x10000, [4096, 4100], [4100, 1])
    assert "extents" in od.tma_encode_args(2, 128, 64, 128, 0x10000, [0, 4096], [4096, 1])
    assert isinstance(od.tma_encode_args(2, 128, 64, 128, 0x10000, [4096, 4096], [4160, 1]), dict)  # padded rows


def test_block_scaled_instr_desc_matches_cute():
    """The restated block-scaled layout against CuTe's make_instr_desc_block_scaled for every row
    the reference dump holds (MXFP8, MXFP6, MXFP4, NVFP4; with and without scale-factor ids)."""
    from golden_util import host_tables

    rows = [t for t in host_tables() if t["kind"] == "idesc_block_scaled"]
    assert len(rows) == 29
    for d in rows:
        a, _, sf = d["a"].partition("/")
        b = d["b"].partition("/")[0]
        got = od.instr_desc_block_scaled(a, b, d["m"], d["n"], d["a_sf_id"], d["b_sf_id"], ue4m3=sf == "ue4m3")
        assert got == int(d["value"], 16), d
