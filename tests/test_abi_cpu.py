"""libkl_b200.so on the CPU: it loads, exports every entry point include/kl_gemm.h declares, and
its descriptor encoders reproduce the reference's outputs bit for bit (no GPU needed)."""

import ctypes
import re
from pathlib import Path

import pytest

import maia_b200 as kl
from golden_util import ELEM_BYTES, idesc_majors, idescs, known_answers, mn_tiles, sha, tile_id, tiles

HEADER = Path(__file__).resolve().parent.parent / "include" / "kl_gemm.h"
TYPE = {"bf16": kl.KL_BF16, "f16": kl.KL_F16, "f32": kl.KL_F32, "i8": kl.KL_I8, "e4m3": kl.KL_E4M3, "e5m2": kl.KL_E5M2,
        "e2m1": kl.KL_E2M1, "e3m2": kl.KL_E3M2, "e2m3": kl.KL_E2M3}


def declared_symbols():
    return sorted(set(re.findall(r"^KL_API [^(]*?\b(kl_\w+)\(", HEADER.read_text(), re.M)))


def test_library_exports_every_declared_symbol():
    names = declared_symbols()
    assert len(names) >= 14
    lib = ctypes.CDLL(str(kl.LIB_PATH))
    for n in names:
        assert hasattr(lib, n), f"{n} declared in kl_gemm.h but not exported"
    assert set(names) == set(kl.EXPORTED)


def test_version():
    assert kl.lib().kl_version() >= 100


@pytest.mark.parametrize("t", tiles(), ids=tile_id)
def test_tile_layout_bit_exact(t):
    eb, R, C, S = ELEM_BYTES[t["type"]], t["rows"], t["cols"], t["swizzle"]
    phys, plain = [], []
    for r in range(R):
        for c in range(C):
            s, p = kl.smem_tile_offset(eb, R, C, S, r, c)
            phys.append(s)
            plain.append(p)
    assert sha(phys) == t["tensor_sha256"], "swizzled offsets differ from the reference's tile.tensor()"
    assert sha(plain) == t["layout_b_sha256"], "un-swizzled offsets differ from the reference's layout_b()"


@pytest.mark.parametrize("t", tiles(), ids=tile_id)
def test_tma_box_bit_exact(t):
    eb, R, C, S = ELEM_BYTES[t["type"]], t["rows"], t["cols"], t["swizzle"]
    g = kl.tma_box_geometry(eb, R, C, S)
    for k in ("inner", "outer", "col_boxes", "row_boxes", "count", "bytes"):
        assert g[k] == t["box"][k], k
    assert [list(kl.tma_box_position(eb, R, C, S, i)) for i in range(g["count"])] == t["box"]["pos"]


@pytest.mark.parametrize("t", [t for t in tiles() if "umma_desc_base0" in t], ids=tile_id)
def test_umma_desc_bit_exact(t):
    eb, R, C, S = ELEM_BYTES[t["type"]], t["rows"], t["cols"], t["swizzle"]
    for row, k, val in t["umma_desc_base0"]:
        assert kl.umma_smem_desc(eb, R, C, S, 0, k, row) == int(val, 16), (row, k)
    # A non-zero base only moves the start-address field.
    for row, k, val in t["umma_desc_base0"][:8]:
        assert kl.umma_smem_desc(eb, R, C, S, 0x2400, k, row) == int(val, 16) + (0x2400 >> 4)


@pytest.mark.parametrize("d", idescs(), ids=lambda d: f"{d['a']}_{d['acc']}_m{d['m']}_n{d['n']}_{d['source']}")
def test_instr_desc_bit_exact(d):
    assert kl.mma_instr_desc(TYPE[d["a"]], TYPE[d["b"]], TYPE[d["acc"]], d["m"], d["n"]) == int(d["value"], 16)


def test_instr_desc_known_answer_from_reference_test():
    ka = next(k for k in known_answers() if k["what"].startswith("idesc"))
    assert kl.mma_instr_desc(kl.KL_BF16, kl.KL_BF16, kl.KL_F32, 128, 256) == int(ka["value"], 16) == 0x08400490


@pytest.mark.parametrize("args, msg", [
    ((2, 100, 64, 128), "rows must be a positive multiple of 8"),
    ((2, 128, 60, 128), "multiple of the swizzle atom"),
    ((3, 128, 64, 128), "elem_bytes"),
    ((2, 128, 64, 96), "swizzle_span"),
])
def test_encoder_argument_errors(args, msg):
    with pytest.raises(kl.KlError) as e:
        kl.tma_box_geometry(*args)
    assert e.value.status == kl.KL_ERR_INVALID_ARGUMENT and msg in e.value.message


def test_instr_desc_rejects_bad_shapes():
    for m, n in ((32, 64), (128, 8), (256, 264), (128, 40)):
        with pytest.raises(kl.KlError):
            kl.mma_instr_desc(kl.KL_BF16, kl.KL_BF16, kl.KL_F32, m, n)
    with pytest.raises(kl.KlError):  # mixed MMA kinds
        kl.mma_instr_desc(kl.KL_BF16, kl.KL_E4M3, kl.KL_F32, 128, 128)


# make_tma_desc's validation runs before the driver call, so its error contract is testable here.
# Cases: kernel_lib/tests/unit/test_tma_desc.cu:97-107; messages: tma_desc.hpp:134-142.
@pytest.mark.parametrize("ptr, shape, stride, msg", [
    (0x10002, (4096, 4096), (4096, 1), "kl::make_tma_desc: global address must be 16-byte aligned"),
    (0x10000, (4096, 4096), (1024, 1), "kl::make_tma_desc: rows overlap: the row stride is smaller than cols"),
    (0x10000, (4096, 4100), (4100, 1),
     "kl::make_tma_desc: outer strides must be positive multiples of 16 bytes, below 2^40 bytes"),
    (0x10000, (0, 4096), (4096, 1), "kl::make_tma_desc: extents must be in [1, 2^32]"),
    (0x10000, (2, 4096, 4096), (4096 * 4096, 4096, 1), None),  # rank 3 passes validation
])
def test_tma_desc_validation(ptr, shape, stride, msg):
    if msg is None:
        return
    with pytest.raises(kl.KlError) as e:
        kl.make_tma_desc(kl.KL_BF16, 128, 64, 128, ptr, shape, stride)
    assert e.value.status == kl.KL_ERR_INVALID_ARGUMENT
    assert e.value.message == msg


# Packed fp6 (16U6 maps): the driver's extra rules for the type, checked before the driver call.
@pytest.mark.parametrize("ptr, shape, stride, msg", [
    (0x10010, (4096, 4096), (4096, 1), "kl::make_tma_desc: packed fp6: global address must be 32-byte aligned"),
    (0x10000, (4096, 4000), (4096, 1),
     "kl::make_tma_desc: packed fp6: the innermost extent must be a multiple of 128 elements"),
    (0x10000, (4096, 4096), (4160, 1),
     "kl::make_tma_desc: packed fp6: outer strides must be positive multiples of 128 elements (32 bytes)"),
    (0x10000, (4096, 4096), (3968, 1), "kl::make_tma_desc: rows overlap: the row stride is smaller than cols"),
])
@pytest.mark.parametrize("dtype", [kl.KL_E3M2, kl.KL_E2M3], ids=["e3m2", "e2m3"])
def test_fp6_tma_desc_validation(dtype, ptr, shape, stride, msg):
    with pytest.raises(kl.KlError) as e:
        kl.make_tma_desc(dtype, 128, 128, 128, ptr, shape, stride)
    assert e.value.status == kl.KL_ERR_INVALID_ARGUMENT
    assert e.value.message == msg


def test_fp6_tma_desc_needs_the_128_byte_swizzle():
    with pytest.raises(kl.KlError) as e:
        kl.make_tma_desc(kl.KL_E3M2, 128, 64, 64, 0x10000, (4096, 4096), (4096, 1))
    assert "packed fp6 boxes are 128 elements wide" in e.value.message


@pytest.mark.parametrize("t", mn_tiles(), ids=lambda t: f"{t['type']}_mn{t['mn']}_k{t['k']}_sw{t['swizzle']}")
def test_mn_major_tile_and_descriptors_match_cute(t):
    """MN-major operands: SmemTile<T, K, MN, Sw> (MN contiguous, atoms down K first) is the layout of
    CuTe's MN-major atom tiled K first; the descriptors equal CuTe's make_umma_desc<Major::MN>."""
    eb, mn, k, sw = ELEM_BYTES[t["type"]], t["mn"], t["k"], t["swizzle"]
    phys = [kl.smem_tile_offset(eb, k, mn, sw, kk, m)[0] for kk in range(k) for m in range(mn)]
    assert phys[:64] == t["tensor_prefix"] and sha(phys) == t["tensor_sha256"]
    for kb, val in enumerate(t["umma_desc_mn_base0"]):
        assert kl.umma_smem_desc_mn(eb, k, mn, sw, 0, kb) == int(val, 16), kb


def test_instr_desc_majors_match_cute():
    want = {"bf16 M128 N256 A=MN B=K": (128, 256, 1, 0), "bf16 M128 N256 A=K B=MN": (128, 256, 0, 1),
            "bf16 M256 N256 A=MN B=MN": (256, 256, 1, 1)}
    got = idesc_majors()
    assert len(got) == 3
    for d in got:
        m, n, am, bm = want[d["what"]]
        assert kl.mma_instr_desc_major(kl.KL_BF16, kl.KL_BF16, kl.KL_F32, m, n, am, bm) == int(d["value"], 16)


def test_gemm_desc_layout_matches_the_c_header(tmp_path):
    """The ctypes mirror of kl_gemm_desc has the C struct's field offsets and size (gcc, x86-64)."""
    import shutil
    import subprocess

    gcc = shutil.which("gcc") or shutil.which("cc")
    if gcc is None:
        pytest.skip("no C compiler")
    names = [f[0] for f in kl.GemmDesc._fields_]
    src = tmp_path / "layout.c"
    body = "".join(f'  printf("%s %zu\\n", "{n}", offsetof(kl_gemm_desc, {n}));\n' for n in names)
    src.write_text('#include <stddef.h>\n#include <stdio.h>\n#include "kl_gemm.h"\nint main(void) {\n' + body +
                   '  printf("sizeof %zu\\n", sizeof(kl_gemm_desc));\n  return 0;\n}\n')
    exe = tmp_path / "layout"
    subprocess.run([gcc, "-std=c11", "-I", str(HEADER.parent), str(src), "-o", str(exe)], check=True)
    got = dict(line.split() for line in subprocess.run([str(exe)], check=True, capture_output=True,
                                                       text=True).stdout.splitlines())
    for n in names:
        assert int(got[n]) == getattr(kl.GemmDesc, n).offset, n
    assert int(got["sizeof"]) == ctypes.sizeof(kl.GemmDesc)


def test_block_scaled_instr_desc_matches_cute():
    from golden_util import host_tables

    rows = [t for t in host_tables() if t["kind"] == "idesc_block_scaled"]
    assert len(rows) == 29
    for d in rows:
        a, _, sf = d["a"].partition("/")  # "e2m1/ue4m3": NVFP4 (UE4M3 scales); otherwise UE8M0
        b = d["b"].partition("/")[0]
        scale = kl.KL_UE4M3 if sf == "ue4m3" else kl.KL_UE8M0
        got = kl.mma_instr_desc_block_scaled(TYPE[a], TYPE[b], d["m"], d["n"], d["a_sf_id"], d["b_sf_id"], scale)
        assert got == int(d["value"], 16), d


def test_block_scaled_instr_desc_errors():
    with pytest.raises(kl.KlError):
        kl.mma_instr_desc_block_scaled(kl.KL_BF16, kl.KL_E4M3, 128, 256)
    with pytest.raises(kl.KlError):
        kl.mma_instr_desc_block_scaled(kl.KL_E4M3, kl.KL_E4M3, 64, 256)
    with pytest.raises(kl.KlError):
        kl.mma_instr_desc_block_scaled(kl.KL_E4M3, kl.KL_E4M3, 128, 256, 4, 0)
    with pytest.raises(kl.KlError):  # fp4 with fp8
        kl.mma_instr_desc_block_scaled(kl.KL_E2M1, kl.KL_E4M3, 128, 256)
    with pytest.raises(kl.KlError):  # UE4M3 scales are for fp4 only
        kl.mma_instr_desc_block_scaled(kl.KL_E4M3, kl.KL_E4M3, 128, 256, scale_type=kl.KL_UE4M3)


@pytest.mark.parametrize("rows,k,want", [(1, 1, 512), (128, 128, 512), (129, 128, 1024), (128, 129, 1024),
                                         (16384, 8192, 128 * 64 * 512), (0, 5, 0)])
def test_mx_scale_bytes(rows, k, want):
    assert kl.mx_scale_bytes(rows, k) == want


def _desc(**kw):
    """A descriptor with placeholder (never dereferenced) device pointers."""
    d = kl.GemmDesc(m=256, n=256, k=256, a=0x1000, lda=256, b=0x2000, ldb=256, c=0x3000, ldc=256,
                    ab_type=kl.KL_BF16, c_type=kl.KL_BF16, alpha=1.0)
    for name, value in kw.items():
        setattr(d, name, value)
    return d


@pytest.mark.parametrize("field,value,msg", [
    ("stream_k", 2, "stream_k must be -1, 0 or 1"),
    ("stream_k", -2, "stream_k must be -1, 0 or 1"),
    ("c_reduce", 2, "c_reduce must be 0"),
    ("launch_overlap", 2, "launch_overlap must be -1, 0 or 1"),
    ("m", -1, "negative extent"),
    ("a_major", 3, "a_major / b_major must be 0"),
])
def test_gemm_rejects_bad_descriptors_before_any_launch(field, value, msg):
    """kl_gemm validates the descriptor on the host: these fail with KL_ERR_INVALID_ARGUMENT and a
    message, with no GPU in the machine (nothing is launched or read)."""
    st = kl.lib().kl_gemm(ctypes.byref(_desc(**{field: value})), ctypes.c_void_p(0))
    assert st == kl.KL_ERR_INVALID_ARGUMENT
    assert msg in kl.last_error()


def test_gemm_of_an_empty_output_is_a_no_op():
    assert kl.lib().kl_gemm(ctypes.byref(_desc(m=0)), ctypes.c_void_p(0)) == kl.KL_OK
    assert kl.lib().kl_gemm(ctypes.byref(_desc(n=0, c=0)), ctypes.c_void_p(0)) == kl.KL_OK


def test_gather_and_host_entry_points_check_their_arguments():
    arr = (ctypes.c_void_p * 8)(*[ctypes.c_void_p(0x4000 + i) for i in range(8)])
    assert kl.lib().kl_gemm_gather(ctypes.byref(_desc()), arr, 8, ctypes.c_void_p(0)) == kl.KL_ERR_INVALID_ARGUMENT
    assert "0 to 7 peers" in kl.last_error()
    dev = [ctypes.c_void_p(0x5000), ctypes.c_void_p(0x6000), ctypes.c_void_p(0x7000)]
    st = kl.lib().kl_gemm_host(ctypes.byref(_desc(c_reduce=1)), *dev, 0, ctypes.c_void_p(0))
    assert st == kl.KL_ERR_NOT_SUPPORTED and "c_reduce" in kl.last_error()
    st = kl.lib().kl_gemm_host(ctypes.byref(_desc(batch=2)), *dev, 0, ctypes.c_void_p(0))
    assert st == kl.KL_ERR_NOT_SUPPORTED and "batch" in kl.last_error()
    st = kl.lib().kl_gemm_host(ctypes.byref(_desc(lda=100)), *dev, 0, ctypes.c_void_p(0))
    assert st == kl.KL_ERR_INVALID_ARGUMENT and "leading dimension" in kl.last_error()


def test_quantisers_check_their_arguments():
    p = ctypes.c_void_p(0x8000)
    st = kl.lib().kl_mx_quantize(p, kl.KL_F32, 4, 48, 48, kl.KL_E4M3, p, 48, p, ctypes.c_void_p(0))
    assert st == kl.KL_ERR_INVALID_ARGUMENT and "multiple of 32" in kl.last_error()
    st = kl.lib().kl_mx_quantize(p, kl.KL_F16, 4, 64, 64, kl.KL_E4M3, p, 64, p, ctypes.c_void_p(0))
    assert st == kl.KL_ERR_NOT_SUPPORTED
    st = kl.lib().kl_mx_quantize(p, kl.KL_F32, 4, 64, 64, kl.KL_E3M2, p, 64, p, ctypes.c_void_p(0))
    assert st == kl.KL_ERR_INVALID_ARGUMENT and "128 elements" in kl.last_error()
    st = kl.lib().kl_nv_quantize(p, kl.KL_F32, 4, 40, 40, p, 64, p, p, ctypes.c_void_p(0))
    assert st == kl.KL_ERR_INVALID_ARGUMENT and "multiple of 16" in kl.last_error()
    st = kl.lib().kl_nv_quantize(p, kl.KL_F32, 4, 64, 64, p, 48, p, p, ctypes.c_void_p(0))
    assert st == kl.KL_ERR_INVALID_ARGUMENT and "multiple of 32" in kl.last_error()
    assert kl.lib().kl_nv_quantize(p, kl.KL_F32, 0, 64, 64, p, 64, p, p, ctypes.c_void_p(0)) == kl.KL_OK


def test_release_workspaces_with_none_allocated():
    """Nothing allocated yet (no GPU here): a no-op that succeeds, twice."""
    kl.release_workspaces()
    kl.release_workspaces()


@pytest.mark.parametrize("m, n, k, ab, c, want", [
    (16, 28672, 8192, "KL_BF16", "KL_BF16", "ALGO_SKINNY"),
    (64, 28672, 8192, "KL_BF16", "KL_BF16", "ALGO_SKINNY"),
    (128, 28672, 8192, "KL_BF16", "KL_BF16", "ALGO_1CTA"),
    (128, 28672, 8192, "KL_E4M3", "KL_BF16", "ALGO_SKINNY"),
    (8192, 8192, 8192, "KL_BF16", "KL_BF16", "ALGO_2CTA"),
    (16384, 16384, 8192, "KL_E4M3", "KL_BF16", "ALGO_2CTA"),
])
def test_resolve_algo_names_the_default_route(kl, m, n, k, ab, c, want):
    """kl_gemm_resolve_algo reports the kernel family KL_ALGO_AUTO runs, with no GPU and no launch."""
    import ctypes

    d = kl.GemmDesc(m=m, n=n, k=k, a=0x1000, lda=k, b=0x2000, ldb=k, c=0x3000, ldc=n, ab_type=getattr(kl, ab),
                    c_type=getattr(kl, c), alpha=1.0, algo=kl.ALGO_AUTO)
    out = ctypes.c_int32(-1)
    assert kl.lib().kl_gemm_resolve_algo(ctypes.byref(d), ctypes.byref(out)) == kl.KL_OK
    assert out.value == getattr(kl, want)
    d.algo = kl.ALGO_SKINNY
    assert kl.lib().kl_gemm_resolve_algo(ctypes.byref(d), ctypes.byref(out)) == kl.KL_OK
    assert out.value == kl.ALGO_SKINNY


def test_gather_multicast_argument_checks(kl):
    """kl_gemm_gather_multicast's checks that need no GPU: a null multicast address, C += result and
    batched problems are refused before anything is queued."""
    import ctypes

    d = kl.GemmDesc(m=512, n=1024, k=512, a=0x1000, lda=512, b=0x2000, ldb=512, c=0x3000, ldc=2048,
                    ab_type=kl.KL_BF16, c_type=kl.KL_BF16, alpha=1.0, algo=kl.ALGO_AUTO)
    assert kl.lib().kl_gemm_gather_multicast(ctypes.byref(d), None, None) == kl.KL_ERR_INVALID_ARGUMENT
    d.c_reduce = 1
    assert kl.lib().kl_gemm_gather_multicast(ctypes.byref(d), ctypes.c_void_p(0x4000), None) == kl.KL_ERR_NOT_SUPPORTED
    d.c_reduce, d.batch = 0, 2
    assert kl.lib().kl_gemm_gather_multicast(ctypes.byref(d), ctypes.c_void_p(0x4000), None) == kl.KL_ERR_NOT_SUPPORTED
    d.batch, d.m = 0, 0  # an empty shard: nothing to do
    assert kl.lib().kl_gemm_gather_multicast(ctypes.byref(d), ctypes.c_void_p(0x4000), None) == kl.KL_OK


def test_resolve_tile_reports_a_missing_device(kl):
    """kl_gemm_resolve_tile needs the device's SM count for the CTA pair's choice: with no GPU it
    returns KL_ERR_CUDA with a message instead of guessing; the skinny and one-CTA routes answer
    from the descriptor alone."""
    import ctypes

    tm, tn = ctypes.c_int32(-1), ctypes.c_int32(-1)
    d = kl.GemmDesc(m=16, n=28672, k=8192, a=0x1000, lda=8192, b=0x2000, ldb=8192, c=0x3000, ldc=28672,
                    ab_type=kl.KL_BF16, c_type=kl.KL_BF16, alpha=1.0, algo=kl.ALGO_AUTO)
    assert kl.lib().kl_gemm_resolve_tile(ctypes.byref(d), ctypes.byref(tm), ctypes.byref(tn)) == kl.KL_OK
    assert (tm.value, tn.value) == (0, 0)
    d.m = 128
    assert kl.lib().kl_gemm_resolve_tile(ctypes.byref(d), ctypes.byref(tm), ctypes.byref(tn)) == kl.KL_OK
    assert (tm.value, tn.value) == (128, 256)
    d.m = 8192
    d.n = d.ldc = 8192
    st = kl.lib().kl_gemm_resolve_tile(ctypes.byref(d), ctypes.byref(tm), ctypes.byref(tn))
    assert st == kl.KL_ERR_CUDA and b"no CUDA device" in kl.lib().kl_last_error()
