"""Descriptors on the GPU, bit for bit against the reference's own code compiled here
(oracle/_ref/libkl_ref.so: kernel_lib/include/kl + CuTe 4.5.0):
  * UMMA smem descriptors computed on the device at a real shared address
    (kernel_lib/tests/unit/test_umma_desc.cu:116-172), ours vs the reference's kl::umma_desc vs
    CuTe's iterator;
  * 128-byte TMA tensor maps (kernel_lib/tests/unit/test_tma_desc.cu:41-95), ours (the C ABI)
    vs the reference's kl::make_tma_load vs CuTe's make_tma_copy;
  * the error messages of invalid layouts (test_tma_desc.cu:97-118).
"""

import ctypes
from pathlib import Path

import pytest

import maia_b200 as kl

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
REF_LIB = ROOT / "oracle" / "_ref" / "libkl_ref.so"
PROBE_LIB = ROOT / "tests" / "native" / "libkl_testprobe.so"

# case -> (elem_bytes, rows, cols, swizzle, block_rows); numbering shared with the probes.
DESC_CASES = {
    0: (2, 128, 64, 128, 128), 1: (2, 256, 64, 128, 256), 2: (2, 128, 128, 128, 128), 3: (2, 128, 64, 64, 128),
    4: (2, 128, 32, 32, 128), 5: (1, 128, 128, 128, 128), 6: (1, 128, 128, 128, 128), 7: (4, 128, 32, 128, 128),
    8: (2, 256, 64, 128, 128), 9: (2, 512, 64, 128, 256), 10: (2, 128, 128, 128, 64), 11: (2, 256, 64, 64, 128),
    12: (1, 256, 128, 128, 128), 13: (1, 256, 128, 128, 128),
}
# case -> (dtype, tile_rows, tile_cols, swizzle, gmem rows, gmem cols)
TMA_CASES = {
    0: (kl.KL_BF16, 128, 64, 128, 4096, 4096), 1: (kl.KL_BF16, 256, 64, 128, 8192, 4096),
    2: (kl.KL_I8, 128, 128, 128, 4096, 4096), 3: (kl.KL_BF16, 128, 128, 128, 4096, 4096),
    4: (kl.KL_BF16, 128, 32, 64, 4096, 8192), 5: (kl.KL_BF16, 128, 16, 32, 4096, 4096),
    6: (kl.KL_BF16, 128, 8, 16, 4096, 4096), 7: (kl.KL_BF16, 512, 64, 128, 4096, 4096),
    8: (kl.KL_E4M3, 128, 128, 128, 4096, 4096), 9: (kl.KL_F32, 32, 32, 128, 1000, 4096),
    10: (kl.KL_BF16, 32, 64, 128, 8192, 8192),
}


@pytest.fixture(scope="module")
def ref():
    assert REF_LIB.exists(), f"{REF_LIB} missing: build it with `make -C oracle` where the reference is present"
    L = ctypes.CDLL(str(REF_LIB))
    P = ctypes.POINTER
    L.kl_ref_umma_descs.argtypes = [ctypes.c_int, P(ctypes.c_uint64), P(ctypes.c_uint64), P(ctypes.c_uint32),
                                    P(ctypes.c_int)]
    L.kl_ref_tma_desc.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
                                  ctypes.c_void_p]
    L.kl_ref_tma_desc_batched.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                          ctypes.c_void_p, ctypes.c_void_p]
    L.kl_ref_tma_error.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_char_p,
                                   ctypes.c_int]
    L.kl_ref_tma_desc_rank.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_int64), ctypes.c_void_p,
                                       ctypes.c_void_p]
    return L


@pytest.fixture(scope="module")
def probe():
    assert PROBE_LIB.exists(), f"{PROBE_LIB} missing: run __graft_entry__.build()"
    L = ctypes.CDLL(str(PROBE_LIB))
    P = ctypes.POINTER
    L.kl_test_umma_descs.argtypes = [ctypes.c_int, P(ctypes.c_uint64), P(ctypes.c_uint32), P(ctypes.c_int)]
    return L


@pytest.mark.parametrize("case", sorted(DESC_CASES))
def test_device_umma_desc_matches_reference(cuda, ref, probe, case):
    n = 64
    ours, theirs, cute = (ctypes.c_uint64 * n)(), (ctypes.c_uint64 * n)(), (ctypes.c_uint64 * n)()
    b_ours, b_ref = ctypes.c_uint32(), ctypes.c_uint32()
    c_ours, c_ref = ctypes.c_int(), ctypes.c_int()
    assert probe.kl_test_umma_descs(case, ours, ctypes.byref(b_ours), ctypes.byref(c_ours)) == 0
    assert ref.kl_ref_umma_descs(case, theirs, cute, ctypes.byref(b_ref), ctypes.byref(c_ref)) == 0
    assert c_ours.value == c_ref.value > 0
    shift = (b_ours.value >> 4) - (b_ref.value >> 4)  # same tile offset in both kernels' smem
    for i in range(c_ref.value):
        assert theirs[i] == cute[i], f"reference vs CuTe differ at {i}"
        assert ours[i] - shift == theirs[i], f"descriptor {i}: ours {ours[i]:#x} reference {theirs[i]:#x}"
    # And the host encoder (C ABI) agrees with both at the device's actual address.
    eb, rows, cols, sw, br = DESC_CASES[case]
    nk = cols // (32 // eb)
    for i in range(c_ours.value):
        m, k = divmod(i, nk)
        assert kl.umma_smem_desc(eb, rows, cols, sw, b_ours.value, k, m * br) == ours[i]


@pytest.mark.parametrize("case", sorted(TMA_CASES))
def test_tensor_map_matches_reference(cuda, ref, case):
    import torch

    dt, tr, tc, sw, rows, cols = TMA_CASES[case]
    eb = {kl.KL_BF16: 2, kl.KL_I8: 1, kl.KL_E4M3: 1, kl.KL_F32: 4}[dt]
    buf = torch.empty(rows * cols * eb, dtype=torch.uint8, device=cuda)
    ours = kl.make_tma_desc(dt, tr, tc, sw, buf.data_ptr(), (rows, cols), (cols, 1))
    kl_map, cute_map = ctypes.create_string_buffer(128), ctypes.create_string_buffer(128)
    assert ref.kl_ref_tma_desc(case, ctypes.c_void_p(buf.data_ptr()), rows, cols, kl_map, cute_map) == 0
    assert ours == kl_map.raw, "tensor map differs from the reference's make_tma_load"
    if tr <= 256:
        assert ours == cute_map.raw, "tensor map differs from CuTe's make_tma_copy"


def test_tall_tile_map_equals_256_row_map(cuda):
    """kernel_lib/tests/unit/test_tma_desc.cu:86-95: a 512-row tile loads as 256-row boxes."""
    import torch

    buf = torch.empty(4096 * 4096, dtype=torch.bfloat16, device=cuda)
    tall = kl.make_tma_desc(kl.KL_BF16, 512, 64, 128, buf.data_ptr(), (4096, 4096), (4096, 1))
    one = kl.make_tma_desc(kl.KL_BF16, 256, 64, 128, buf.data_ptr(), (4096, 4096), (4096, 1))
    assert tall == one


def test_batched_rank3_map_matches_reference(cuda, ref):
    import torch

    B, M, K = 4, 1024, 512
    buf = torch.empty(B * M * K, dtype=torch.bfloat16, device=cuda)
    ours = kl.make_tma_desc(kl.KL_BF16, 128, 64, 128, buf.data_ptr(), (B, M, K), (M * K, K, 1))
    kl_map, cute_map = ctypes.create_string_buffer(128), ctypes.create_string_buffer(128)
    assert ref.kl_ref_tma_desc_batched(ctypes.c_void_p(buf.data_ptr()), B, M, K, kl_map, cute_map) == 0
    assert ours == kl_map.raw == cute_map.raw


@pytest.mark.parametrize("shape", [(3, 4, 512, 256), (2, 3, 4, 256, 512), (1, 1, 2, 128, 64)])
def test_rank4_rank5_maps_match_reference(cuda, ref, shape):
    """Outer modes beyond one batch mode (tma_desc.hpp allows rank 2..5): ours = the reference's
    make_tma_load(row_major(p, extents...)) = CuTe's make_tma_copy."""
    import torch

    n = 1
    for e in shape:
        n *= e
    buf = torch.empty(n, dtype=torch.bfloat16, device=cuda)
    strides, acc = [], 1
    for e in reversed(shape):
        strides.insert(0, acc)
        acc *= e
    ours = kl.make_tma_desc(kl.KL_BF16, 128, 64, 128, buf.data_ptr(), shape, strides)
    kl_map, cute_map = ctypes.create_string_buffer(128), ctypes.create_string_buffer(128)
    ext = (ctypes.c_int64 * len(shape))(*shape)
    assert ref.kl_ref_tma_desc_rank(ctypes.c_void_p(buf.data_ptr()), len(shape), ext, kl_map, cute_map) == 0
    assert ours == kl_map.raw, "tensor map differs from the reference's make_tma_load"
    assert ours == cute_map.raw, "tensor map differs from CuTe's make_tma_copy"


@pytest.mark.parametrize("offset, rows, cols, stride", [
    (1, 4096, 4096, 4096),      # misaligned base
    (0, 4096, 4096, 1024),      # row stride < cols
    (0, 4096, 4100, 4100),      # pitch not a multiple of 16 bytes
    (0, 0, 4096, 4096),         # empty extent
    (0, 4096, 4096, 4096 + 64), # padded rows: valid
])
def test_error_contract_matches_reference(cuda, ref, offset, rows, cols, stride):
    import torch

    buf = torch.empty(4096 * 4200 + 64, dtype=torch.bfloat16, device=cuda)
    ptr = buf.data_ptr() + 2 * offset
    msg = ctypes.create_string_buffer(512)
    ref_failed = ref.kl_ref_tma_error(ctypes.c_void_p(ptr), rows, cols, stride, msg, 512)
    try:
        kl.make_tma_desc(kl.KL_BF16, 128, 64, 128, ptr, (rows, cols), (stride, 1))
        ours = None
    except kl.KlError as e:
        ours = e.message
    if ref_failed:
        assert ours == msg.value.decode()
    else:
        assert ours is None
