"""The CPU GEMM oracle (oracle/gemm_oracle.c) pinned against numpy float64 matmul, and its element
decoders against the format definitions."""

import numpy as np
import pytest

from maia_b200 import workloads as wl
from oracle import gemm as og


def test_bf16_decode_and_rounding():
    x = np.array([0.0, 1.0, -2.5, 3.140625, 1e-3, 65504.0, 1.00390625, 1.01171875], dtype=np.float32)
    bits = wl.f32_to_bf16_bits(x)
    # 1 + 2^-8 ties to even (1.0); 1 + 3*2^-8 ties up to 1 + 2^-6.
    np.testing.assert_array_equal(og.decode(bits)[[0, 1, 2, 6, 7]], [0.0, 1.0, -2.5, 1.0, 1.015625])
    np.testing.assert_allclose(og.decode(bits), x, rtol=2 ** -8)


def test_e4m3_table():
    v = wl.e4m3_values()
    assert v[0x7E] == 448.0 and v[0x01] == 2.0 ** -9 and v[0x38] == 1.0 and np.isnan(v[0x7F]) and v[0xB8] == -1.0
    np.testing.assert_array_equal(og.decode(np.arange(256, dtype=np.uint8))[~np.isnan(v)], v[~np.isnan(v)])


def test_e4m3_fast_rounding_matches_nearest_search():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(200000).astype(np.float32) * s for s in (1e-3, 0.05, 1.0, 30.0, 200.0)])
    grid = wl.e4m3_values()[:0x7F].astype(np.float32)
    mids = ((grid[1:] + grid[:-1]) / 2).astype(np.float32)  # exact ties
    x = np.concatenate([x, grid, -grid, mids, -mids, np.array([447.9, 448.0, 460.0, 5e-4, 1e-9], np.float32)])
    np.testing.assert_array_equal(wl.f32_to_e4m3_bits(x), wl.f32_to_e4m3_bits_nearest(x))


def test_e4m3_quantise_round_trip():
    finite = np.array([i for i in range(256) if i not in (0x7F, 0xFF, 0x80)], dtype=np.uint8)
    vals = wl.e4m3_values()[finite]
    np.testing.assert_array_equal(wl.f32_to_e4m3_bits(vals.astype(np.float32)), finite)
    # Midpoint between 1.0 (0x38) and 1.125 (0x39) rounds to even mantissa -> 0x38; saturation at 448.
    assert wl.f32_to_e4m3_bits(np.array([1.0625, 1000.0, -1000.0], dtype=np.float32)).tolist() == [0x38, 0x7E, 0xFE]


@pytest.mark.parametrize("dtype", ["bf16", "e4m3"])
@pytest.mark.parametrize("shape", [(1, 1, 1), (7, 5, 3), (64, 48, 96), (130, 70, 257)])
def test_gemm_f64_matches_numpy(dtype, shape):
    from gpu_util import random_inputs

    m, n, k = shape
    a, b, sa, sb = random_inputs(m, n, k, dtype, seed=m + n + k)
    ref = og.decode(a) @ og.decode(b).T * (sa * sb)
    got = og.gemm_f64(a, b, sa * sb, threads=3)
    np.testing.assert_allclose(got, ref, rtol=1e-12, atol=1e-12)


def test_gemm_f32_baseline_close_to_f64():
    from gpu_util import random_inputs

    a, b, _, _ = random_inputs(100, 90, 300, "bf16", seed=3)
    ref = og.gemm_f64(a, b)
    got = og.gemm_f32(a, b, threads=4)
    elem, norm = og.rel_error(got, ref)
    assert norm < 1e-5


def test_c1_inputs_are_seeded_and_stable():
    a1, b1, _, _ = wl.make_inputs(wl.C1)
    a2, b2, _, _ = wl.make_inputs(wl.C1)
    assert a1.shape == (256, 256) and b1.shape == (256, 256) and a1.dtype == np.uint16
    np.testing.assert_array_equal(a1, a2)
    x = og.decode(a1)
    assert x.min() >= -1.0 and x.max() <= 1.0 and abs(x.mean()) < 0.02


def test_rel_error_floor():
    ref = np.array([1.0, -1.0, 0.0, 1e-9])
    elem, norm = og.rel_error(ref + np.array([1e-3, 0, 1e-6, 0]), ref)
    # rms(ref) = sqrt(1/2): the zero entry is measured against the floor 1e-2 * rms.
    elem, norm = og.rel_error(ref + np.array([1e-3, 0, 1e-5, 0]), ref)
    assert abs(elem - 1e-5 / (1e-2 * np.sqrt(0.5))) < 1e-9 and abs(norm - 1e-3) < 1e-12
    elem, _ = og.rel_error(ref + np.array([1e-3, 0, 1e-6, 0]), ref, floor_frac=1e-3)
    assert abs(elem - 1e-6 / (1e-3 * np.sqrt(0.5))) < 1e-9


def test_e5m2_table_and_decode():
    v = wl.e5m2_values()
    assert v[0x7B] == 57344.0 and v[0x01] == 2.0 ** -16 and v[0x3C] == 1.0 and v[0x7C] == np.inf
    assert np.isnan(v[0x7D]) and v[0xBC] == -1.0 and v[0xFC] == -np.inf
    got = og.decode(np.arange(256, dtype=np.uint8), "e5m2")
    same = (got == v) | (np.isnan(got) & np.isnan(v))
    assert same.all()


def test_e5m2_fast_rounding_matches_nearest_search():
    rng = np.random.default_rng(1)
    x = np.concatenate([rng.standard_normal(200000).astype(np.float32) * s for s in (1e-5, 1e-2, 1.0, 300.0, 3e4)])
    grid = wl.e5m2_values()[:0x7C].astype(np.float32)
    mids = ((grid[1:] + grid[:-1]) / 2).astype(np.float32)  # exact ties
    x = np.concatenate([x, grid, -grid, mids, -mids, np.array([57343.0, 57344.0, 61440.0, 1e6, 1e-9], np.float32)])
    np.testing.assert_array_equal(wl.f32_to_e5m2_bits(x), wl.f32_to_e5m2_bits_nearest(x))
    # 1 + 1/8 lies halfway between 1.0 (0x3C) and 1.25 (0x3D): ties to the even mantissa.
    assert wl.f32_to_e5m2_bits(np.array([1.125, 1.375, 1e6, -1e6], np.float32)).tolist() == [0x3C, 0x3E, 0x7B, 0xFB]


def test_f16_decode_matches_ieee_binary16():
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    want = bits.view(np.float16).astype(np.float64)
    got = og.decode(bits, "f16")
    assert ((got == want) | (np.isnan(got) & np.isnan(want))).all()
    # float16 arrays are recognised without a kind.
    np.testing.assert_array_equal(og.decode(np.array([1.5, -2.0], np.float16)), [1.5, -2.0])


@pytest.mark.parametrize("dtype", ["f16", "e5m2"])
def test_gemm_f64_other_formats(dtype):
    from gpu_util import random_inputs

    a, b, sa, sb = random_inputs(33, 17, 70, dtype, seed=5)
    ref = og.decode(a, dtype) @ og.decode(b, dtype).T * (sa * sb)
    np.testing.assert_allclose(og.gemm_f64(a, b, sa * sb, threads=2, kind=dtype), ref, rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(og.gemm_f32(a, b, sa * sb, threads=2, kind=dtype), ref, rtol=1e-4, atol=1e-4)


def test_kind_must_match_the_bits():
    with pytest.raises(TypeError):
        og.decode(np.zeros(4, np.uint8), "f16")


def test_mx_quantise_and_oracle():
    """MX quantisation keeps every block within the element format, and the MX oracle equals the
    plain fp64 product of the dequantised inputs."""
    rng = np.random.default_rng(4)
    x = rng.standard_normal((40, 200)).astype(np.float32) * np.float32(7.0)
    for kind, fmax in (("e4m3", 448.0), ("e5m2", 57344.0)):
        q, s = wl.mx_quantize(x, kind)
        assert s.shape == (40, 7)
        deq = og.decode(q, kind) * np.repeat(og.e8m0_values(s), 32, axis=1)[:, :200]
        assert np.abs(og.decode(q, kind)).max() <= fmax
        rel = np.abs(deq - x).max() / np.abs(x).max()
        assert rel < (2.0 ** -3 if kind == "e4m3" else 2.0 ** -2)
    qa, sa = wl.mx_quantize(x[:13], "e4m3")
    qb, sb = wl.mx_quantize(x[13:], "e4m3")
    da = og.decode(qa, "e4m3") * np.repeat(og.e8m0_values(sa), 32, axis=1)[:, :200]
    db = og.decode(qb, "e4m3") * np.repeat(og.e8m0_values(sb), 32, axis=1)[:, :200]
    np.testing.assert_allclose(og.gemm_mx_f64(qa, qb, sa, sb, "e4m3", 3.0), 3.0 * da @ db.T, rtol=1e-13)


def test_pack_mx_scales_layout():
    sf = np.arange(300 * 9, dtype=np.int64).reshape(300, 9).astype(np.uint8)
    k = 9 * 32 - 5
    pk = og.pack_mx_scales(sf, k)
    kb = -(-k // 128)
    assert pk.size == 3 * kb * 512
    for r in (0, 31, 32, 127, 128, 200, 299):
        for j in range(9):
            rb, rr = divmod(r, 128)
            kk, jj = divmod(j, 4)
            assert pk[(rb * kb + kk) * 512 + (rr % 32) * 16 + (rr // 32) * 4 + jj] == sf[r, j]
    assert pk[(2 * kb + 2) * 512 + 1 * 16 + 3 * 4 + 1] == 127  # row 2*128+97 >= 300: padding


def test_e2m1_rounding_packing_and_decode():
    grid = wl.E2M1_GRID
    # Every code decodes to its value; ties go to the even code (mantissa 0); saturation at 6.
    codes = np.arange(16, dtype=np.uint8)
    vals = np.where(codes & 8, -1.0, 1.0) * grid[codes & 7]
    got = og.decode(wl.pack_e2m1(codes.reshape(1, 16)), "e2m1")[0]
    np.testing.assert_array_equal(got, vals)
    x = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 7.0, -5.0, 100.0], np.float32)
    assert wl.f32_to_e2m1_codes(x).tolist() == [0, 2, 2, 4, 4, 6, 6, 7, 14, 7]
    # Packing: the first element in the low nibble.
    assert wl.pack_e2m1(np.array([[1, 2, 15, 0]], np.uint8)).tolist() == [[0x21, 0x0F]]
    # Random values: the chosen code is a nearest grid point of the clipped value.
    rng = np.random.default_rng(2)
    y = np.clip(rng.standard_normal(5000).astype(np.float32) * 3, -6, 6)
    c = wl.f32_to_e2m1_codes(y)
    err = np.abs(np.where(c & 8, -1.0, 1.0) * grid[c & 7] - y)
    nearest = np.abs(np.abs(y)[:, None] - grid[None, :]).min(axis=1)
    np.testing.assert_allclose(err, nearest, atol=1e-7)


def test_gemm_mx_f64_packed_fp4():
    rng = np.random.default_rng(6)
    qa, sa = wl.mx_quantize(rng.standard_normal((17, 96)).astype(np.float32), "e2m1")
    qb, sb = wl.mx_quantize(rng.standard_normal((11, 96)).astype(np.float32), "e2m1")
    assert qa.shape == (17, 48) and sa.shape == (17, 3)
    da = og.decode(qa, "e2m1") * np.repeat(og.e8m0_values(sa), 32, axis=1)
    db = og.decode(qb, "e2m1") * np.repeat(og.e8m0_values(sb), 32, axis=1)
    np.testing.assert_allclose(og.gemm_mx_f64(qa, qb, sa, sb, "e2m1"), da @ db.T, rtol=1e-13, atol=1e-13)
    np.testing.assert_allclose(og.gemm_mx_f32(qa, qb, sa, sb, "e2m1"), da @ db.T, rtol=1e-5, atol=1e-5)
