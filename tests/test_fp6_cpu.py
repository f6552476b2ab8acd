"""Packed fp6 (e3m2 / e2m3) on the CPU: the formats' value grids, the oracle's bit-stream decoder,
the numpy packing and rounding the GPU tests quantise with, the MX quantiser, the oracle's MX
product on fp6 inputs, and the descriptor fields the Python binding derives from byte tensors."""

import numpy as np
import pytest
import torch

import maia_b200 as kl
from maia_b200 import workloads as wl
from oracle import gemm as og

FP6 = ("e3m2", "e2m3")


def test_grids():
    e3m2, e2m3 = wl.FP6_GRID["e3m2"], wl.FP6_GRID["e2m3"]
    assert e3m2[-1] == 28.0 and e2m3[-1] == 7.5
    assert e3m2[1] == 2.0 ** -4 and e2m3[1] == 0.125  # smallest subnormals
    assert e3m2[0b01100] == 1.0 and e2m3[0b01000] == 1.0  # exponent = bias, mantissa 0
    for g in (e3m2, e2m3):
        assert np.all(np.diff(g) > 0) and len(g) == 32


@pytest.mark.parametrize("kind", FP6)
def test_oracle_decoder_matches_the_grid(kind):
    """The C oracle reads elements at bits [6i, 6i + 6) of a row; numpy's pack_fp6 writes them
    there. Both sides restate the format independently."""
    codes = np.arange(64, dtype=np.uint8).reshape(2, 32)
    want = np.where(codes & 32, -1.0, 1.0) * wl.FP6_GRID[kind][codes & 31]
    np.testing.assert_array_equal(og.decode(wl.pack_fp6(codes), kind), want)


def test_pack_layout_known_answer():
    # 1 | 2 << 6 | 3 << 12 | 4 << 18 = 0x103081: bytes 0x81, 0x30, 0x10 (least significant first).
    assert wl.pack_fp6(np.array([[1, 2, 3, 4]], dtype=np.uint8)).tolist() == [[0x81, 0x30, 0x10]]
    assert wl.pack_fp6(np.array([[63, 0, 0, 0, 0, 0, 0, 63]], dtype=np.uint8)).tolist() == [[63, 0, 0, 0, 0, 0xFC]]


def test_pack_unpack_round_trip():
    codes = np.random.default_rng(0).integers(0, 64, (7, 256), dtype=np.uint8)
    packed = wl.pack_fp6(codes)
    assert packed.shape == (7, 192)
    np.testing.assert_array_equal(wl.unpack_fp6(packed), codes)


@pytest.mark.parametrize("kind", FP6)
def test_rounding_is_nearest_even_and_saturating(kind):
    grid = wl.FP6_GRID[kind]
    x = np.concatenate([np.linspace(-40, 40, 20001), (grid[1:] + grid[:-1]) / 2, -(grid[1:] + grid[:-1]) / 2,
                        [1e9, -1e9, 0.0, -0.0]]).astype(np.float32)
    codes = wl.f32_to_fp6_codes(x, kind)
    got = np.where(codes & 32, -1.0, 1.0) * grid[codes & 31]
    a = np.minimum(np.abs(x.astype(np.float64)), grid[-1])
    dist = np.abs(grid[None, :] - a[:, None])
    best = dist.min(axis=1)
    assert np.array_equal(np.abs(np.abs(got) - a), best)  # always a nearest value
    tie = (dist == best[:, None]).sum(axis=1) > 1
    assert np.all((codes[tie] & 1) == 0)  # ties go to the even mantissa
    assert np.all(np.sign(got[np.abs(x) > grid[1]]) == np.sign(x[np.abs(x) > grid[1]]))


@pytest.mark.parametrize("kind", FP6)
def test_mx_quantize_fp6(kind):
    rng = np.random.default_rng(3)
    x = rng.standard_normal((5, 256)).astype(np.float32) * np.float32(3.0)
    q, s = wl.mx_quantize(x, kind)
    assert q.shape == (5, 192) and s.shape == (5, 8)
    amax = np.abs(x.reshape(5, 8, 32)).max(axis=2)
    np.testing.assert_array_equal(s.astype(int) - 127, np.floor(np.log2(amax)).astype(int) - wl.MX_EMAX[kind])
    deq = og.decode(q, kind) * og.e8m0_values(s).repeat(32, axis=1)
    # Elements land within half a step of their grid: relative error <= 2^-(mantissa bits + 1) of the
    # block's scale times the largest grid step, loosely bounded by amax * 2^-(mb).
    mb = 2 if kind == "e3m2" else 3
    err = np.abs(deq - x).reshape(5, 8, 32).max(axis=2)
    assert np.all(err <= amax * 2.0 ** -mb)


@pytest.mark.parametrize("kind", FP6)
def test_oracle_mx_product_on_fp6(kind):
    rng = np.random.default_rng(4)
    qa, sa = wl.mx_quantize(rng.standard_normal((9, 128)).astype(np.float32), kind)
    qb, sb = wl.mx_quantize(rng.standard_normal((6, 128)).astype(np.float32), kind)
    da = og.decode(qa, kind) * og.e8m0_values(sa).repeat(32, axis=1)
    db = og.decode(qb, kind) * og.e8m0_values(sb).repeat(32, axis=1)
    np.testing.assert_allclose(og.gemm_mx_f64(qa, qb, sa, sb, kind, threads=2), da @ db.T, rtol=1e-12, atol=1e-12)


def test_descriptor_fields_from_packed_bytes():
    a = torch.zeros(64, 288, dtype=torch.uint8)   # K = 384
    b = torch.zeros(2, 40, 288, dtype=torch.uint8)
    c = torch.zeros(64, 40, dtype=torch.bfloat16)
    d = kl.gemm_desc(a, b[0], c, ab_type="e2m3")
    assert (d.k, d.lda, d.ldb, d.ab_type) == (384, 384, 384, kl.KL_E2M3)
    d = kl.gemm_desc(a, b[1], c, ab_type=kl.KL_E3M2)
    assert d.ab_type == kl.KL_E3M2
    with pytest.raises(ValueError):  # 3 K / 4 bytes: whole groups of 3
        kl.gemm_desc(torch.zeros(64, 100, dtype=torch.uint8), torch.zeros(40, 100, dtype=torch.uint8), c, ab_type="e3m2")
    with pytest.raises(ValueError):  # fp6 travels as uint8
        kl.gemm_desc(a.view(torch.float8_e4m3fn), b[0].view(torch.float8_e4m3fn), c, ab_type="e3m2")
    with pytest.raises(ValueError):
        kl.gemm_desc(a, b[0], c, ab_type=kl.KL_E4M3)
    with pytest.raises(ValueError):
        kl.gemm_desc(a, b[0], c, ab_type="e5m3")
    with pytest.raises(ValueError):
        kl.mx_quantize(torch.zeros(4, 128), "e3m3")


def test_instr_desc_fp6_formats():
    """kind::f8f6f4 operand formats: e2m3 = 3, e3m2 = 4 (bits 7-9 for A, 10-12 for B)."""
    v = kl.mma_instr_desc(kl.KL_E3M2, kl.KL_E2M3, kl.KL_F32, 128, 256)
    assert (v >> 7) & 7 == 4 and (v >> 10) & 7 == 3


@pytest.mark.parametrize("eb,mb", [(2, 1), (3, 2), (2, 3)], ids=["e2m1", "e3m2", "e2m3"])
def test_minifloat_rounding_matches_a_grid_search(eb, mb):
    """workloads.minifloat_codes (binade scaling and rint) against the definition: the nearest value
    of the sorted grid, ties to the even code, saturating; zeros, subnormals, exact ties and the
    values one ulp either side of every tie included."""
    bias = (1 << (eb - 1)) - 1
    codes = np.arange(1 << (eb + mb))
    e, m = codes >> mb, codes & ((1 << mb) - 1)
    grid = np.where(e == 0, m * 2.0 ** (1 - bias - mb), (m + (1 << mb)) * 2.0 ** (e - bias - mb))
    mids = (grid[1:] + grid[:-1]) / 2
    rng = np.random.default_rng(eb * 10 + mb)
    x = np.concatenate([rng.standard_normal(200_000) * s for s in (0.01, 0.3, 2.0, 30.0)] +
                       [mids, -mids, grid, -grid, np.nextafter(mids, 0), np.nextafter(mids, 1e9),
                        [0.0, -0.0, 1e30, -1e30, 1e-30, -1e-30]]).astype(np.float32)
    a = np.minimum(np.abs(x.astype(np.float64)), grid[-1])
    idx = np.clip(np.searchsorted(grid, a), 1, len(grid) - 1)
    lo, hi = grid[idx - 1], grid[idx]
    pick_hi = (a - lo > hi - a) | ((a - lo == hi - a) & (idx % 2 == 0))
    q = np.where(pick_hi, idx, idx - 1)
    want = np.where(np.signbit(x) & (q != 0), q | (1 << (eb + mb)), q)
    np.testing.assert_array_equal(wl.minifloat_codes(x, eb, mb), want)
