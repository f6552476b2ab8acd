"""MXFP8 (block-scaled e4m3 / e5m2) on the GPU against the fp64 oracle, and the scale repacking
kernel against the oracle's restatement of the blocked layout.

Inputs are MX-quantised (OCP MX v1.0: a UE8M0 scale per 32 K-elements, elements rounded to the
8-bit format), so the oracle multiplies exactly the values the GPU sees; the tolerance (5e-2, as
for every fp8 input) only has to cover fp32 accumulation and the rounding of C.
"""

import numpy as np
import pytest
import torch

import maia_b200 as kl
from maia_b200 import workloads as wl
from oracle import gemm as og

from gpu_util import TORCH_TYPES, to_device

pytestmark = pytest.mark.gpu

FP8_TOL = 5e-2


def mx_inputs(m, n, k, kind, seed, spread=0.0):
    """MX-quantised A, B; `spread` widens the per-block magnitudes by up to 2^spread."""
    rng = np.random.Generator(np.random.PCG64(seed))
    xa = rng.standard_normal((m, k), dtype=np.float32)
    xb = rng.standard_normal((n, k), dtype=np.float32)
    if spread:
        xa *= np.exp2(rng.uniform(-spread, spread, (m, -(-k // 32)))).repeat(32, axis=1)[:, :k].astype(np.float32)
        xb *= np.exp2(rng.uniform(-spread, spread, (n, -(-k // 32)))).repeat(32, axis=1)[:, :k].astype(np.float32)
    qa, sa = wl.mx_quantize(xa, kind)
    qb, sb = wl.mx_quantize(xb, kind)
    return qa, sa, qb, sb


FP6 = ("e3m2", "e2m3")


def run_mx(qa, sa, qb, sb, kind, out, device, **kw):
    k = og.elements(kind, qa.shape[1])
    a, b = to_device(qa, kind, device), to_device(qb, kind, device)
    if kind in FP6:
        kw.setdefault("ab_type", kind)
    psa = kl.mx_pack_scales(torch.from_numpy(sa).to(device), k)
    psb = kl.mx_pack_scales(torch.from_numpy(sb).to(device), k)
    c = kw.pop("c", None)
    if c is None:
        c = torch.full((qa.shape[0], qb.shape[0]), float("nan"), dtype=TORCH_TYPES[out], device=device)
    kl.gemm(a, b, c, sfa=psa, sfb=psb, **kw)
    torch.cuda.synchronize()
    assert kl.read_status() == 0, "a device-side wait timed out"
    return c.float().cpu().numpy()


def check_mx(c, qa, sa, qb, sb, kind, tol=FP8_TOL, c0=None, scale=1.0):
    ref = og.gemm_mx_f64(qa, qb, sa, sb, kind, scale)
    if c0 is not None:
        ref = ref + c0
    assert not np.isnan(c).any(), "output has unwritten (NaN) entries"
    elem, norm = og.rel_error(c, ref)
    assert norm <= tol and elem <= tol, f"normwise {norm:.3e}, element-wise {elem:.3e} > {tol}"


@pytest.mark.parametrize("rows,k", [(1, 1), (128, 128), (200, 300), (129, 1000), (1024, 4096), (300, 32)])
def test_pack_scales_matches_the_blocked_layout(cuda, rows, k):
    rng = np.random.default_rng(rows + k)
    sf = rng.integers(0, 255, (rows, -(-k // 32)), dtype=np.uint8)
    got = kl.mx_pack_scales(torch.from_numpy(sf).to(cuda), k).cpu().numpy()
    assert got.size == kl.mx_scale_bytes(rows, k)
    np.testing.assert_array_equal(got, og.pack_mx_scales(sf, k))


def test_pack_scales_strided_source(cuda):
    sf = np.random.default_rng(3).integers(100, 150, (256, 40), dtype=np.uint8)
    src = torch.from_numpy(sf).to(cuda)[:, :32]  # row pitch 40, 32 groups = K 1024
    got = kl.mx_pack_scales(src, 1024).cpu().numpy()
    np.testing.assert_array_equal(got, og.pack_mx_scales(sf[:, :32], 1024))


KERNELS = pytest.mark.parametrize("algo,variant", [(kl.ALGO_1CTA, 0), (kl.ALGO_1CTA, 2), (kl.ALGO_2CTA, 0),
                                                   (kl.ALGO_2CTA, 2), (kl.ALGO_2CTA, 3)],
                                  ids=["1cta_n256", "1cta_n128", "2cta_n256", "2cta_n128", "2cta_n192"])


@KERNELS
@pytest.mark.parametrize("kind,out", [("e4m3", "bf16"), ("e4m3", "f32"), ("e5m2", "bf16"), ("e5m2", "f32")])
@pytest.mark.parametrize("shape", [(128, 256, 128), (200, 304, 320), (256, 512, 1024), (1000, 1000, 1008)])
def test_mx_gemm(cuda, algo, variant, kind, out, shape):
    m, n, k = shape
    qa, sa, qb, sb = mx_inputs(m, n, k, kind, seed=m + n + k)
    c = run_mx(qa, sa, qb, sb, kind, out, cuda, algo=algo, variant=variant)
    check_mx(c, qa, sa, qb, sb, kind)


@KERNELS
@pytest.mark.parametrize("out", ["bf16", "f32"])
@pytest.mark.parametrize("shape", [(128, 256, 256), (200, 304, 320), (256, 512, 1024), (1000, 1000, 1024),
                                   (130, 264, 96)])
def test_mxfp4_gemm(cuda, algo, variant, out, shape):
    """Packed fp4 (e2m1, two per byte) with UE8M0 scales per 32 elements: kind::mxf4, 64 K-elements
    and two scale bytes per MMA, two scale atoms along K per stage."""
    m, n, k = shape
    qa, sa, qb, sb = mx_inputs(m, n, k, "e2m1", seed=3 * m + n + k)
    c = run_mx(qa, sa, qb, sb, "e2m1", out, cuda, algo=algo, variant=variant)
    check_mx(c, qa, sa, qb, sb, "e2m1")


def test_mxfp4_wide_scale_range(cuda):
    qa, sa, qb, sb = mx_inputs(384, 512, 768, "e2m1", seed=6, spread=10.0)
    c = run_mx(qa, sa, qb, sb, "e2m1", "f32", cuda, algo=kl.ALGO_2CTA)
    check_mx(c, qa, sa, qb, sb, "e2m1")


@KERNELS
@pytest.mark.parametrize("kind", FP6)
@pytest.mark.parametrize("out", ["bf16", "f32"])
@pytest.mark.parametrize("shape", [(128, 256, 128), (200, 304, 384), (1000, 1000, 1024)])
def test_mxfp6_gemm(cuda, algo, variant, kind, out, shape):
    """Packed fp6 (four elements per three bytes) read through TMA's 16U6 type, which gives every 16
    elements a 16-byte shared-memory slot, into kind::mxf8f6f4 MMAs with UE8M0 scales per 32."""
    m, n, k = shape
    qa, sa, qb, sb = mx_inputs(m, n, k, kind, seed=5 * m + n + k)
    c = run_mx(qa, sa, qb, sb, kind, out, cuda, algo=algo, variant=variant)
    check_mx(c, qa, sa, qb, sb, kind)


@pytest.mark.parametrize("kind", FP6)
@pytest.mark.parametrize("algo", [kl.ALGO_1CTA, kl.ALGO_2CTA], ids=["1cta", "2cta"])
def test_mxfp6_equals_mxfp8_on_the_same_values(cuda, kind, algo):
    """Every e3m2 and e2m3 value is an e4m3 value: the fp6 kernel and the MXFP8 kernel, given the
    same values and scales, run the same MMA kind in the same order and agree bit for bit."""
    qa, sa, qb, sb = mx_inputs(384, 512, 768, kind, seed=11)
    c6 = run_mx(qa, sa, qb, sb, kind, "f32", cuda, algo=algo)
    to8 = lambda q: wl.f32_to_e4m3_bits(og.decode(q, kind).astype(np.float32))
    assert np.array_equal(og.decode(to8(qa), "e4m3"), og.decode(qa, kind))
    c8 = run_mx(to8(qa), sa, to8(qb), sb, "e4m3", "f32", cuda, algo=algo)
    assert np.array_equal(c6, c8)


@pytest.mark.parametrize("kind", FP6)
def test_mxfp6_wide_scale_range(cuda, kind):
    qa, sa, qb, sb = mx_inputs(384, 512, 768, kind, seed=7, spread=10.0)
    c = run_mx(qa, sa, qb, sb, kind, "f32", cuda, algo=kl.ALGO_2CTA, variant=3)
    check_mx(c, qa, sa, qb, sb, kind)


def test_mxfp6_decode_kernels_agree(cuda):
    """16 rows of fp6 on the skinny kernel (the KL_ALGO_AUTO choice) and on the one-CTA tile kernel:
    both within tolerance of the oracle; the skinny kernel writes bf16 C only."""
    qa, sa, qb, sb = mx_inputs(16, 1024, 512, "e3m2", seed=8)
    for algo in (kl.ALGO_AUTO, kl.ALGO_SKINNY, kl.ALGO_1CTA):
        check_mx(run_mx(qa, sa, qb, sb, "e3m2", "bf16", cuda, algo=algo), qa, sa, qb, sb, "e3m2")
    with pytest.raises(kl.KlError) as e:
        run_mx(qa, sa, qb, sb, "e3m2", "f32", cuda, algo=kl.ALGO_SKINNY)
    assert e.value.status == kl.KL_ERR_NOT_SUPPORTED


def test_mxfp6_limits(cuda):
    """The 16U6 tensor maps' rules, checked on the host before any launch: K, pitches and strides
    in whole 128-element (96-byte) blocks, A and B 32-byte aligned."""
    c = torch.zeros(128, 128, dtype=torch.bfloat16, device=cuda)
    sf = torch.full((kl.block_scale_bytes(128, 256),), 127, dtype=torch.uint8, device=cuda)
    a = torch.zeros(128, 120, dtype=torch.uint8, device=cuda)  # K = 160
    with pytest.raises(kl.KlError) as e:
        kl.gemm(a, a, c, sfa=sf, sfb=sf, ab_type="e3m2", algo=kl.ALGO_1CTA)
    assert e.value.status == kl.KL_ERR_INVALID_ARGUMENT
    buf = torch.zeros(128 * 96 + 64, dtype=torch.uint8, device=cuda)
    assert buf.data_ptr() % 32 == 0
    shifted = buf[16:16 + 128 * 96].view(128, 96)  # 16-byte but not 32-byte aligned
    with pytest.raises(kl.KlError) as e:
        kl.gemm(shifted, buf[:128 * 96].view(128, 96), c, sfa=sf, sfb=sf, ab_type="e2m3", algo=kl.ALGO_2CTA)
    assert e.value.status == kl.KL_ERR_INVALID_ARGUMENT
    with pytest.raises(ValueError):
        kl.gemm(torch.zeros(128, 95, dtype=torch.uint8, device=cuda), a, c, sfa=sf, sfb=sf, ab_type="e3m2")
    with pytest.raises(kl.KlError) as e:  # fp6 is MX-only
        kl.gemm(buf[:128 * 96].view(128, 96), buf[:128 * 96].view(128, 96), c, sfa=sf, sfb=sf, scale_vec=16,
                ab_type="e3m2")
    assert e.value.status == kl.KL_ERR_NOT_SUPPORTED
    torch.cuda.synchronize()
    assert kl.read_status() == 0


@KERNELS
def test_mx_wide_scale_range(cuda, algo, variant):
    """Block magnitudes spread over 2^-12 .. 2^12: every scale byte matters."""
    qa, sa, qb, sb = mx_inputs(384, 512, 768, "e4m3", seed=5, spread=12.0)
    assert sa.max() - sa.min() > 16 and sb.max() - sb.min() > 16
    c = run_mx(qa, sa, qb, sb, "e4m3", "f32", cuda, algo=algo, variant=variant)
    check_mx(c, qa, sa, qb, sb, "e4m3")


@pytest.mark.parametrize("algo", [kl.ALGO_1CTA, kl.ALGO_2CTA], ids=["1cta", "2cta"])
def test_mx_persistent_many_tiles(cuda, algo):
    """More tiles than resident CTAs: each CTA walks several tiles through its accumulators."""
    qa, sa, qb, sb = mx_inputs(2048, 4096, 512, "e4m3", seed=31)
    c = run_mx(qa, sa, qb, sb, "e4m3", "bf16", cuda, algo=algo, max_ctas=16)
    check_mx(c, qa, sa, qb, sb, "e4m3")


@pytest.mark.parametrize("algo", [kl.ALGO_1CTA, kl.ALGO_2CTA], ids=["1cta", "2cta"])
def test_mx_each_scale_is_applied_to_its_own_block(cuda, algo):
    """Unit scales except one K-group of one row of A and one of B: only the matching outputs move."""
    m, n, k = 256, 256, 512
    rng = np.random.default_rng(8)
    qa = wl.f32_to_e4m3_bits(rng.standard_normal((m, k)).astype(np.float32))
    qb = wl.f32_to_e4m3_bits(rng.standard_normal((n, k)).astype(np.float32))
    sa = np.full((m, k // 32), 127, np.uint8)
    sb = np.full((n, k // 32), 127, np.uint8)
    sa[77, 9] = 131   # x16 on A row 77, K [288, 320)
    sb[200, 3] = 124  # /8 on B row 200, K [96, 128)
    c = run_mx(qa, sa, qb, sb, "e4m3", "f32", cuda, algo=algo)
    check_mx(c, qa, sa, qb, sb, "e4m3")


def test_mx_with_tensor_scales_and_reduce(cuda):
    m, n, k = 256, 256, 512
    qa, sa, qb, sb = mx_inputs(m, n, k, "e4m3", seed=12)
    c0 = np.random.default_rng(13).standard_normal((m, n)).astype(np.float32)
    c = torch.from_numpy(c0).to(cuda)
    two = torch.tensor([2.0], device=cuda)
    half = torch.tensor([0.25], device=cuda)
    got = run_mx(qa, sa, qb, sb, "e4m3", "f32", cuda, c=c, scale_a=two, scale_b=half, accumulate=True)
    check_mx(got, qa, sa, qb, sb, "e4m3", c0=c0, scale=0.5)


def test_mx_limits(cuda):
    a = torch.zeros(256, 128, dtype=torch.float8_e4m3fn, device=cuda)
    c = torch.zeros(256, 256, dtype=torch.bfloat16, device=cuda)
    s = torch.full((kl.mx_scale_bytes(256, 128),), 127, dtype=torch.uint8, device=cuda)
    with pytest.raises(kl.KlError) as e:  # the block-scaled skinny kernel takes at most 128 rows
        kl.gemm(a, a, c, sfa=s, sfb=s, algo=kl.ALGO_SKINNY)
    assert e.value.status == kl.KL_ERR_INVALID_ARGUMENT
    with pytest.raises(kl.KlError) as e:
        kl.gemm(a, a, c, sfa=s, algo=kl.ALGO_1CTA)  # no scales for B
    assert e.value.status == kl.KL_ERR_INVALID_ARGUMENT
    ab = torch.zeros(256, 128, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(kl.KlError) as e:
        kl.gemm(ab, ab, c, sfa=s, sfb=s)
    assert e.value.status == kl.KL_ERR_NOT_SUPPORTED


@pytest.mark.parametrize("rows,k", [(1, 16), (128, 64), (200, 320), (129, 1000)])
def test_pack_scales_nvfp4_layout(cuda, rows, k):
    rng = np.random.default_rng(rows + 3 * k)
    sf = rng.integers(0, 127, (rows, -(-k // 16)), dtype=np.uint8)
    got = kl.pack_block_scales(torch.from_numpy(sf).to(cuda), k, 16).cpu().numpy()
    assert got.size == kl.block_scale_bytes(rows, k, 16)
    np.testing.assert_array_equal(got, og.pack_mx_scales(sf, k, 16))


def run_nv(m, n, k, out, device, seed, **kw):
    rng = np.random.Generator(np.random.PCG64(seed))
    qa, sa, ga = wl.nv_quantize(rng.standard_normal((m, k), dtype=np.float32))
    qb, sb, gb = wl.nv_quantize(rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.1))
    a, b = to_device(qa, "e2m1", device), to_device(qb, "e2m1", device)
    psa = kl.pack_block_scales(torch.from_numpy(sa).to(device), k, 16)
    psb = kl.pack_block_scales(torch.from_numpy(sb).to(device), k, 16)
    c = torch.full((m, n), float("nan"), dtype=TORCH_TYPES[out], device=device)
    dga = torch.tensor([ga], dtype=torch.float32, device=device)
    dgb = torch.tensor([gb], dtype=torch.float32, device=device)
    kl.gemm(a, b, c, sfa=psa, sfb=psb, scale_vec=16, scale_a=dga, scale_b=dgb, **kw)
    torch.cuda.synchronize()
    assert kl.read_status() == 0, "a device-side wait timed out"
    ref = og.gemm_nv_f64(qa, qb, sa, sb, ga * gb)
    return c.float().cpu().numpy(), ref


@KERNELS
@pytest.mark.parametrize("out", ["bf16", "f32"])
@pytest.mark.parametrize("shape", [(128, 256, 256), (200, 304, 320), (256, 512, 1024), (1000, 1000, 1024),
                                   (130, 264, 96)])
def test_nvfp4_gemm(cuda, algo, variant, out, shape):
    """NVFP4: packed e2m1 with UE4M3 scales per 16 elements and per-tensor fp32 scales
    (kind::mxf4nvf4.block16: four scale atoms along K per stage, a whole scale word per MMA)."""
    m, n, k = shape
    c, ref = run_nv(m, n, k, out, cuda, seed=m + 7 * n + k, algo=algo, variant=variant)
    assert not np.isnan(c).any()
    elem, norm = og.rel_error(c, ref)
    assert norm <= FP8_TOL and elem <= FP8_TOL, f"normwise {norm:.3e}, element-wise {elem:.3e}"


@pytest.mark.parametrize("algo", [kl.ALGO_1CTA, kl.ALGO_2CTA], ids=["1cta", "2cta"])
def test_mx_reduce_into_bf16_c(cuda, algo):
    """Block-scaled GEMM adding into a bf16 C (the one-accumulator, eight-warp epilogue path)."""
    m, n, k = 384, 520, 512
    qa, sa, qb, sb = mx_inputs(m, n, k, "e4m3", seed=19)
    c0 = torch.randn(m, n, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16)
    c = c0.to(cuda)
    got = run_mx(qa, sa, qb, sb, "e4m3", "bf16", cuda, c=c, algo=algo, accumulate=True)
    check_mx(got, qa, sa, qb, sb, "e4m3", c0=c0.float().numpy().astype(np.float64))


@pytest.mark.parametrize("kind,vec", [("e4m3", 32), ("e2m1", 32), ("e2m1", 16), ("e3m2", 32), ("e2m3", 32)],
                         ids=["mxfp8", "mxfp4", "nvfp4", "mxfp6_e3m2", "mxfp6_e2m3"])
@pytest.mark.parametrize("m", [1, 16, 40, 64, 128])
def test_block_scaled_decode_skinny(cuda, kind, vec, m):
    """Decode shapes on the stream-K skinny kernel with block scales (weights' scales on the MMA's A
    side, the tokens' on its B side); K split across CTAs for the 3200-row weight matrix."""
    n, k = 3200, 2048
    rng = np.random.default_rng(m + vec)
    xa = rng.standard_normal((m, k)).astype(np.float32)
    xb = (rng.standard_normal((n, k)) * 0.05).astype(np.float32)
    if vec == 16:
        qa, sa, ga = wl.nv_quantize(xa)
        qb, sb, gb = wl.nv_quantize(xb)
        ref = og.gemm_nv_f64(qa, qb, sa, sb, ga * gb)
        scales = dict(scale_a=torch.tensor([ga], device=cuda), scale_b=torch.tensor([gb], device=cuda))
    else:
        qa, sa = wl.mx_quantize(xa, kind)
        qb, sb = wl.mx_quantize(xb, kind)
        ref = og.gemm_mx_f64(qa, qb, sa, sb, kind)
        scales = {}
    psa = kl.pack_block_scales(torch.from_numpy(sa).to(cuda), k, vec)
    psb = kl.pack_block_scales(torch.from_numpy(sb).to(cuda), k, vec)
    a, b = to_device(qa, kind, cuda), to_device(qb, kind, cuda)
    for algo in (kl.ALGO_SKINNY, kl.ALGO_AUTO):
        c = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=cuda)
        kl.gemm(a, b, c, sfa=psa, sfb=psb, scale_vec=vec, algo=algo, ab_type=kind if kind in FP6 else None, **scales)
        torch.cuda.synchronize()
        assert kl.read_status() == 0
        got = c.float().cpu().numpy()
        assert not np.isnan(got).any()
        elem, norm = og.rel_error(got, ref)
        assert elem <= FP8_TOL and norm <= FP8_TOL, f"algo {algo}: {elem:.3e} / {norm:.3e}"


@pytest.mark.parametrize("kind", ["e4m3", "e2m1", "e3m2", "e2m3"])
@pytest.mark.parametrize("src", ["f32", "bf16"])
@pytest.mark.parametrize("rows,k", [(1, 32), (200, 320), (129, 1024)])
def test_device_mx_quantize_matches_reference(cuda, kind, src, rows, k):
    """kl_mx_quantize = the OCP MX quantisation restated in maia_b200.workloads.mx_quantize: the same
    scales bit for bit, the same element values (compared as values: the device may encode a
    negative value that rounds to zero as -0). Packed fp6 rows are whole 128-element blocks."""
    if kind in FP6:
        k = -(-k // 128) * 128
    rng = np.random.default_rng(rows + k)
    x = (rng.standard_normal((rows, k)) * np.exp2(rng.uniform(-8, 8, (rows, 1)))).astype(np.float32)
    if src == "bf16":
        x = wl.bf16_bits_to_f32(wl.f32_to_bf16_bits(x))
    xt = torch.from_numpy(x).to(cuda)
    if src == "bf16":
        xt = xt.to(torch.bfloat16)
    q, sc = kl.mx_quantize(xt, kind)
    torch.cuda.synchronize()
    want_q, want_s = wl.mx_quantize(x, kind)
    np.testing.assert_array_equal(sc.cpu().numpy(), og.pack_mx_scales(want_s, k))
    got_v = og.decode(q.view(torch.uint8).cpu().numpy(), kind)
    np.testing.assert_array_equal(got_v, og.decode(want_q, kind))


@pytest.mark.parametrize("kind", ["e4m3", "e2m1", "e3m2", "e2m3"])
def test_device_quantize_then_gemm(cuda, kind):
    """Activations and weights quantised on the device feed the block-scaled GEMM directly."""
    rng = np.random.default_rng(9)
    xa = rng.standard_normal((256, 512)).astype(np.float32)
    xb = rng.standard_normal((384, 512)).astype(np.float32)
    qa, sa = kl.mx_quantize(torch.from_numpy(xa).to(cuda), kind)
    qb, sb = kl.mx_quantize(torch.from_numpy(xb).to(cuda), kind)
    c = kl.gemm(qa, qb, sfa=sa, sfb=sb, out_dtype=torch.float32, ab_type=kind if kind in FP6 else None)
    torch.cuda.synchronize()
    assert kl.read_status() == 0
    ra, rsa = wl.mx_quantize(xa, kind)
    rb, rsb = wl.mx_quantize(xb, kind)
    ref = og.gemm_mx_f64(ra, rb, rsa, rsb, kind)
    elem, norm = og.rel_error(c.cpu().numpy(), ref)
    assert elem <= FP8_TOL and norm <= FP8_TOL


@pytest.mark.parametrize("src", ["f32", "bf16"])
@pytest.mark.parametrize("rows,k", [(1, 16), (200, 336), (129, 1024)])
def test_device_nv_quantize_matches_reference(cuda, src, rows, k):
    """kl_nv_quantize = the NVFP4 quantisation restated in maia_b200.workloads.nv_quantize: the same
    per-tensor scale (to fp32), the same UE4M3 block scales bit for bit, the same element values."""
    rng = np.random.default_rng(rows + 3 * k)
    x = (rng.standard_normal((rows, k)) * np.exp2(rng.uniform(-6, 6, (rows, 1)))).astype(np.float32)
    if src == "bf16":
        x = wl.bf16_bits_to_f32(wl.f32_to_bf16_bits(x))
    xt = torch.from_numpy(x).to(cuda)
    if src == "bf16":
        xt = xt.to(torch.bfloat16)
    q, sc, g = kl.nv_quantize(xt)
    torch.cuda.synchronize()
    want_q, want_s, want_g = wl.nv_quantize(x)
    assert g.item() == np.float32(want_g)
    np.testing.assert_array_equal(sc.cpu().numpy(), og.pack_mx_scales(want_s, k, 16))
    got_v = og.decode(q.view(torch.uint8).cpu().numpy(), "e2m1")
    np.testing.assert_array_equal(got_v, og.decode(want_q, "e2m1"))


def test_device_nv_quantize_then_gemm(cuda):
    rng = np.random.default_rng(12)
    xa = rng.standard_normal((256, 512)).astype(np.float32)
    xb = (rng.standard_normal((384, 512)) * 0.05).astype(np.float32)
    qa, sa, ga = kl.nv_quantize(torch.from_numpy(xa).to(cuda))
    qb, sb, gb = kl.nv_quantize(torch.from_numpy(xb).to(cuda))
    c = kl.gemm(qa, qb, sfa=sa, sfb=sb, scale_vec=16, scale_a=ga, scale_b=gb, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert kl.read_status() == 0
    ra, rsa, rga = wl.nv_quantize(xa)
    rb, rsb, rgb = wl.nv_quantize(xb)
    elem, norm = og.rel_error(c.cpu().numpy(), og.gemm_nv_f64(ra, rb, rsa, rsb, rga * rgb))
    assert elem <= FP8_TOL and norm <= FP8_TOL


def test_device_nv_quantize_all_zero(cuda):
    """g = 1 and every scale 0 for an all-zero x; the elements are zeros."""
    q, sc, g = kl.nv_quantize(torch.zeros(130, 64, device=cuda))
    torch.cuda.synchronize()
    assert g.item() == 1.0
    blocked = sc.cpu().numpy().reshape(-1, 512)
    want = og.pack_mx_scales(np.zeros((130, 4), dtype=np.uint8), 64, 16).reshape(-1, 512)
    np.testing.assert_array_equal(blocked, want)
    assert not q.view(torch.uint8).any()
