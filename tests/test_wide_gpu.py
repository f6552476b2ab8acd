"""256 x 512 CTA-pair tiles (kl_gemm_desc.variant = 4: two MMAs of N = 256 per stage of A, one TMEM
accumulator of 512 columns) against the fp64 CPU oracle, on every entry: shapes that fill whole
tiles, ragged M / N / K (the second sub-tile partly or wholly past N), several waves of tiles,
e4m3 inputs with per-tensor scales, batched and C += result.

Tolerances as in test_gemm_gpu.py: 1e-2 for bf16 inputs, 5e-2 for fp8.
"""

import pytest
import torch

import maia_b200 as kl

from gpu_util import check, random_inputs, run_kl, to_device

pytestmark = pytest.mark.gpu

TOL16 = 1e-2
FP8_TOL = 5e-2
WIDE = dict(variant=4)

# N a multiple of 8 and K of 8 (bf16) or 16 (e4m3): the 16-byte row pitches TMA needs.
SHAPES = [(256, 512, 64), (256, 512, 8192), (512, 1024, 1024), (300, 712, 200), (257, 296, 136),
          (1000, 1536, 520), (2048, 4096, 512)]


@pytest.mark.parametrize("shape", SHAPES)
def test_wide_bf16(cuda, shape):
    m, n, k = shape
    a, b, _, _ = random_inputs(m, n, k, "bf16", seed=7 * m + n + k)
    check(run_kl(a, b, "bf16", "bf16", cuda, kl.ALGO_2CTA, **WIDE), a, b, 1.0, TOL16)


@pytest.mark.parametrize("shape", [(256, 512, 256), (300, 712, 208), (1024, 2048, 1024)])
def test_wide_e4m3(cuda, shape):
    m, n, k = shape
    a, b, sa, sb = random_inputs(m, n, k, "e4m3", seed=11 * m + k)
    c = run_kl(a, b, "e4m3", "bf16", cuda, kl.ALGO_2CTA, scale_a=sa, scale_b=sb, **WIDE)
    check(c, a, b, sa * sb, FP8_TOL, kind="e4m3")


def test_wide_matches_narrow_tiles(cuda):
    """Same K order per output element on both tile shapes: the fp32 sums, and so the bf16 C,
    agree bit for bit with the 256 x 256 kernel."""
    a_bits, b_bits, _, _ = random_inputs(768, 1280, 640, "bf16", seed=5)
    a = to_device(a_bits, "bf16", cuda)
    b = to_device(b_bits, "bf16", cuda)
    c0 = kl.gemm(a, b, algo=kl.ALGO_2CTA, stream_k=-1)
    c4 = kl.gemm(a, b, algo=kl.ALGO_2CTA, variant=4)
    torch.cuda.synchronize()
    assert torch.equal(c0.view(torch.int16), c4.view(torch.int16))


def test_wide_batched_and_accumulate(cuda):
    l, m, n, k = 3, 256, 1024, 384
    bits = [random_inputs(m, n, k, "bf16", seed=40 + i) for i in range(l)]
    a = torch.stack([to_device(x[0], "bf16", cuda) for x in bits])
    b = torch.stack([to_device(x[1], "bf16", cuda) for x in bits])
    c = kl.gemm(a, b, algo=kl.ALGO_2CTA, variant=4, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    for i in range(l):
        check(c[i].float().cpu().numpy(), bits[i][0], bits[i][1], 1.0, TOL16)
    # C += A . B^T on a bf16 C (read, add in fp32, one rounding).
    c0 = c[0].clone()
    kl.gemm(a[0], b[0], c0, algo=kl.ALGO_2CTA, variant=4, accumulate=True)
    torch.cuda.synchronize()
    assert kl.read_status() == 0
    check(c0.float().cpu().numpy(), bits[0][0], bits[0][1], 1.0, TOL16, c0=c[0].float().cpu().numpy())


def test_wide_rejects_other_types(cuda):
    a = torch.zeros((256, 64), dtype=torch.bfloat16, device=cuda)
    b = torch.zeros((512, 64), dtype=torch.bfloat16, device=cuda)
    c = torch.zeros((256, 512), dtype=torch.float32, device=cuda)
    with pytest.raises(kl.KlError, match="variant 4"):
        kl.gemm(a, b, c, algo=kl.ALGO_2CTA, variant=4)


@pytest.mark.parametrize("m,n,k,dtype,want", [
    (8192, 8192, 8192, "bf16", (256, 512)),    # 512 tiles on 74 pairs: as full as 1024 narrow ones
    (8192, 1024, 8192, "bf16", (256, 512)),    # one rank's shard of 8: one wave of 64 tiles
    (8192, 4096, 8192, "bf16", (256, 256)),    # wide tiles would fill 3.46 waves instead of 6.92
    (8192, 2048, 8192, "bf16", (256, 256)),    # the split tail fills the narrow tiles' last wave
    (16384, 16384, 8192, "e4m3", (256, 256)),  # fp8 stays on 256 x 256
    (128, 28672, 8192, "bf16", (128, 256)),    # decode, 128 rows: one CTA
    (16, 28672, 8192, "bf16", (0, 0)),         # decode, 16 rows: the stream-K skinny kernel
])
def test_default_tile_choice(cuda, m, n, k, dtype, want):
    """kl_gemm_resolve_tile names the tile kl_gemm's defaults run (nothing is launched)."""
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float8_e4m3fn
    a = torch.empty((m, k), dtype=tdt, device=cuda)
    b = torch.empty((n, k), dtype=tdt, device=cuda)
    c = torch.empty((m, n), dtype=torch.bfloat16, device=cuda)
    assert kl.resolve_tile(a, b, c) == want
    if m >= 256:  # variant 1 asks for the 256 x 256 tiles, variant 4 for the wide ones
        assert kl.resolve_tile(a, b, c, algo=kl.ALGO_2CTA, variant=1) == (256, 256)
        assert kl.resolve_tile(a, b, c, algo=kl.ALGO_2CTA, variant=4) == (256, 512)
