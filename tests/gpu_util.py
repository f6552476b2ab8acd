"""Helpers for the GPU tests: move oracle-format inputs to the device and check results."""

import numpy as np
import torch

import maia_b200 as kl
from maia_b200 import workloads as wl
from oracle import gemm as og


TORCH_TYPES = {"bf16": torch.bfloat16, "f16": torch.float16, "e4m3": torch.float8_e4m3fn,
               "e5m2": torch.float8_e5m2, "f32": torch.float32, "e2m1": torch.float4_e2m1fn_x2,
               "e3m2": torch.uint8, "e2m3": torch.uint8}  # packed fp6 travels as bytes
FP8_MAX = {"e4m3": 448.0, "e5m2": 57344.0}


def to_device(bits: np.ndarray, dtype: str, device) -> torch.Tensor:
    bits = np.ascontiguousarray(bits)
    if bits.dtype.itemsize == 2:
        return torch.from_numpy(bits.view(np.int16)).to(device).view(TORCH_TYPES[dtype])
    return torch.from_numpy(bits).to(device).view(TORCH_TYPES[dtype])


def random_inputs(m, n, k, dtype="bf16", seed=0, scale=1.0):
    """Raw bits of A [m,k] and B [n,k] drawn from N(0, scale^2), and their dequantisation scales
    (per-tensor amax / format max for the fp8 formats, 1 otherwise)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    xa = rng.standard_normal((m, k), dtype=np.float32) * np.float32(scale)
    xb = rng.standard_normal((n, k), dtype=np.float32) * np.float32(scale)
    if dtype == "bf16":
        return wl.f32_to_bf16_bits(xa), wl.f32_to_bf16_bits(xb), 1.0, 1.0
    if dtype == "f16":
        return wl.f32_to_f16_bits(xa), wl.f32_to_f16_bits(xb), 1.0, 1.0
    enc = wl.f32_to_e4m3_bits if dtype == "e4m3" else wl.f32_to_e5m2_bits
    sa = float(np.abs(xa).max()) / FP8_MAX[dtype]
    sb = float(np.abs(xb).max()) / FP8_MAX[dtype]
    return enc(xa / np.float32(sa)), enc(xb / np.float32(sb)), sa, sb


def run_kl(a_bits, b_bits, dtype, out, device, algo, scale_a=1.0, scale_b=1.0, **kw):
    a = to_device(a_bits, dtype, device)
    b = to_device(b_bits, dtype, device)
    m, n = a.shape[0], b.shape[0]
    c = torch.full((m, n), float("nan"), dtype=TORCH_TYPES[out], device=device)
    sa = sb = None
    if dtype in FP8_MAX:
        sa = torch.tensor([scale_a], dtype=torch.float32, device=device)
        sb = torch.tensor([scale_b], dtype=torch.float32, device=device)
    kl.gemm(a, b, c, scale_a=sa, scale_b=sb, algo=algo, **kw)
    torch.cuda.synchronize()
    assert kl.read_status() == 0, "a device-side wait timed out"
    return c.float().cpu().numpy()


def check(c, a_bits, b_bits, scale, tol, threads=None, kind=None, c0=None):
    """Compare c with scale * A . B^T (+ c0, the C that a reducing call added into)."""
    ref = og.gemm_f64(a_bits, b_bits, scale, threads=threads, kind=kind)
    if c0 is not None:
        ref = ref + np.asarray(c0, dtype=np.float64)
    assert not np.isnan(c).any(), "output has unwritten (NaN) entries"
    elem, norm = og.rel_error(c, ref)
    assert norm <= tol, f"max relative error (normwise) {norm:.3e} > {tol}"
    assert elem <= tol, f"max element-wise relative error {elem:.3e} > {tol} (normwise {norm:.3e})"
    return elem, norm
