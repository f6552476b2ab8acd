"""Helpers for the GPU tests: move oracle-format inputs to the device and check results."""

import numpy as np
import torch

import maia_b200 as kl
from maia_b200 import workloads as wl
from oracle import gemm as og


def to_device(bits: np.ndarray, dtype: str, device) -> torch.Tensor:
    if dtype == "bf16":
        return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).to(device).view(torch.bfloat16)
    return torch.from_numpy(np.ascontiguousarray(bits)).to(device).view(torch.float8_e4m3fn)


def random_inputs(m, n, k, dtype="bf16", seed=0, scale=1.0):
    rng = np.random.Generator(np.random.PCG64(seed))
    xa = rng.standard_normal((m, k), dtype=np.float32) * np.float32(scale)
    xb = rng.standard_normal((n, k), dtype=np.float32) * np.float32(scale)
    if dtype == "bf16":
        return wl.f32_to_bf16_bits(xa), wl.f32_to_bf16_bits(xb), 1.0, 1.0
    sa = float(np.abs(xa).max()) / 448.0
    sb = float(np.abs(xb).max()) / 448.0
    return wl.f32_to_e4m3_bits(xa / np.float32(sa)), wl.f32_to_e4m3_bits(xb / np.float32(sb)), sa, sb


def run_kl(a_bits, b_bits, dtype, out, device, algo, scale_a=1.0, scale_b=1.0, **kw):
    a = to_device(a_bits, dtype, device)
    b = to_device(b_bits, dtype, device)
    m, n = a.shape[0], b.shape[0]
    odt = torch.bfloat16 if out == "bf16" else torch.float32
    c = torch.full((m, n), float("nan"), dtype=odt, device=device)
    sa = sb = None
    if dtype == "e4m3":
        sa = torch.tensor([scale_a], dtype=torch.float32, device=device)
        sb = torch.tensor([scale_b], dtype=torch.float32, device=device)
    kl.gemm(a, b, c, scale_a=sa, scale_b=sb, algo=algo, **kw)
    torch.cuda.synchronize()
    assert kl.read_status() == 0, "a device-side wait timed out"
    return c.float().cpu().numpy()


def check(c, a_bits, b_bits, scale, tol, threads=None):
    ref = og.gemm_f64(a_bits, b_bits, scale, threads=threads)
    assert not np.isnan(c).any(), "output has unwritten (NaN) entries"
    elem, norm = og.rel_error(c, ref)
    assert norm <= tol, f"max relative error (normwise) {norm:.3e} > {tol}"
    assert elem <= tol, f"max element-wise relative error {elem:.3e} > {tol} (normwise {norm:.3e})"
    return elem, norm
