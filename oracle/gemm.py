"""ctypes binding of libkl_oracle.so (gemm_oracle.c). TEST INFRASTRUCTURE ONLY.

Inputs are raw element bits as numpy arrays, row-major: uint16 for bf16, uint8 for e4m3 (the
defaults), np.float16 for f16; pass `kind` for the other formats (F16 on uint16 bits, E5M2 on
uint8 bits, E2M1 on uint8 bytes that each hold two fp4 elements, the first in the low nibble, so a
row of K elements is K / 2 bytes; E3M2 / E2M3 on uint8 bytes of packed fp6, element i of a row at
bits [6i, 6i + 6), least significant bit first, so a row of K elements is 3 K / 4 bytes). Type codes
follow the library's kl_dtype.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libkl_oracle.so"
BF16, F16, E4M3, E5M2, E2M1, E3M2, E2M3 = 0, 1, 2, 3, 8, 11, 12
KINDS = {"bf16": BF16, "f16": F16, "e4m3": E4M3, "e5m2": E5M2, "e2m1": E2M1, "e3m2": E3M2, "e2m3": E2M3}
_lib = None


def build() -> Path:
    src = HERE / "gemm_oracle.c"
    if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-C", str(HERE), "libkl_oracle.so"], check=True, capture_output=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(str(LIB_PATH))
        vp, i64, i32, dbl = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_double
        L.kl_oracle_gemm_f64.argtypes = [i32, vp, i64, vp, i64, i64, i64, i64, dbl, vp, i64, i32]
        L.kl_oracle_gemm_f64.restype = i32
        L.kl_oracle_gemm_f32.argtypes = [i32, vp, i64, vp, i64, i64, i64, i64, dbl, vp, i64, i32]
        L.kl_oracle_gemm_f32.restype = i32
        L.kl_oracle_decode.argtypes = [i32, vp, i64, vp]
        L.kl_oracle_decode.restype = None
        bs = [i32, vp, i64, vp, i64, i64, i64, i64, vp, i64, vp, i64, i32, i32, dbl, vp, i64, i32]
        L.kl_oracle_gemm_bs_f64.argtypes = bs
        L.kl_oracle_gemm_bs_f64.restype = i32
        L.kl_oracle_gemm_bs_f32.argtypes = bs
        L.kl_oracle_gemm_bs_f32.restype = i32
        _lib = L
    return _lib


def _kind(a: np.ndarray, kind=None) -> int:
    if kind is not None:
        k = KINDS[kind] if isinstance(kind, str) else int(kind)
        if (k in (BF16, F16)) != (a.dtype.itemsize == 2) or a.dtype.itemsize not in (1, 2):
            raise TypeError(f"element kind {kind} does not match {a.dtype} bits")
        return k
    if a.dtype == np.uint16:
        return BF16
    if a.dtype == np.float16:
        return F16
    if a.dtype == np.uint8:
        return E4M3
    raise TypeError("inputs are raw bits: uint16 (bf16), uint8 (e4m3), float16, or pass kind=")


def threads_default() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)


def elements(kind, units: int) -> int:
    """Elements in `units` storage units of a row: two per byte for packed e2m1, four per three
    bytes for packed fp6 (units a multiple of 3), else one."""
    code = None if kind is None else (KINDS.get(kind) if isinstance(kind, str) else int(kind))
    if code == E2M1:
        return 2 * units
    if code in (E3M2, E2M3):
        if units % 3:
            raise ValueError("packed fp6 rows are whole groups of 3 bytes (4 elements)")
        return units // 3 * 4
    return units


def decode(bits: np.ndarray, kind=None) -> np.ndarray:
    bits = np.ascontiguousarray(bits)
    if bits.ndim == 0:
        bits = bits.reshape(1)
    n = elements(kind, bits.shape[-1])
    out = np.empty(bits.shape[:-1] + (n,), dtype=np.float64)
    rows = bits.size // bits.shape[-1] if bits.shape[-1] else 0
    for r, row in enumerate(bits.reshape(rows, bits.shape[-1])):  # one call per row: fp6 rows pack apart
        lib().kl_oracle_decode(_kind(bits, kind), row.ctypes.data, n, out.reshape(rows, n)[r].ctypes.data)
    return out


def gemm_f64(a: np.ndarray, b: np.ndarray, scale: float = 1.0, threads: int | None = None, kind=None) -> np.ndarray:
    """scale * A . B^T with fp64 accumulation; A [M,K], B [N,K] raw bits."""
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    assert a.dtype == b.dtype and a.shape[1] == b.shape[1]
    m, k = a.shape[0], elements(kind, a.shape[1])
    n = b.shape[0]
    c = np.empty((m, n), dtype=np.float64)
    rc = lib().kl_oracle_gemm_f64(_kind(a, kind), a.ctypes.data, k, b.ctypes.data, k, m, n, k, float(scale),
                                  c.ctypes.data, n, threads or threads_default())
    assert rc == 0
    return c


def gemm_f32(a: np.ndarray, b: np.ndarray, scale: float = 1.0, threads: int | None = None, kind=None) -> np.ndarray:
    """scale * A . B^T with fp32 accumulation (the timed CPU baseline)."""
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    m, k = a.shape[0], elements(kind, a.shape[1])
    n = b.shape[0]
    c = np.empty((m, n), dtype=np.float32)
    rc = lib().kl_oracle_gemm_f32(_kind(a, kind), a.ctypes.data, k, b.ctypes.data, k, m, n, k, float(scale),
                                  c.ctypes.data, n, threads or threads_default())
    assert rc == 0
    return c


def e8m0_values(s: np.ndarray) -> np.ndarray:
    """UE8M0 scales (OCP Microscaling Formats v1.0): value 2^(s - 127), s = 255 is NaN."""
    s = np.asarray(s, dtype=np.float64)
    return np.where(s == 255, np.nan, np.exp2(s - 127.0))


def _mx_call(fn, out_dtype, a, b, sfa, sfb, kind, scale, threads, vec=32, sf_format="ue8m0"):
    a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
    sfa, sfb = np.ascontiguousarray(sfa, dtype=np.uint8), np.ascontiguousarray(sfb, dtype=np.uint8)
    m, k = a.shape[0], elements(kind, a.shape[1])
    n = b.shape[0]
    groups = -(-k // vec)
    assert sfa.shape == (m, groups) and sfb.shape == (n, groups) and b.shape[1] == a.shape[1]
    c = np.empty((m, n), dtype=out_dtype)
    rc = fn(_kind(a, kind), a.ctypes.data, k, b.ctypes.data, k, m, n, k, sfa.ctypes.data, groups, sfb.ctypes.data,
            groups, int(vec), int(sf_format == "ue4m3"), float(scale), c.ctypes.data, n, threads or threads_default())
    assert rc == 0
    return c


def gemm_mx_f64(a: np.ndarray, b: np.ndarray, sfa: np.ndarray, sfb: np.ndarray, kind=None,
                scale: float = 1.0, threads: int | None = None) -> np.ndarray:
    """MX block-scaled product in fp64: scale * sum_k (A[m,k] sfa[m, k/32]) (B[n,k] sfb[n, k/32]).

    a, b: raw 8-bit element bits [M,K] / [N,K]; sfa, sfb: UE8M0 bits [M, ceil(K/32)] /
    [N, ceil(K/32)], one scale per 32 consecutive K-elements (the OCP MX block size)."""
    return _mx_call(lib().kl_oracle_gemm_bs_f64, np.float64, a, b, sfa, sfb, kind, scale, threads)


def gemm_mx_f32(a: np.ndarray, b: np.ndarray, sfa: np.ndarray, sfb: np.ndarray, kind=None,
                scale: float = 1.0, threads: int | None = None) -> np.ndarray:
    """The same with fp32 accumulation (the timed CPU baseline of the MX workload)."""
    return _mx_call(lib().kl_oracle_gemm_bs_f32, np.float32, a, b, sfa, sfb, kind, scale, threads)


def gemm_nv_f64(a: np.ndarray, b: np.ndarray, sfa: np.ndarray, sfb: np.ndarray, scale: float = 1.0,
                threads: int | None = None) -> np.ndarray:
    """NVFP4 product in fp64: packed e2m1 A [M, K/2], B [N, K/2] with UE4M3 scales [rows,
    ceil(K/16)], one per 16 consecutive K-elements (an e4m3 byte read as a magnitude), times the
    product of the per-tensor scales `scale`."""
    return _mx_call(lib().kl_oracle_gemm_bs_f64, np.float64, a, b, sfa, sfb, "e2m1", scale, threads, 16, "ue4m3")


def gemm_nv_f32(a, b, sfa, sfb, scale: float = 1.0, threads: int | None = None) -> np.ndarray:
    return _mx_call(lib().kl_oracle_gemm_bs_f32, np.float32, a, b, sfa, sfb, "e2m1", scale, threads, 16, "ue4m3")


def pack_mx_scales(sf: np.ndarray, k: int, vec: int = 32) -> np.ndarray:
    """The blocked scale layout of the block-scaled GEMMs, restated: rows in blocks of 128 and K in
    blocks of 4 scales (4 * vec elements) form 512-byte atoms stored row-block major; inside an atom
    the scale of row r, K-group j is byte (r % 32) * 16 + (r / 32) * 4 + j. Padding holds a scale of
    1 (UE8M0 127 for vec 32, UE4M3 0x38 for vec 16). This is the 128 x 4 scale-factor atom of
    CUTLASS's Sm1xxBlockScaledBasicChunk (K-major)."""
    rows, groups = sf.shape
    rb, kb = -(-rows // 128), -(-k // (4 * vec))
    full = np.full((rb * 128, kb * 4), 127 if vec == 32 else 0x38, dtype=np.uint8)
    full[:rows, :groups] = sf
    t = full.reshape(rb, 4, 32, kb, 4)                  # (row block, r / 32, r % 32, K block, j)
    return np.ascontiguousarray(t.transpose(0, 3, 2, 1, 4)).reshape(-1)


def rel_error(c: np.ndarray, ref: np.ndarray, floor_frac: float = 1e-2) -> tuple[float, float]:
    """(element-wise max of |c - r| / max(|r|, floor_frac * rms(r)), normwise max|c - r| / max|r|).

    Entries smaller than 1% of the typical entry are judged against that scale: fp32 accumulation
    over K terms leaves absolute errors of order sqrt(K) * 2^-24 * rms(r), which no relative bound
    can hold for entries that happen to land near zero."""
    c = np.asarray(c, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    diff = np.abs(c - ref)
    rms = float(np.sqrt(np.mean(ref * ref))) if ref.size else 0.0
    floor = max(floor_frac * rms, 1e-30)
    elem = float(np.max(diff / np.maximum(np.abs(ref), floor))) if ref.size else 0.0
    norm = float(diff.max() / max(np.abs(ref).max(), 1e-30)) if ref.size else 0.0
    return elem, norm
