"""The benchmark workloads of this GEMM engine, with seeded synthetic inputs.

Each tensor comes from its own numpy PCG64 stream seeded ``seed * 1000 + tensor_id`` (A = 0,
B = 1), drawn in row-major order as float32, then rounded to the input type:
  * bf16: round-to-nearest-even of the float32 value;
  * e4m3: per-tensor scale = amax / 448, q = RNE(x / scale) (|x / scale| <= 448, so no overflow);
  * mxfp8: MX quantisation to e4m3 with a UE8M0 scale per 32 K-elements (mx_quantize).
Inputs are returned as raw bits (uint16 / uint8 numpy arrays) so that the GPU and the CPU oracle
see byte-identical operands.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class Workload:
    name: str
    m: int
    n: int
    k: int
    dtype: str          # "bf16", "e4m3", "mxfp8" (e4m3 elements with MX block scales), "mxfp6" (e2m3),
                        # "mxfp4" or "nvfp4" (e2m1)
    out: str            # "bf16" or "f32"
    dist: str           # "uniform" (on [-1, 1]) or "normal"
    a_scale: float      # multiplier of A's standard normal (normal) draws
    b_scale: float
    seed: int

    @property
    def flops(self) -> float:
        return 2.0 * self.m * self.n * self.k

    @property
    def in_bytes(self) -> float:
        return 2 if self.dtype == "bf16" else 0.5 if self.dtype in ("mxfp4", "nvfp4") else 0.75 if self.dtype == "mxfp6" else 1

    @property
    def scale_bytes(self) -> int:
        """MX block scales: one byte per 32 K-elements of every row of A and B."""
        if self.dtype == "nvfp4":
            return (self.m + self.n) * -(-self.k // 16)
        return (self.m + self.n) * -(-self.k // 32) if self.dtype in ("mxfp8", "mxfp6", "mxfp4") else 0

    @property
    def out_bytes(self) -> int:
        return 2 if self.out == "bf16" else 4

    @property
    def bytes(self) -> int:
        """Algorithmic bytes: every matrix moved once."""
        return int((self.m * self.k + self.n * self.k) * self.in_bytes) + self.m * self.n * self.out_bytes + self.scale_bytes


# C1..C5: the reference's GEMM contract at its benchmark shapes.
C1 = Workload("c1_256_bf16_f32", 256, 256, 256, "bf16", "f32", "uniform", 1.0, 1.0, 0)
C2 = Workload("c2_4096_bf16", 4096, 4096, 4096, "bf16", "bf16", "normal", 0.05, 0.05, 1)
C3 = Workload("c3_8192_bf16", 8192, 8192, 8192, "bf16", "bf16", "normal", 0.02, 0.02, 2)
C4 = Workload("c4_16384x16384x8192_e4m3", 16384, 16384, 8192, "e4m3", "bf16", "normal", 1.0, 1.0, 3)
C5 = {m: Workload(f"c5_skinny_m{m}", m, 28672, 8192, "bf16", "bf16", "normal", 1.0, 0.02, 4) for m in (16, 64, 128)}
# C4's shape and draws, MX-quantised instead of per-tensor scaled (block-scaled fp8); and C3's.
C4MX = Workload("c4mx_16384x16384x8192_mxfp8", 16384, 16384, 8192, "mxfp8", "bf16", "normal", 1.0, 1.0, 3)
C3MX = Workload("c3mx_8192_mxfp8", 8192, 8192, 8192, "mxfp8", "bf16", "normal", 0.02, 0.02, 2)
# The same shapes in MXFP4 (packed e2m1 elements, UE8M0 scales per 32).
C3MXF4 = Workload("c3mxf4_8192_mxfp4", 8192, 8192, 8192, "mxfp4", "bf16", "normal", 0.02, 0.02, 2)
C4MXF4 = Workload("c4mxf4_16384x16384x8192_mxfp4", 16384, 16384, 8192, "mxfp4", "bf16", "normal", 1.0, 1.0, 3)
C3NVF4 = Workload("c3nvf4_8192_nvfp4", 8192, 8192, 8192, "nvfp4", "bf16", "normal", 0.02, 0.02, 2)
# C3's shape in MXFP6 (packed e2m3 elements, UE8M0 scales per 32; kind::mxf8f6f4 at the fp8 rate).
C3MXF6 = Workload("c3mxf6_8192_mxfp6", 8192, 8192, 8192, "mxfp6", "bf16", "normal", 0.02, 0.02, 2)

# C5's decode shapes with MX-quantised weights and activations (block-scaled decode).
C5MX = {m: Workload(f"c5mx_skinny_m{m}_mxfp8", m, 28672, 8192, "mxfp8", "bf16", "normal", 1.0, 0.02, 4) for m in (16, 64, 128)}
C5MXF4 = {m: Workload(f"c5mxf4_skinny_m{m}_mxfp4", m, 28672, 8192, "mxfp4", "bf16", "normal", 1.0, 0.02, 4)
          for m in (16, 64, 128)}

ALL = {w.name: w for w in (C1, C2, C3, C4, C4MX, C3MX, C3MXF4, C4MXF4, C3NVF4, C3MXF6, *C5.values(), *C5MX.values(),
                           *C5MXF4.values())}
MX_ELEMENT = {"mxfp8": "e4m3", "mxfp6": "e2m3", "mxfp4": "e2m1"}  # element format of each MX workload dtype


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 to bf16 (nearest, ties to even); returns the 16-bit patterns."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounding = ((u >> 16) & np.uint32(1)) + np.uint32(0x7FFF)
    return ((u + rounding) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


_E4M3_TABLE = None


def e4m3_values() -> np.ndarray:
    """The 256 e4m3 ("fn") values by bit pattern (NaN at 0x7F and 0xFF)."""
    global _E4M3_TABLE
    if _E4M3_TABLE is None:
        v = np.arange(256)
        sign = np.where(v & 0x80, -1.0, 1.0)
        exp = (v >> 3) & 0xF
        man = v & 7
        mag = np.where(exp == 0, man / 8.0 * 2.0 ** -6, (1 + man / 8.0) * 2.0 ** (exp - 7.0))
        vals = sign * mag
        vals[(exp == 15) & (man == 7)] = np.nan
        _E4M3_TABLE = vals
    return _E4M3_TABLE


def f32_to_e4m3_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 to the nearest e4m3 value (ties to even mantissa), saturating at +-448.

    Normal range: keep 3 mantissa bits of the float32 pattern with round-to-nearest-even (a carry
    moves into the exponent) and rebias the exponent from 127 to 7. Below 2^-6 the e4m3 grid is
    uniform (step 2^-9), so the pattern is the rounded multiple of 2^-9."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    flat = x.reshape(-1)
    out = np.empty(flat.shape, dtype=np.uint8)
    for i in range(0, flat.size, 1 << 22):  # bounded temporaries on large matrices
        v = flat[i:i + (1 << 22)]
        u = v.view(np.uint32)
        sign = ((u >> 24) & np.uint32(0x80)).astype(np.uint8)
        mag = u & np.uint32(0x7FFFFFFF)
        rounded = (mag + np.uint32(0x7FFFF) + ((mag >> 20) & np.uint32(1))) >> 20
        normal = rounded.astype(np.int32) - (120 << 3)
        # Below 2^-6 (0x3C800000) the value times 512 is below 8: exact in float32, rint ties to even.
        sub = np.rint(np.minimum(np.abs(v), np.float32(1.0)) * np.float32(512.0)).astype(np.int32)
        q = np.where(mag < np.uint32(0x3C800000), sub, normal)
        q = np.clip(q, 0, 0x7E).astype(np.uint8)
        out[i:i + v.size] = np.where(q != 0, q | sign, q)
    return out.reshape(x.shape)


def f32_to_e4m3_bits_nearest(x: np.ndarray) -> np.ndarray:
    """Slow definition of the same rounding: search the sorted grid of e4m3 values."""
    vals = e4m3_values()
    grid = vals[np.arange(0, 0x7F)]
    a = np.minimum(np.abs(np.asarray(x, dtype=np.float64)), 448.0)
    idx = np.clip(np.searchsorted(grid, a), 1, len(grid) - 1)
    lo, hi = grid[idx - 1], grid[idx]
    pick_hi = (a - lo > hi - a) | ((a - lo == hi - a) & (idx % 2 == 0))
    q = np.where(pick_hi, idx, idx - 1).astype(np.uint8)
    return np.where(np.signbit(x) & (q != 0), q | 0x80, q).astype(np.uint8)


_E5M2_TABLE = None


def e5m2_values() -> np.ndarray:
    """The 256 e5m2 values by bit pattern (infinities at 0x7C / 0xFC, NaN above them)."""
    global _E5M2_TABLE
    if _E5M2_TABLE is None:
        v = np.arange(256)
        sign = np.where(v & 0x80, -1.0, 1.0)
        exp = (v >> 2) & 0x1F
        man = v & 3
        mag = np.where(exp == 0, man / 4.0 * 2.0 ** -14, (1 + man / 4.0) * 2.0 ** (exp - 15.0))
        vals = sign * mag
        vals[exp == 31] = np.where(man[exp == 31] == 0, np.inf, np.nan) * sign[exp == 31]
        _E5M2_TABLE = vals
    return _E5M2_TABLE


def f32_to_e5m2_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 to the nearest e5m2 value (ties to even mantissa), saturating at +-57344.

    As for e4m3: keep 2 mantissa bits of the float32 pattern with round-to-nearest-even and rebias
    the exponent from 127 to 15; below 2^-14 the grid is uniform with step 2^-16."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    flat = x.reshape(-1)
    out = np.empty(flat.shape, dtype=np.uint8)
    for i in range(0, flat.size, 1 << 22):  # bounded temporaries on large matrices
        v = flat[i:i + (1 << 22)]
        u = v.view(np.uint32)
        sign = ((u >> 24) & np.uint32(0x80)).astype(np.uint8)
        mag = u & np.uint32(0x7FFFFFFF)
        rounded = (mag + np.uint32(0xFFFFF) + ((mag >> 21) & np.uint32(1))) >> 21
        normal = rounded.astype(np.int32) - (112 << 2)
        # Below 2^-14 the value times 65536 is below 4: exact in float32, rint ties to even.
        sub = np.rint(np.minimum(np.abs(v), np.float32(1.0)) * np.float32(65536.0)).astype(np.int32)
        q = np.where(mag < np.uint32(0x38800000), sub, normal)
        q = np.clip(q, 0, 0x7B).astype(np.uint8)
        out[i:i + v.size] = np.where(q != 0, q | sign, q)
    return out.reshape(x.shape)


def f32_to_e5m2_bits_nearest(x: np.ndarray) -> np.ndarray:
    """Slow definition of the same rounding: search the sorted grid of finite e5m2 values."""
    grid = e5m2_values()[np.arange(0, 0x7C)]
    a = np.minimum(np.abs(np.asarray(x, dtype=np.float64)), 57344.0)
    idx = np.clip(np.searchsorted(grid, a), 1, len(grid) - 1)
    lo, hi = grid[idx - 1], grid[idx]
    pick_hi = (a - lo > hi - a) | ((a - lo == hi - a) & (idx % 2 == 0))
    q = np.where(pick_hi, idx, idx - 1).astype(np.uint8)
    return np.where(np.signbit(x) & (q != 0), q | 0x80, q).astype(np.uint8)


def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 to IEEE binary16 (nearest, ties to even); returns the 16-bit patterns."""
    return np.ascontiguousarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


E2M1_GRID = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])  # the e2m1 magnitudes, by code 0..7


def minifloat_codes(x: np.ndarray, eb: int, mb: int) -> np.ndarray:
    """Round float32 to a sign-magnitude minifloat with `eb` exponent bits (bias 2^(eb-1) - 1), `mb`
    mantissa bits and no special values: nearest, ties to the even code, saturating at the largest
    magnitude; returns the codes (sign in bit eb + mb) as uint8. Each value's binade is scaled so
    that the representable values there are consecutive integers n, rounded with rint (half to
    even); code = ((e + bias) << mb) + n - 2^mb, which also covers the subnormals (lowest binade)
    and a carry into the next binade. Every step is exact in float32 for these widths."""
    bias = (1 << (eb - 1)) - 1
    vmax = np.float32((2.0 - 2.0 ** -mb) * 2.0 ** ((1 << eb) - 1 - bias))
    x = np.asarray(x, dtype=np.float32)
    flat = x.reshape(-1)
    out = np.empty(flat.shape, dtype=np.uint8)
    for i in range(0, flat.size, 1 << 24):  # bounded temporaries on large matrices
        v = flat[i:i + (1 << 24)]
        a = np.minimum(np.abs(v), vmax)
        e = np.maximum(np.frexp(a)[1].astype(np.int32) - 1, 1 - bias)  # binade exponent
        e[a == 0] = 1 - bias  # frexp(0) reports exponent 0, above the lowest binade when bias > 1
        n = np.rint(np.ldexp(a, mb - e)).astype(np.int32)              # a / 2^(e - mb), exact
        code = ((e + bias) << mb) + n - (1 << mb)
        out[i:i + v.size] = np.where(np.signbit(v) & (code != 0), code | (1 << (eb + mb)), code)
    return out.reshape(x.shape)


def f32_to_e2m1_codes(x: np.ndarray) -> np.ndarray:
    """Round float32 to the nearest e2m1 value (ties to the even code, i.e. mantissa 0), saturating
    at +-6; returns 4-bit codes (sign in bit 3) as uint8."""
    return minifloat_codes(x, 2, 1)


def pack_e2m1(codes: np.ndarray) -> np.ndarray:
    """Pack 4-bit codes [rows, K] (K even) two per byte, the first element in the low nibble."""
    c = np.ascontiguousarray(codes, dtype=np.uint8)
    return (c[..., 0::2] | (c[..., 1::2] << 4)).astype(np.uint8)


def _fp6_grid(eb: int) -> np.ndarray:
    """The 32 magnitudes of an fp6 format with `eb` exponent bits (bias 2^(eb-1) - 1) and 5 - eb
    mantissa bits, by code (exponent in the high bits): increasing, no special values."""
    mb, bias = 5 - eb, (1 << (eb - 1)) - 1
    c = np.arange(32)
    e, m = c >> mb, c & ((1 << mb) - 1)
    return np.where(e == 0, m * 2.0 ** (1 - bias - mb), (m + (1 << mb)) * 2.0 ** (e - bias - mb))


FP6_GRID = {"e3m2": _fp6_grid(3), "e2m3": _fp6_grid(2)}  # largest 28 and 7.5


def f32_to_fp6_codes(x: np.ndarray, kind: str) -> np.ndarray:
    """Round float32 to the nearest fp6 (e3m2 or e2m3) value, ties to the even code (mantissa LSB
    0), saturating at the largest magnitude; returns 6-bit codes (sign in bit 5) as uint8."""
    return minifloat_codes(x, 3, 2) if kind == "e3m2" else minifloat_codes(x, 2, 3)


def pack_fp6(codes: np.ndarray) -> np.ndarray:
    """Pack 6-bit codes [rows, K] (K a multiple of 4) into [rows, 3 K / 4] bytes: element i at bits
    [6i, 6i + 6) of the row, least significant bit first (four elements per three bytes)."""
    c = np.ascontiguousarray(codes, dtype=np.uint32)
    w = c[..., 0::4] | (c[..., 1::4] << 6) | (c[..., 2::4] << 12) | (c[..., 3::4] << 18)
    out = np.stack([w & 0xFF, (w >> 8) & 0xFF, (w >> 16) & 0xFF], axis=-1).astype(np.uint8)
    return out.reshape(c.shape[:-1] + (c.shape[-1] // 4 * 3,))


def unpack_fp6(packed: np.ndarray) -> np.ndarray:
    """Inverse of pack_fp6: [rows, 3 K / 4] bytes to 6-bit codes [rows, K]."""
    b = np.ascontiguousarray(packed, dtype=np.uint32).reshape(packed.shape[:-1] + (-1, 3))
    w = b[..., 0] | (b[..., 1] << 8) | (b[..., 2] << 16)
    out = np.stack([(w >> (6 * j)) & 63 for j in range(4)], axis=-1).astype(np.uint8)
    return out.reshape(packed.shape[:-1] + (-1,))


MX_EMAX = {"e4m3": 8, "e5m2": 15, "e2m1": 2, "e3m2": 4, "e2m3": 2}  # exponent of the largest normal element value


def mx_quantize(x: np.ndarray, kind: str = "e4m3") -> tuple[np.ndarray, np.ndarray]:
    """MX quantisation (OCP Microscaling Formats v1.0) of float32 rows in blocks of 32 K-elements:
    shared scale 2^(floor(log2(amax)) - emax) as UE8M0 bits, elements x / scale rounded to the
    element format (nearest, ties to even, saturating). Returns (element bits, scale bits
    [rows, ceil(K/32)]); e2m1 elements come packed two per byte ([rows, K/2], K even), e3m2 /
    e2m3 elements four per three bytes ([rows, 3 K / 4], K a multiple of 4)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, k = x.shape
    groups = -(-k // 32)
    padded = np.zeros((rows, groups * 32), dtype=np.float32)
    padded[:, :k] = x
    amax = np.abs(padded.reshape(rows, groups, 32)).max(axis=2).astype(np.float64)
    e = np.where(amax > 0, np.floor(np.log2(np.where(amax > 0, amax, 1.0))), 0.0) - MX_EMAX[kind]
    sbits = np.clip(e + 127, 0, 254).astype(np.uint8)
    inv = np.exp2(127.0 - sbits.astype(np.float64))
    q = (padded.reshape(rows, groups, 32) * inv[:, :, None]).reshape(rows, groups * 32)[:, :k].astype(np.float32)
    if kind == "e2m1":
        return pack_e2m1(f32_to_e2m1_codes(q)), sbits
    if kind in FP6_GRID:
        return pack_fp6(f32_to_fp6_codes(q, kind)), sbits
    enc = f32_to_e4m3_bits if kind == "e4m3" else f32_to_e5m2_bits
    return enc(q), sbits


def nv_quantize(x: np.ndarray) -> tuple[np.ndarray, np.ndarray, float]:
    """NVFP4 quantisation of float32 rows: a per-tensor scale g = amax / (448 * 6), then per block
    of 16 K-elements a UE4M3 scale s = e4m3(amax_block / (6 g)) (round to nearest, saturating),
    elements e2m1(x / (s g)). Returns (packed e2m1 [rows, K/2], UE4M3 bits [rows, ceil(K/16)], g);
    x ~ g * s * e2m1."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, k = x.shape
    groups = -(-k // 16)
    padded = np.zeros((rows, groups * 16), dtype=np.float32)
    padded[:, :k] = x
    amax = float(np.abs(x).max()) if x.size else 0.0
    g = amax / (448.0 * 6.0) if amax > 0 else 1.0
    bmax = np.abs(padded.reshape(rows, groups, 16)).max(axis=2)
    sbits = f32_to_e4m3_bits((bmax / (6.0 * g)).astype(np.float32)) & np.uint8(0x7F)
    s = e4m3_values()[sbits].astype(np.float64)
    with np.errstate(divide="ignore", invalid="ignore"):
        inv = np.where(s > 0, 1.0 / (s * g), 0.0)
    q = (padded.reshape(rows, groups, 16) * inv[:, :, None]).reshape(rows, groups * 16)[:, :k].astype(np.float32)
    return pack_e2m1(f32_to_e2m1_codes(q)), sbits, g


def draw(w: Workload, tensor_id: int, rows: int, cols: int, scale: float) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(w.seed * 1000 + tensor_id))
    if w.dist == "uniform":
        x = rng.random((rows, cols), dtype=np.float32) * np.float32(2.0) - np.float32(1.0)
    else:
        x = rng.standard_normal((rows, cols), dtype=np.float32)
        if scale != 1.0:
            x *= np.float32(scale)
    return x


def make_inputs(w: Workload, rows_a: int | None = None):
    """(A bits, B bits, scale_a, scale_b). rows_a limits A to its first rows (a bounded CPU sample).
    For mxfp8 / mxfp4 the scales are the row-major UE8M0 arrays [rows, ceil(K/32)] of A and B; for
    nvfp4 they are (UE4M3 array [rows, ceil(K/16)], per-tensor fp32 scale) pairs."""
    ra = w.m if rows_a is None else min(rows_a, w.m)
    xa = draw(w, 0, w.m, w.k, w.a_scale)[:ra] if rows_a is not None else draw(w, 0, w.m, w.k, w.a_scale)
    xb = draw(w, 1, w.n, w.k, w.b_scale)
    if w.dtype == "bf16":
        return f32_to_bf16_bits(xa), f32_to_bf16_bits(xb), 1.0, 1.0
    if w.dtype == "nvfp4":
        qa, sfa, ga = nv_quantize(xa)
        qb, sfb, gb = nv_quantize(xb)
        return qa, qb, (sfa, ga), (sfb, gb)
    if w.dtype in MX_ELEMENT:
        kind = MX_ELEMENT[w.dtype]
        qa, sfa = mx_quantize(xa, kind)
        qb, sfb = mx_quantize(xb, kind)
        return qa, qb, sfa, sfb
    # fp8: per-tensor scales from the full tensors' amax.
    sa = float(np.abs(draw(w, 0, w.m, w.k, w.a_scale)).max()) / 448.0 if rows_a is not None else float(np.abs(xa).max()) / 448.0
    sb = float(np.abs(xb).max()) / 448.0
    return f32_to_e4m3_bits(xa / np.float32(sa)), f32_to_e4m3_bits(xb / np.float32(sb)), sa, sb
