"""Python binding of libkl_b200.so, the B200 dense-GEMM engine (C ABI in include/kl_gemm.h).

Device memory, streams and the process group come from PyTorch; every GEMM runs in the library's
own sm_100a kernels. There is no fallback: if the library is missing or a call fails, the error is
raised.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libkl_b200.so"

# kl_status
KL_OK = 0
KL_ERR_INVALID_ARGUMENT = 1
KL_ERR_NOT_SUPPORTED = 2
KL_ERR_CUDA = 3
KL_ERR_TIMEOUT = 4
KL_ERR_NCCL = 5

# kl_dtype
KL_BF16, KL_F16, KL_E4M3, KL_E5M2, KL_F32, KL_I8, KL_U8, KL_I32, KL_E2M1, KL_UE8M0, KL_UE4M3, KL_E3M2, KL_E2M3 = range(13)
FP6_TYPES = {"e3m2": KL_E3M2, "e2m3": KL_E2M3}

# kl_algo
ALGO_AUTO, ALGO_1CTA, ALGO_2CTA, ALGO_SKINNY = range(4)

EXPORTED = (
    "kl_version", "kl_last_error", "kl_gemm", "kl_gemm_workspace_size", "kl_gemm_resolve_algo", "kl_gemm_resolve_tile", "kl_gemm_ws", "kl_release_workspaces",
    "kl_set_wait_timeout_ns", "kl_read_status", "kl_probe_wait_timeout", "kl_smem_tile_offset",
    "kl_tma_box_geometry", "kl_tma_box_position", "kl_umma_smem_desc", "kl_mma_instr_desc",
    "kl_make_tma_desc", "kl_gemm_skinny_noalloc", "kl_gemm_host", "kl_gemm_host_b", "kl_gemm_clock_probe", "kl_gemm_gather", "kl_gemm_gather_multicast",
    "kl_ipc_get_handle", "kl_ipc_open_handle", "kl_ipc_close", "kl_umma_smem_desc_mn", "kl_mma_instr_desc_major",
    "kl_mma_instr_desc_block_scaled", "kl_mx_scale_bytes", "kl_mx_pack_scales", "kl_block_scale_bytes",
    "kl_pack_block_scales", "kl_mx_quantize", "kl_nv_quantize",
    "kl_comm_get_unique_id", "kl_comm_init", "kl_comm_all_gather", "kl_comm_wait", "kl_comm_is_aborted",
    "kl_comm_destroy",
)


class KlError(RuntimeError):
    """A kl_status other than KL_OK, with the library's message."""

    def __init__(self, status: int, message: str):
        super().__init__(f"kl status {status}: {message}")
        self.status = status
        self.message = message


class GemmDesc(ctypes.Structure):
    _fields_ = [
        ("m", ctypes.c_int64), ("n", ctypes.c_int64), ("k", ctypes.c_int64),
        ("a", ctypes.c_void_p), ("lda", ctypes.c_int64),
        ("b", ctypes.c_void_p), ("ldb", ctypes.c_int64),
        ("c", ctypes.c_void_p), ("ldc", ctypes.c_int64),
        ("ab_type", ctypes.c_int32), ("c_type", ctypes.c_int32),
        ("alpha", ctypes.c_float),
        ("scale_a", ctypes.c_void_p), ("scale_b", ctypes.c_void_p),
        ("algo", ctypes.c_int32), ("group_m", ctypes.c_int32),
        ("max_ctas", ctypes.c_int32), ("variant", ctypes.c_int32),
        ("prefetch", ctypes.c_int32),
        ("batch", ctypes.c_int64),
        ("stride_a", ctypes.c_int64), ("stride_b", ctypes.c_int64), ("stride_c", ctypes.c_int64),
        ("a_major", ctypes.c_int32), ("b_major", ctypes.c_int32),
        ("c_reduce", ctypes.c_int32), ("swizzle", ctypes.c_int32),
        ("block_scale", ctypes.c_int32), ("stream_k", ctypes.c_int32),
        ("sfa", ctypes.c_void_p), ("sfb", ctypes.c_void_p),
        ("groups", ctypes.c_int32), ("launch_overlap", ctypes.c_int32),
        ("m_block_group", ctypes.c_void_p),
    ]


class TmaBox(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("inner", "outer", "col_boxes", "row_boxes", "count", "bytes")]


_lib = None


def lib() -> ctypes.CDLL:
    """The loaded library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m maia_b200.build`")
        L = ctypes.CDLL(str(LIB_PATH))
        i32, i64, u32, u64, vp = ctypes.c_int32, ctypes.c_int64, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_void_p
        P = ctypes.POINTER
        sig = {
            "kl_version": (i32, []),
            "kl_release_workspaces": (i32, []),
            "kl_last_error": (ctypes.c_char_p, []),
            "kl_gemm": (i32, [P(GemmDesc), vp]),
            "kl_gemm_workspace_size": (i32, [P(GemmDesc), P(ctypes.c_size_t)]),
            "kl_gemm_resolve_algo": (i32, [P(GemmDesc), P(ctypes.c_int32)]),
            "kl_gemm_resolve_tile": (i32, [P(GemmDesc), P(ctypes.c_int32), P(ctypes.c_int32)]),
            "kl_gemm_ws": (i32, [P(GemmDesc), vp, ctypes.c_size_t, vp]),
            "kl_set_wait_timeout_ns": (None, [u64]),
            "kl_read_status": (i32, [P(i32), i32]),
            "kl_probe_wait_timeout": (i32, [u64, vp]),
            "kl_smem_tile_offset": (i32, [i32, i32, i32, i32, i32, i32, P(i64), P(i64)]),
            "kl_tma_box_geometry": (i32, [i32, i32, i32, i32, P(TmaBox)]),
            "kl_tma_box_position": (i32, [i32, i32, i32, i32, i32, P(i32), P(i32), P(u32)]),
            "kl_umma_smem_desc": (i32, [i32, i32, i32, i32, u32, i32, i32, P(u64)]),
            "kl_mma_instr_desc": (i32, [i32, i32, i32, i32, i32, P(u32)]),
            "kl_make_tma_desc": (i32, [i32, i32, i32, i32, i32, vp, i32, P(i64), P(i64), vp]),
            "kl_gemm_skinny_noalloc": (i32, [P(GemmDesc), vp]),
            "kl_gemm_host": (i32, [P(GemmDesc), vp, vp, vp, i32, vp]),
            "kl_gemm_host_b": (i32, [P(GemmDesc), vp, vp, vp, i32, vp]),
            "kl_gemm_clock_probe": (i32, [P(GemmDesc), P(u64), i32, P(i32), vp]),
            "kl_gemm_gather": (i32, [P(GemmDesc), P(vp), i32, vp]),
            "kl_gemm_gather_multicast": (i32, [P(GemmDesc), vp, vp]),
            "kl_ipc_get_handle": (i32, [vp, vp, P(i64)]),
            "kl_ipc_open_handle": (i32, [vp, P(vp)]),
            "kl_ipc_close": (i32, [vp]),
            "kl_umma_smem_desc_mn": (i32, [i32, i32, i32, i32, u32, i32, i32, i32, P(u64)]),
            "kl_mma_instr_desc_major": (i32, [i32, i32, i32, i32, i32, i32, i32, P(u32)]),
            "kl_mma_instr_desc_block_scaled": (i32, [i32, i32, i32, i32, i32, i32, i32, P(u32)]),
            "kl_mx_scale_bytes": (i64, [i64, i64]),
            "kl_mx_pack_scales": (i32, [vp, i64, i64, i64, vp, vp]),
            "kl_block_scale_bytes": (i64, [i64, i64, i32]),
            "kl_pack_block_scales": (i32, [vp, i64, i64, i32, i64, vp, vp]),
            "kl_mx_quantize": (i32, [vp, i32, i64, i64, i64, i32, vp, i64, vp, vp]),
            "kl_nv_quantize": (i32, [vp, i32, i64, i64, i64, vp, i64, vp, vp, vp]),
            "kl_comm_get_unique_id": (i32, [vp]),
            "kl_comm_init": (i32, [vp, i32, i32, i64, P(vp)]),
            "kl_comm_all_gather": (i32, [vp, vp, vp, i64, vp]),
            "kl_comm_wait": (i32, [vp, vp, i64]),
            "kl_comm_is_aborted": (i32, [vp]),
            "kl_comm_destroy": (i32, [vp, i64]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    return lib().kl_last_error().decode()


def check(status: int) -> None:
    if status != KL_OK:
        raise KlError(status, last_error())


# ------------------------------------------------------------------------------------- encoders

def smem_tile_offset(elem_bytes, rows, cols, span, row, col):
    sw, pl = ctypes.c_int64(), ctypes.c_int64()
    check(lib().kl_smem_tile_offset(elem_bytes, rows, cols, span, row, col, ctypes.byref(sw), ctypes.byref(pl)))
    return sw.value, pl.value


def tma_box_geometry(elem_bytes, rows, cols, span):
    b = TmaBox()
    check(lib().kl_tma_box_geometry(elem_bytes, rows, cols, span, ctypes.byref(b)))
    return {f: getattr(b, f) for f, _ in TmaBox._fields_}


def tma_box_position(elem_bytes, rows, cols, span, i):
    r, c, o = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_uint32()
    check(lib().kl_tma_box_position(elem_bytes, rows, cols, span, i, ctypes.byref(r), ctypes.byref(c), ctypes.byref(o)))
    return r.value, c.value, o.value


def umma_smem_desc(elem_bytes, rows, cols, span, tile_addr, k_block=0, row=0) -> int:
    out = ctypes.c_uint64()
    check(lib().kl_umma_smem_desc(elem_bytes, rows, cols, span, tile_addr, k_block, row, ctypes.byref(out)))
    return out.value


def umma_smem_desc_mn(elem_bytes, k_rows, mn_cols, span, tile_addr, k_block=0, mn_col=0, mn_extent=0) -> int:
    out = ctypes.c_uint64()
    check(lib().kl_umma_smem_desc_mn(elem_bytes, k_rows, mn_cols, span, tile_addr, k_block, mn_col, mn_extent,
                                     ctypes.byref(out)))
    return out.value


def mma_instr_desc_major(a_type, b_type, acc_type, m, n, a_major, b_major) -> int:
    out = ctypes.c_uint32()
    check(lib().kl_mma_instr_desc_major(a_type, b_type, acc_type, m, n, a_major, b_major, ctypes.byref(out)))
    return out.value


def mma_instr_desc_block_scaled(a_type, b_type, m, n, a_sf_id=0, b_sf_id=0, scale_type=KL_UE8M0) -> int:
    out = ctypes.c_uint32()
    check(lib().kl_mma_instr_desc_block_scaled(a_type, b_type, scale_type, m, n, a_sf_id, b_sf_id, ctypes.byref(out)))
    return out.value


def mma_instr_desc(a_type, b_type, acc_type, m, n) -> int:
    out = ctypes.c_uint32()
    check(lib().kl_mma_instr_desc(a_type, b_type, acc_type, m, n, ctypes.byref(out)))
    return out.value


def make_tma_desc(dtype, tile_rows, tile_cols, span, ptr, shape, stride, is_store=False) -> bytes:
    """128-byte tensor map (needs a CUDA driver)."""
    rank = len(shape)
    sh = (ctypes.c_int64 * rank)(*shape)
    st = (ctypes.c_int64 * rank)(*stride)
    buf = ctypes.create_string_buffer(128)
    check(lib().kl_make_tma_desc(dtype, tile_rows, tile_cols, span, int(is_store), ctypes.c_void_p(ptr), rank, sh, st, buf))
    return buf.raw


# ------------------------------------------------------------------------------------- GEMM

_TORCH_DTYPES = None


def _dtype_code(t) -> int:
    import torch

    global _TORCH_DTYPES
    if _TORCH_DTYPES is None:
        _TORCH_DTYPES = {torch.bfloat16: KL_BF16, torch.float16: KL_F16, torch.float8_e4m3fn: KL_E4M3,
                         torch.float8_e5m2: KL_E5M2, torch.float32: KL_F32, torch.int8: KL_I8,
                         torch.uint8: KL_U8, torch.int32: KL_I32, torch.float4_e2m1fn_x2: KL_E2M1}
    return _TORCH_DTYPES[t]


def _operand_type(x, ab_type) -> int:
    """kl_dtype of an A / B tensor: from its torch dtype, or `ab_type` (KL_E3M2 / KL_E2M3, or
    "e3m2" / "e2m3") for packed fp6, which torch has no dtype for and which travels as uint8."""
    import torch

    if ab_type is None:
        return _dtype_code(x.dtype)
    if isinstance(ab_type, str) and ab_type not in FP6_TYPES:
        raise ValueError(f"ab_type {ab_type!r}: packed fp6 is 'e3m2' or 'e2m3'")
    code = FP6_TYPES[ab_type] if isinstance(ab_type, str) else int(ab_type)
    if code not in (KL_E3M2, KL_E2M3) or x.dtype != torch.uint8:
        raise ValueError("ab_type names packed fp6 (KL_E3M2 / KL_E2M3) on uint8 tensors")
    return code


def _elements(code: int, units: int) -> int:
    """Elements in `units` storage units: two per byte for packed fp4, four per three bytes for
    packed fp6, else one."""
    if code == KL_E2M1:
        return 2 * units
    if code in (KL_E3M2, KL_E2M3):
        if units % 3:
            raise ValueError("packed fp6 extents and strides are whole groups of 3 bytes (4 elements)")
        return units // 3 * 4
    return units


def gemm_desc(a, b, c, alpha=1.0, scale_a=None, scale_b=None, algo=ALGO_AUTO, group_m=0, max_ctas=0,
              variant=0, prefetch=0, a_major=0, b_major=0, c_reduce=0, swizzle=0, sfa=None, sfb=None,
              scale_vec=32, ab_type=None, stream_k=0, overlap=0) -> GemmDesc:
    """Descriptor for C = alpha * A . B^T on torch CUDA tensors: A [M,K], B [N,K], C [M,N], or the
    batched forms A [L,M,K], B [L,N,K], C [L,M,N] (L independent GEMMs). a_major / b_major = 1
    pass the operand MN-major: `a` as the stored [K, M] (A transposed in memory), `b` as [K, N].
    c_reduce = 1 adds the result into C instead of overwriting it; swizzle picks the operand
    swizzle span in bytes (0 = 128, 64, 32). sfa / sfb (uint8 device tensors in the blocked layout of
    pack_block_scales) make it a block-scaled GEMM: one UE8M0 scale per 32 K-elements of each row
    (MX, scale_vec 32) or one UE4M3 scale per 16 (NVFP4, scale_vec 16, fp4 operands). ab_type =
    KL_E3M2 / KL_E2M3 passes uint8 `a` / `b` as packed fp6 ([rows, 3 K / 4] bytes). stream_k: the
    tile kernels' split tail (the last wave's tiles cut into K-ranges), 0 = where the last wave
    would leave workers idle, 1 = always, -1 = never. overlap: programmatic dependent launch (the
    kernel's prologue overlaps the end of the kernel before it on the stream), 0 = library default
    (on), 1 = on, -1 = off."""
    for name, t in (("a", a), ("b", b), ("c", c)):
        if t.dim() not in (2, 3) or t.stride(-1) != 1:
            raise ValueError(f"{name} must be a 2-D or 3-D tensor with a contiguous last dimension")
    if not a.dim() == b.dim() == c.dim():
        raise ValueError("a, b and c must all be 2-D or all 3-D")
    # Packed fp4 (torch.float4_e2m1fn_x2) holds two elements per storage unit, packed fp6 four per
    # three bytes: the descriptor counts elements, so K, the pitches and the batch strides of A and B
    # are converted.
    ta, tb = _operand_type(a, ab_type), _operand_type(b, ab_type)
    if {ta, tb} & {KL_E2M1, KL_E3M2, KL_E2M3} and (a_major or b_major):
        raise ValueError("packed fp4 / fp6 operands are K-major")
    m, k = (a.shape[-1], a.shape[-2]) if a_major else (a.shape[-2], _elements(ta, a.shape[-1]))
    n, kb = (b.shape[-1], b.shape[-2]) if b_major else (b.shape[-2], _elements(tb, b.shape[-1]))
    batch = a.shape[0] if a.dim() == 3 else 0
    if kb != k or tuple(c.shape[-2:]) != (m, n) or (a.dim() == 3 and not (b.shape[0] == c.shape[0] == batch)):
        raise ValueError(f"shape mismatch: a {tuple(a.shape)}, b {tuple(b.shape)}, c {tuple(c.shape)}")
    bs = (_elements(ta, a.stride(0)), _elements(tb, b.stride(0)), c.stride(0)) if a.dim() == 3 else (0, 0, 0)
    return GemmDesc(m=m, n=n, k=k, a=a.data_ptr(), lda=_elements(ta, a.stride(-2)), b=b.data_ptr(),
                    ldb=_elements(tb, b.stride(-2)), c=c.data_ptr(), ldc=c.stride(-2), ab_type=ta,
                    c_type=_dtype_code(c.dtype),
                    alpha=float(alpha), scale_a=None if scale_a is None else scale_a.data_ptr(),
                    scale_b=None if scale_b is None else scale_b.data_ptr(), algo=algo, group_m=group_m,
                    max_ctas=max_ctas, variant=variant, prefetch=prefetch, batch=batch, stride_a=bs[0],
                    stride_b=bs[1], stride_c=bs[2], a_major=a_major, b_major=b_major, c_reduce=int(c_reduce),
                    swizzle=swizzle,
                    block_scale=0 if sfa is None and sfb is None else (2 if scale_vec == 16 else 1),
                    stream_k=int(stream_k), launch_overlap=int(overlap),
                    sfa=None if sfa is None else sfa.data_ptr(), sfb=None if sfb is None else sfb.data_ptr())


def gemm(a, b, out=None, *, out_dtype=None, alpha=1.0, scale_a=None, scale_b=None, algo=ALGO_AUTO,
         group_m=0, max_ctas=0, variant=0, prefetch=0, a_major=0, b_major=0, accumulate=False, swizzle=0,
         sfa=None, sfb=None, scale_vec=32, ab_type=None, stream_k=0, overlap=0, workspace=None, stream=None):
    """out = alpha * a @ b.T [* scale_a * scale_b] on the current CUDA stream, via kl_gemm.
    accumulate=True: out += alpha * a @ b.T (out must be given). sfa/sfb: block scales (see
    pack_block_scales). ab_type="e3m2" / "e2m3": a and b are uint8 packed fp6."""
    import torch

    if accumulate and out is None:
        raise ValueError("accumulate=True adds into `out`, which must be given")
    if out is None:
        m = a.shape[-1] if a_major else a.shape[-2]
        n = b.shape[-1] if b_major else b.shape[-2]
        shape = (a.shape[0], m, n) if a.dim() == 3 else (m, n)
        out = torch.empty(shape, dtype=out_dtype or torch.bfloat16, device=a.device)
    d = gemm_desc(a, b, out, alpha, scale_a, scale_b, algo, group_m, max_ctas, variant, prefetch, a_major, b_major,
                  int(bool(accumulate)), swizzle, sfa, sfb, scale_vec, ab_type, stream_k, overlap)
    s = stream if stream is not None else torch.cuda.current_stream(a.device).cuda_stream
    if workspace is None:
        check(lib().kl_gemm(ctypes.byref(d), ctypes.c_void_p(s)))
    else:
        check(lib().kl_gemm_ws(ctypes.byref(d), ctypes.c_void_p(workspace.data_ptr()), workspace.numel() *
                               workspace.element_size(), ctypes.c_void_p(s)))
    return out


def gemm_launcher(a, b, out, *, stream=None, **kw):
    """A zero-argument callable that queues out = a @ b.T (the options of `gemm`) with a descriptor
    built once: each call is one kl_gemm through the C ABI, for loops where the launch itself must
    cost the host as little as possible (short decode-shaped GEMMs). The tensors must stay alive and
    in place while the callable is used."""
    import torch

    accumulate = kw.pop("accumulate", False)
    d = gemm_desc(a, b, out, c_reduce=int(bool(accumulate)), **kw)
    s = ctypes.c_void_p(stream if stream is not None else torch.cuda.current_stream(a.device).cuda_stream)
    ref = ctypes.byref(d)
    fn = lib().kl_gemm

    def launch():
        st = fn(ref, s)
        if st != KL_OK:
            check(st)

    launch.desc = d  # keeps the descriptor alive with the callable
    return launch


def block_scale_bytes(rows: int, k: int, vec: int = 32) -> int:
    """Bytes of the blocked scale array for `rows` rows of `k` K-elements, one scale per `vec`."""
    return int(lib().kl_block_scale_bytes(int(rows), int(k), int(vec)))


def gemm_grouped(a, b, m_block_group, out=None, *, out_dtype=None, alpha=1.0, scale_a=None, scale_b=None,
                 accumulate=False, algo=ALGO_1CTA, sfa=None, sfb=None, scale_vec=32, ab_type=None, stream_k=0,
                 stream=None):
    """m-grouped GEMM (mixture-of-experts layout): a [M, K] holds the groups' rows back to back,
    each group padded to a multiple of 128 rows; b [G, N, K] holds one matrix per group;
    m_block_group is an int32 device tensor of ceil(M / 128) entries naming the group of every
    128-row block (-1 = padding). out[rows of block i] = a[rows] @ b[m_block_group[i]].T.
    algo=ALGO_2CTA runs the CTA-pair kernel, which needs the groups padded to 256 rows. Block
    scaling: sfa = A's blocked scales, sfb = the groups' blocked scales concatenated."""
    import torch

    if b.dim() != 3 or a.dim() != 2 or b.shape[2] != a.shape[1]:
        raise ValueError("a must be [M, K] and b [G, N, K]")
    if m_block_group.dtype != torch.int32 or m_block_group.numel() < -(-a.shape[0] // 128):
        raise ValueError("m_block_group must be int32 with ceil(M / 128) entries")
    if accumulate and out is None:
        raise ValueError("accumulate=True adds into `out`, which must be given")
    if out is None:
        out = torch.empty((a.shape[0], b.shape[1]), dtype=out_dtype or torch.bfloat16, device=a.device)
    d = gemm_desc(a, b[0], out, alpha, scale_a, scale_b, algo, c_reduce=int(bool(accumulate)), sfa=sfa, sfb=sfb,
                  scale_vec=scale_vec, ab_type=ab_type, stream_k=stream_k)
    d.groups = b.shape[0]
    d.stride_b = _elements(_operand_type(b, ab_type), b.stride(0))
    d.m_block_group = m_block_group.data_ptr()
    s = stream if stream is not None else torch.cuda.current_stream(a.device).cuda_stream
    check(lib().kl_gemm(ctypes.byref(d), ctypes.c_void_p(s)))
    return out


def mx_scale_bytes(rows: int, k: int) -> int:
    return block_scale_bytes(rows, k, 32)


def pack_block_scales(scales, k: int, vec: int = 32, out=None, stream=None):
    """Repack row-major scales (uint8 device tensor [rows, ceil(k/vec)], unit stride in its last
    dimension) into the blocked layout the block-scaled GEMMs read; returns the uint8 tensor."""
    import torch

    rows = scales.shape[0]
    if scales.dtype != torch.uint8 or scales.dim() != 2 or scales.stride(1) != 1:
        raise ValueError("scales must be a 2-D uint8 tensor with a contiguous last dimension")
    if out is None:
        out = torch.empty(block_scale_bytes(rows, k, vec), dtype=torch.uint8, device=scales.device)
    s = stream if stream is not None else torch.cuda.current_stream(scales.device).cuda_stream
    check(lib().kl_pack_block_scales(ctypes.c_void_p(scales.data_ptr()), rows, int(k), int(vec), scales.stride(0),
                                     ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(s)))
    return out


def mx_quantize(x, kind: str = "e4m3", stream=None):
    """MX-quantise x (fp32 or bf16 device tensor [rows, K], K a multiple of 32) on the device:
    returns (q, scales) with q float8_e4m3fn [rows, K], float4_e2m1fn_x2 [rows, K/2], or for
    kind "e3m2" / "e2m3" uint8 packed fp6 [rows, 3 K / 4] (K a multiple of 128), and scales the
    blocked UE8M0 array, ready for gemm(..., sfa=scales) (with ab_type=kind for fp6)."""
    import torch

    rows, k = x.shape
    if x.stride(1) != 1:
        raise ValueError("x must have a contiguous last dimension")
    kinds = {"e4m3": KL_E4M3, "e2m1": KL_E2M1, **FP6_TYPES}
    if kind not in kinds:
        raise ValueError(f"MX element format {kind!r}: one of {sorted(kinds)}")
    code = kinds[kind]
    if code in (KL_E3M2, KL_E2M3) and k % 128:
        raise ValueError("packed fp6 rows are whole 128-element (96-byte) blocks")
    width = k // 2 if code == KL_E2M1 else k // 4 * 3 if code in (KL_E3M2, KL_E2M3) else k
    q = torch.empty((rows, width), dtype=torch.uint8, device=x.device)
    sc = torch.empty(block_scale_bytes(rows, k, 32), dtype=torch.uint8, device=x.device)
    s = stream if stream is not None else torch.cuda.current_stream(x.device).cuda_stream
    check(lib().kl_mx_quantize(ctypes.c_void_p(x.data_ptr()), _dtype_code(x.dtype), rows, k, x.stride(0),
                               code, ctypes.c_void_p(q.data_ptr()), k, ctypes.c_void_p(sc.data_ptr()),
                               ctypes.c_void_p(s)))
    if code == KL_E2M1:
        return q.view(torch.float4_e2m1fn_x2), sc
    return (q, sc) if code != KL_E4M3 else (q.view(torch.float8_e4m3fn), sc)


def nv_quantize(x, stream=None):
    """NVFP4-quantise x (fp32 or bf16 device tensor [rows, K], K a multiple of 16) on the device:
    returns (q float4_e2m1fn_x2 [rows, K/2], blocked UE4M3 scales per 16 elements, g) with g the
    per-tensor fp32 scale as a one-element device tensor, ready for gemm(..., sfa=scales,
    scale_a=g, scale_vec=16)."""
    import torch

    rows, k = x.shape
    if x.stride(1) != 1:
        raise ValueError("x must have a contiguous last dimension")
    ldq = -(-k // 32) * 32
    q = torch.empty((rows, ldq // 2), dtype=torch.uint8, device=x.device)
    sc = torch.empty(block_scale_bytes(rows, k, 16), dtype=torch.uint8, device=x.device)
    g = torch.empty(1, dtype=torch.float32, device=x.device)
    s = stream if stream is not None else torch.cuda.current_stream(x.device).cuda_stream
    check(lib().kl_nv_quantize(ctypes.c_void_p(x.data_ptr()), _dtype_code(x.dtype), rows, k, x.stride(0),
                               ctypes.c_void_p(q.data_ptr()), ldq, ctypes.c_void_p(sc.data_ptr()),
                               ctypes.c_void_p(g.data_ptr()), ctypes.c_void_p(s)))
    return q[:, :k // 2].view(torch.float4_e2m1fn_x2), sc, g


def mx_pack_scales(scales, k: int, out=None, stream=None):
    """pack_block_scales for MX (UE8M0 scales per 32 elements)."""
    return pack_block_scales(scales, k, 32, out, stream)


def gemm_host(a_host, b_host, c_host, a_dev, b_dev, c_dev, *, alpha=1.0, scale_a=None, scale_b=None,
              algo=ALGO_AUTO, chunks=0, sfa=None, sfb=None, scale_vec=32, ab_type=None, stream_k=0, stream=None):
    """c_host = alpha * a_host @ b_host.T with host (ideally pinned) tensors, through kl_gemm_host:
    the copies in and out overlap the GEMM. a_dev/b_dev/c_dev are device staging tensors of the
    same shapes; sfa/sfb: host MXFP8 scales in the blocked layout (staged by the library). Only
    queues the work on the stream: synchronise it before reading c_host."""
    import torch

    d = gemm_desc(a_host, b_host, c_host, alpha, scale_a, scale_b, algo, sfa=sfa, sfb=sfb, scale_vec=scale_vec,
                  ab_type=ab_type, stream_k=stream_k)
    s = stream if stream is not None else torch.cuda.current_stream(a_dev.device).cuda_stream
    check(lib().kl_gemm_host(ctypes.byref(d), ctypes.c_void_p(a_dev.data_ptr()), ctypes.c_void_p(b_dev.data_ptr()),
                             ctypes.c_void_p(c_dev.data_ptr()), int(chunks), ctypes.c_void_p(s)))
    return c_host


def gemm_host_b(a_dev, b_host, c_host, b_dev, c_dev, *, a_ready=None, alpha=1.0, scale_a=None, scale_b=None,
                algo=ALGO_AUTO, chunks=0, sfa=None, sfb=None, scale_vec=32, ab_type=None, stream_k=0, stream=None):
    """c_host = alpha * a_dev @ b_host.T with A already on the device and B, C in host memory, through
    kl_gemm_host_b: B streams in over b_dev in column blocks while the GEMMs (which also wait for the
    recorded torch.cuda.Event `a_ready`, if given) and the copies of C back to c_host follow. sfa is
    then A's device-side blocked scales, sfb B's host-side ones. Queues the work only."""
    import torch

    d = gemm_desc(a_dev, b_host, c_host, alpha, scale_a, scale_b, algo, sfa=sfa, sfb=sfb, scale_vec=scale_vec,
                  ab_type=ab_type, stream_k=stream_k)
    s = stream if stream is not None else torch.cuda.current_stream(a_dev.device).cuda_stream
    ev = ctypes.c_void_p(a_ready.cuda_event) if a_ready is not None else None
    check(lib().kl_gemm_host_b(ctypes.byref(d), ev, ctypes.c_void_p(b_dev.data_ptr()),
                               ctypes.c_void_p(c_dev.data_ptr()), int(chunks), ctypes.c_void_p(s)))
    return c_host


def gemm_gather(a, b, c_shard, peer_ptrs, *, alpha=1.0, scale_a=None, scale_b=None, algo=ALGO_AUTO,
                group_m=0, max_ctas=0, sfa=None, sfb=None, scale_vec=32, ab_type=None, stream_k=0, stream=None):
    """c_shard = alpha * a @ b.T, and the same tiles written to each peer pointer (a view of the same
    columns in another GPU's copy of C, with c_shard's pitch), through kl_gemm_gather."""
    import torch

    d = gemm_desc(a, b, c_shard, alpha, scale_a, scale_b, algo, group_m, max_ctas, sfa=sfa, sfb=sfb,
                  scale_vec=scale_vec, ab_type=ab_type, stream_k=stream_k)
    arr = (ctypes.c_void_p * max(1, len(peer_ptrs)))(*[ctypes.c_void_p(p) for p in peer_ptrs])
    s = stream if stream is not None else torch.cuda.current_stream(a.device).cuda_stream
    check(lib().kl_gemm_gather(ctypes.byref(d), arr, len(peer_ptrs), ctypes.c_void_p(s)))
    return c_shard


def gemm_gather_multicast(a, b, c_shard, mc_ptr, *, alpha=1.0, scale_a=None, scale_b=None, algo=ALGO_AUTO,
                          group_m=0, max_ctas=0, sfa=None, sfb=None, scale_vec=32, ab_type=None, stream_k=0,
                          stream=None):
    """c_shard = alpha * a @ b.T written once through `mc_ptr`, the NVLink multicast address of
    c_shard's first element (kl_gemm_gather_multicast): every GPU bound to the multicast object gets
    the tiles in its copy of C, this one's included."""
    import torch

    d = gemm_desc(a, b, c_shard, alpha, scale_a, scale_b, algo, group_m, max_ctas, sfa=sfa, sfb=sfb,
                  scale_vec=scale_vec, ab_type=ab_type, stream_k=stream_k)
    s = stream if stream is not None else torch.cuda.current_stream(a.device).cuda_stream
    check(lib().kl_gemm_gather_multicast(ctypes.byref(d), ctypes.c_void_p(mc_ptr), ctypes.c_void_p(s)))
    return c_shard


def ipc_handle(ptr: int) -> tuple[bytes, int]:
    """(64-byte IPC handle of the allocation containing ptr, ptr's byte offset in it)."""
    buf = ctypes.create_string_buffer(64)
    off = ctypes.c_int64()
    check(lib().kl_ipc_get_handle(ctypes.c_void_p(ptr), buf, ctypes.byref(off)))
    return buf.raw, off.value


def ipc_open(handle: bytes) -> int:
    """Map another process's allocation; returns its base address in this process."""
    out = ctypes.c_void_p()
    raw = ctypes.create_string_buffer(handle, 64)
    check(lib().kl_ipc_open_handle(raw, ctypes.byref(out)))
    return out.value


def ipc_close(ptr: int) -> None:
    check(lib().kl_ipc_close(ctypes.c_void_p(ptr)))


def clock_probe(a, b, c, **kw) -> dict:
    """Run one tile-kernel GEMM with per-CTA clock64/%globaltimer stamps; return the SM clock it ran at."""
    import torch

    d = gemm_desc(a, b, c, **kw)
    buf = (ctypes.c_uint64 * (4 * 4096))()
    ctas = ctypes.c_int32()
    s = torch.cuda.current_stream(a.device).cuda_stream
    check(lib().kl_gemm_clock_probe(ctypes.byref(d), buf, 4 * 4096, ctypes.byref(ctas), ctypes.c_void_p(s)))
    mhz, us = [], []
    for i in range(ctas.value):
        cyc, ns = buf[4 * i + 2] - buf[4 * i], buf[4 * i + 3] - buf[4 * i + 1]
        if ns > 0:
            mhz.append(cyc / ns * 1e3)
            us.append(ns / 1e3)
    mhz.sort()
    return {"ctas": ctas.value, "sm_mhz_median": mhz[len(mhz) // 2] if mhz else None,
            "sm_mhz_min": mhz[0] if mhz else None, "sm_mhz_max": mhz[-1] if mhz else None,
            "cta_us_max": max(us) if us else None}


def resolve_algo(a, b, c, **kw) -> int:
    """The kernel family kl_gemm runs for these operands and options (ALGO_1CTA, ALGO_2CTA or
    ALGO_SKINNY), through kl_gemm_resolve_algo; nothing is launched."""
    d = gemm_desc(a, b, c, **kw)
    out = ctypes.c_int32()
    check(lib().kl_gemm_resolve_algo(ctypes.byref(d), ctypes.byref(out)))
    return out.value


def resolve_tile(a, b, c, **kw) -> tuple:
    """(rows, columns) of the C tile kl_gemm runs for these operands and options, through
    kl_gemm_resolve_tile ((0, 0) for the stream-K skinny kernel); nothing is launched."""
    d = gemm_desc(a, b, c, **kw)
    tm, tn = ctypes.c_int32(), ctypes.c_int32()
    check(lib().kl_gemm_resolve_tile(ctypes.byref(d), ctypes.byref(tm), ctypes.byref(tn)))
    return tm.value, tn.value


def workspace_size(a, b, c, **kw) -> int:
    d = gemm_desc(a, b, c, **kw)
    n = ctypes.c_size_t()
    check(lib().kl_gemm_workspace_size(ctypes.byref(d), ctypes.byref(n)))
    return n.value


def release_workspaces() -> None:
    """Free the library's own workspaces (kl_release_workspaces): nothing that uses them may still
    run or be replayed from a captured graph."""
    check(lib().kl_release_workspaces())


def read_status(clear=True) -> int:
    """Synchronise and return the device status bits (raises KlError on a recorded timeout)."""
    bits = ctypes.c_int32()
    st = lib().kl_read_status(ctypes.byref(bits), int(clear))
    if st not in (KL_OK, KL_ERR_TIMEOUT):
        check(st)
    return bits.value


def set_wait_timeout_ns(ns: int) -> None:
    lib().kl_set_wait_timeout_ns(int(ns))


def probe_wait_timeout(timeout_ns: int, stream=None) -> None:
    import torch

    s = stream if stream is not None else torch.cuda.current_stream().cuda_stream
    check(lib().kl_probe_wait_timeout(int(timeout_ns), ctypes.c_void_p(s)))
