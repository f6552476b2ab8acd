"""Plain-Python restatement of the reference's descriptor encoders. TEST INFRASTRUCTURE ONLY.

Each function follows one reference function (paths inside the govindansriram/maia project) and
is pinned by tests/test_descriptor_oracle.py against tests/golden/ref_host_tables.json (the
reference's own headers compiled against CuTe 4.5.0 and run) and the known answers in the
reference's unit tests (tests/golden/ref_test_known_answers.json).
"""

from __future__ import annotations

SWIZZLE_BITS = {16: 0, 32: 1, 64: 2, 128: 3}
UMMA_LAYOUT = {16: 0, 32: 6, 64: 4, 128: 2}  # SWIZZLE_NONE, 32B, 64B, 128B


def atom_elems(elem_bytes: int, swizzle: int) -> int:
    """Columns per swizzle atom: kernel_lib/include/kl/layout/smem_tile.hpp:61."""
    return swizzle // elem_bytes


def tile_offset(rows: int, cols: int, elem_bytes: int, swizzle: int, r: int, c: int) -> int:
    """Un-swizzled element offset (layout_b): 8-row atoms tiled down the rows first.
    kernel_lib/include/kl/layout/smem_tile.hpp:39-42 (tile_to_shape of smem_atom)."""
    w = atom_elems(elem_bytes, swizzle)
    return (c // w) * (rows * w) + r * w + c % w


def swizzle_byte_address(addr: int, swizzle: int) -> int:
    """Swizzle<B,4,3> on a byte address: bits [4, 4+B) ^= bits [7, 7+B).
    kernel_lib/include/kl/layout/smem_tile.hpp:30-37."""
    b = SWIZZLE_BITS[swizzle]
    mask = (1 << b) - 1
    return addr ^ (((addr >> 7) & mask) << 4)


def physical_offset(rows, cols, elem_bytes, swizzle, r, c) -> int:
    """Element offset of (r, c) through tile.tensor() on a pattern-aligned tile."""
    return swizzle_byte_address(tile_offset(rows, cols, elem_bytes, swizzle, r, c) * elem_bytes, swizzle) // elem_bytes


def tma_box(rows: int, cols: int, elem_bytes: int, swizzle: int) -> dict:
    """kernel_lib/include/kl/layout/tma_desc.hpp:47-74 (TmaBox)."""
    inner = atom_elems(elem_bytes, swizzle)
    outer = min(rows, 256)
    col_boxes, row_boxes = cols // inner, rows // outer
    pos = []
    for i in range(col_boxes * row_boxes):
        r, c = i % row_boxes * outer, i // row_boxes * inner
        pos.append([r, c, tile_offset(rows, cols, elem_bytes, swizzle, r, c) * elem_bytes])
    return {"inner": inner, "outer": outer, "col_boxes": col_boxes, "row_boxes": row_boxes,
            "count": col_boxes * row_boxes, "bytes": inner * outer * elem_bytes, "pos": pos}


def mma_k(elem_bytes: int) -> int:
    """K per dense tcgen05.mma, 32 bytes: kernel_lib/include/kl/layout/umma_desc.hpp:16-17."""
    return 32 // elem_bytes


def block_offset_16B(rows, cols, elem_bytes, swizzle, k_block, row=0) -> int:
    """kernel_lib/include/kl/layout/umma_desc.hpp:22-29."""
    return tile_offset(rows, cols, elem_bytes, swizzle, row, k_block * mma_k(elem_bytes)) * elem_bytes // 16


def umma_smem_desc(rows, cols, elem_bytes, swizzle, k_block=0, row=0, start=0) -> int:
    """kl::umma_desc (kernel_lib/include/kl/layout/umma_desc.hpp:35-47): CuTe's K-major descriptor of
    the first (rows x mma_k) slice, version 1, LBO/SBO from the canonical form, then a 32-bit add of
    block_offset_16B to the low word."""
    lay = UMMA_LAYOUT[swizzle]
    sbo = 8 * swizzle // 16                      # 8 rows of one swizzle span, in 16-byte units
    lbo = rows if swizzle == 16 else 1           # interleave: K-chunk stride = rows * 16 B
    d = ((start >> 4) & 0x3FFF) | (lbo & 0x3FFF) << 16 | (sbo & 0x3FFF) << 32 | 1 << 46 | lay << 61
    lo = ((d & 0xFFFFFFFF) + block_offset_16B(rows, cols, elem_bytes, swizzle, k_block, row)) & 0xFFFFFFFF
    return (d & ~0xFFFFFFFF) | lo


OPERAND_FORMAT = {"f16": 0, "bf16": 1, "tf32": 2, "e4m3": 0, "e5m2": 1, "u8": 0, "i8": 1}
ACCUM_FORMAT = {"f16": 0, "f32": 1, "i32": 2}


def instr_desc(a: str, b: str, acc: str, m: int, n: int, a_major: int = 0, b_major: int = 0) -> int:
    """kernel_lib/include/kl/layout/umma_desc.hpp:51-58 (field layout documented at
    kernel_lib/tests/unit/test_umma_desc.cu:79-90)."""
    return (ACCUM_FORMAT[acc] << 4 | OPERAND_FORMAT[a] << 7 | OPERAND_FORMAT[b] << 10 | a_major << 15 | b_major << 16
            | (n >> 3) << 17 | (m >> 4) << 24)


# Operand format codes of the block-scaled kinds: kind::mxf8f6f4 (e4m3 0, e5m2 1, e2m3 3, e3m2 4) and
# kind::mxf4 / mxf4nvf4 (e2m1 1).
BLOCK_SCALED_FORMAT = {"e4m3": 0, "e5m2": 1, "e2m3": 3, "e3m2": 4, "e2m1": 1}


def instr_desc_block_scaled(a: str, b: str, m: int, n: int, a_sf_id: int = 0, b_sf_id: int = 0,
                            ue4m3: bool = False) -> int:
    """Instruction descriptor of a block-scaled tcgen05.mma (no counterpart in the reference; the
    field layout of CuTe's InstrDescriptorBlockScaled): b_sf_id [4,6), a_fmt [7,10), b_fmt [10,13),
    both operands K-major (bits 15, 16 clear), N >> 3 [17,23), scale format [23] (1 = UE8M0,
    0 = UE4M3), M >> 4 [24,29), a_sf_id [29,31); no accumulator-format field (fp32 always)."""
    return (b_sf_id << 4 | BLOCK_SCALED_FORMAT[a] << 7 | BLOCK_SCALED_FORMAT[b] << 10 | (n >> 3) << 17
            | (0 if ue4m3 else 1) << 23 | (m >> 4) << 24 | a_sf_id << 29)


def tma_encode_args(elem_bytes: int, tile_rows: int, tile_cols: int, swizzle: int, ptr: int, shape, stride):
    """The arguments kl::make_tma_desc hands to cuTensorMapEncodeTiled, or the exception message it
    raises (kernel_lib/include/kl/layout/tma_desc.hpp:114-152)."""
    R = len(shape)
    box = tma_box(tile_rows, tile_cols, elem_bytes, swizzle)
    dims = [shape[R - 1 - i] for i in range(R)]
    boxdim = [box["inner"] if i == 0 else box["outer"] if i == 1 else 1 for i in range(R)]
    strides = [stride[R - 1 - i] * elem_bytes for i in range(1, R)]
    if ptr % 16:
        return "kl::make_tma_desc: global address must be 16-byte aligned"
    if any(s < 1 or s > 1 << 32 for s in shape):
        return "kl::make_tma_desc: extents must be in [1, 2^32]"
    for i in range(R - 1):
        sb = strides[R - 2 - i]
        if stride[i] <= 0 or sb % 16 or sb >= 1 << 40:
            return "kl::make_tma_desc: outer strides must be positive multiples of 16 bytes, below 2^40 bytes"
    if stride[R - 2] < shape[R - 1]:
        return "kl::make_tma_desc: rows overlap: the row stride is smaller than cols"
    return {"rank": R, "dims": dims, "strides": strides, "box": boxdim, "elem_strides": [1] * R,
            "interleave": "NONE", "swizzle": swizzle, "l2_promotion": "L2_128B", "oob_fill": "NONE"}
