"""Element-level restatement of Lava.jl's cooperative-matrix vocabulary — TEST INFRASTRUCTURE
(see ``oracle/__init__.py``: parity unpinned; used only by tests and the CPU baseline).

Each function follows the cited Lava.jl source; matrices here are numpy arrays indexed
[row, col] (zero-based), memory is a flat numpy array of elements.
"""
from __future__ import annotations

import numpy as np

# Clamp modes (src/vocabulary/tensor.jl:46-51).
TENSOR_CLAMP_UNDEFINED = 0
TENSOR_CLAMP_CONSTANT = 1
TENSOR_CLAMP_TO_EDGE = 2

# CoopMatReduce masks (src/vocabulary/coopmat.jl:292-297).
REDUCE_ROW = 1
REDUCE_COLUMN = 2
REDUCE_ROW_AND_COLUMN = 3


def dot4x8(a: int, b: int) -> int:
    """Signed int8×4 dot product of packed words, exact in 32 bits
    (src/vocabulary/vocabulary.jl:31-35: byte i of a times byte i of b, each byte
    reinterpreted as Int8)."""
    def byte(x, i):
        v = (x >> (8 * i)) & 0xFF
        return v - 256 if v >= 128 else v
    return sum(byte(a, i) * byte(b, i) for i in range(4))


def tensor_clampbits(x, T: str) -> int:
    """Operand of tensor_setclampvalue: the bits of x in T, zero-extended to Int32
    (src/vocabulary/tensor.jl:83-85)."""
    if T == "Float16":
        return int(np.array([x], dtype=np.float16).view(np.uint16)[0])
    if T == "Float32":
        return int(np.array([x], dtype=np.float32).view(np.int32)[0])
    return int(x)


def coopmat_load(mem: np.ndarray, offset: int, stride: int, M: int, N: int,
                 rowmajor: bool = False) -> np.ndarray:
    """AcceleratedMatrix{T,M,N,U}(src, offset, stride[, Val(true)]): element (r, c) of the
    M×N tile is read at 1-based ``offset`` + c*stride + r (column-major) or
    + r*stride + c (row-major) (src/device/coopmat_intrinsics.jl:57-75 — base address
    ``ptr + (offset-1)*sizeof``; src/compiler/spirv/coopmat.jl:673-677)."""
    base = offset - 1
    r = np.arange(M)[:, None]
    c = np.arange(N)[None, :]
    idx = base + (r * stride + c if rowmajor else c * stride + r)
    return mem[idx].copy()


def coopmat_store(mem: np.ndarray, offset: int, stride: int, tile: np.ndarray,
                  rowmajor: bool = False) -> None:
    """copyto!(dst, offset, stride, m[, Val(true)]) — the mirror of coopmat_load
    (src/vocabulary/coopmat.jl:150-161; src/device/coopmat_intrinsics.jl:179-218)."""
    M, N = tile.shape
    base = offset - 1
    r = np.arange(M)[:, None]
    c = np.arange(N)[None, :]
    idx = base + (r * stride + c if rowmajor else c * stride + r)
    mem[idx] = tile


def tensor_load_clamped(mat: np.ndarray, r0: int, c0: int, M: int, N: int,
                        clamp: int = TENSOR_CLAMP_CONSTANT, value=0) -> np.ndarray:
    """tensor_load through a sliced layout: rows r0..r0+M-1, cols c0..c0+N-1 of ``mat``;
    outside the tensor, CONSTANT reads ``value`` and TO_EDGE the nearest element
    (src/vocabulary/tensor.jl:46-51,59-108; src/device/tensor_intrinsics.jl:138-171)."""
    R, Cn = mat.shape
    out = np.empty((M, N), dtype=mat.dtype)
    for i in range(M):
        for j in range(N):
            r, c = r0 + i, c0 + j
            if 0 <= r < R and 0 <= c < Cn:
                out[i, j] = mat[r, c]
            elif clamp == TENSOR_CLAMP_TO_EDGE:
                out[i, j] = mat[min(max(r, 0), R - 1), min(max(c, 0), Cn - 1)]
            else:
                out[i, j] = value
    return out


def tensor_store_clamped(mat: np.ndarray, r0: int, c0: int, tile: np.ndarray) -> None:
    """tensor_store through a sliced layout: elements outside the tensor are dropped
    (src/device/tensor_intrinsics.jl:329-402)."""
    R, Cn = mat.shape
    M, N = tile.shape
    r1, c1 = min(R, r0 + M), min(Cn, c0 + N)
    if r1 > r0 and c1 > c0:
        mat[r0:r1, c0:c1] = tile[: r1 - r0, : c1 - c0]


def coopmat_muladd(a: np.ndarray, b: np.ndarray, c: np.ndarray) -> np.ndarray:
    """muladd(a, b, c) = a*b + c accumulated in c's element type; integer operands keep
    their signedness (src/vocabulary/coopmat.jl:190-203; src/compiler/spirv/coopmat.jl:
    112-151 — Int8 operands carry the Signed-components flags, UInt8 do not)."""
    if np.issubdtype(c.dtype, np.integer):
        acc = a.astype(np.int64) @ b.astype(np.int64) + c.astype(np.int64)
        info = np.iinfo(c.dtype)
        # The hardware wraps; every case the tests use stays in range, and this checks it.
        assert acc.min() >= info.min and acc.max() <= info.max, "accumulator overflow"
        return acc.astype(c.dtype)
    return (a.astype(np.float64) @ b.astype(np.float64) + c.astype(np.float64)).astype(c.dtype)


def coopmat_add(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """coopmat_add(a, b): component-wise OpFAdd of two matrices of one type, in that type
    (src/device/coopmat_intrinsics.jl:435-465). A GEMM starts its accumulator from
    bias + residual with it: the bias loaded at stride 0, the residual at its own stride."""
    assert a.dtype == b.dtype and a.shape == b.shape
    return (a + b).astype(a.dtype)


def coopmat_mul(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """coopmat_mul(a, b): component-wise OpFMul (src/device/coopmat_intrinsics.jl:402-433)."""
    assert a.dtype == b.dtype and a.shape == b.shape
    return (a * b).astype(a.dtype)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 with round-to-nearest-even, as uint16 bits (the rounding OpFConvert
    specifies; src/compiler/spirv/coopmat.jl:783-822)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FC0
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Value of x after RNE rounding to bf16, as float32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(np.asarray(x, dtype=np.float32)))


def coopmat_convert(tile: np.ndarray, T: str) -> np.ndarray:
    """convert(AcceleratedMatrix{T,...}, m): component type change, RNE
    (src/vocabulary/coopmat.jl:178-182; src/device/coopmat_intrinsics.jl:232-247).
    Float64 inputs are first rounded to Float32 (the accumulator type)."""
    x = np.asarray(tile)
    if T == "Float32":
        return x.astype(np.float32)
    if T == "Float16":
        return x.astype(np.float32).astype(np.float16)
    if T == "BFloat16":
        return round_bf16(x.astype(np.float32))
    raise ValueError(T)


def coopmat_perelement(f, tile: np.ndarray, *extras) -> np.ndarray:
    """coopmat_perelement(f, m, extras...): element (r, c) becomes f(r, c, e, extras...),
    r and c zero-based UInt32 (src/device/coopmat_intrinsics.jl:551-593;
    src/vocabulary/coopmat.jl:262-270)."""
    out = np.empty_like(tile)
    M, N = tile.shape
    for r in range(M):
        for c in range(N):
            out[r, c] = f(np.uint32(r), np.uint32(c), tile[r, c], *extras)
    return out


def coopmat_reduce(f, tile: np.ndarray, mask: int, dst_shape=None) -> np.ndarray:
    """coopmat_reduce(f, Dst, m, Val(mask)): combine along the mask's axes with the binary
    combiner f; the result has Dst's shape with the reduced value SMEARED along the reduced
    axis, not a vector (src/device/coopmat_intrinsics.jl:702-730)."""
    M, N = tile.shape
    dM, dN = dst_shape if dst_shape is not None else (M, N)
    def fold(v):
        acc = v[0]
        for x in v[1:]:
            acc = f(acc, x)
        return acc
    if mask == REDUCE_ROW:
        rows = np.array([fold(list(tile[r, :])) for r in range(M)], dtype=tile.dtype)
        return np.repeat(rows[:, None], dN, axis=1)[:dM]
    if mask == REDUCE_COLUMN:
        cols = np.array([fold(list(tile[:, c])) for c in range(N)], dtype=tile.dtype)
        return np.repeat(cols[None, :], dM, axis=0)[:, :dN]
    if mask == REDUCE_ROW_AND_COLUMN:
        v = fold(list(tile.reshape(-1)))
        return np.full((dM, dN), v, dtype=tile.dtype)
    raise ValueError("mask")
