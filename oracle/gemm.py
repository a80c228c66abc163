"""GEMM oracle — TEST INFRASTRUCTURE (see ``oracle/__init__.py``; parity unpinned).

Two restatements of Lava's coopmat GEMM:

* ``gemm_tiled`` — the algorithm of ``test/glsl/coopmat2_gemm_regs.comp:53-83``: one
  BM×BN workgroup accumulator per output tile, the k-loop stepping BK, A and B slices read
  through clamp-constant(0) tensor layouts, ``coopMatMulAdd`` into an fp32 (int32)
  accumulator, conversion to the output type, clamped tensor store. Small sizes only.
* ``gemm_ref`` — the same product as one float64 (int64) matmul, rounded once to the output
  type: the value every correct kernel approximates. Used at all sizes.

For fp16/bf16 inputs each product a·b is exact in float64 (11+11 or 8+8 significant bits)
and so are sums of up to 2^(53-22-2·e) such terms of bounded range; the tests use that to
check ``gemm_ref`` bit for bit against exact rational arithmetic on small cases.
"""
from __future__ import annotations

import numpy as np

from .vocab import (coopmat_add, coopmat_convert, coopmat_load, coopmat_muladd, tensor_load_clamped,
                    tensor_store_clamped, round_bf16)

FLOAT_OUT = ("Float32", "Float16", "BFloat16")


def to_float64(x: np.ndarray, T: str) -> np.ndarray:
    """Values of a matrix stored as T (bf16 given as float32 values or uint16 bits)."""
    if T == "BFloat16" and x.dtype == np.uint16:
        from .vocab import bf16_bits_to_f32
        return bf16_bits_to_f32(x).astype(np.float64)
    return np.asarray(x).astype(np.float64)


def gemm_ref(A: np.ndarray, B: np.ndarray, out: str) -> np.ndarray:
    """C = A·B with A (M,K), B (K,N) given as numpy arrays of their stored VALUES
    (float16 / float32-holding-bf16-values / int8 / uint8).

    Floats: float64 accumulation, one RNE rounding to ``out``; returns float32 for
    Float32, float16 for Float16, float32 holding bf16 values for BFloat16.
    Integers: exact int64 accumulation; returns int32 / uint32 and asserts the result fits
    (Lava's integer muladd accumulates in the accumulator's 32-bit type,
    src/compiler/spirv/coopmat.jl:112-151)."""
    if np.issubdtype(A.dtype, np.integer):
        acc = A.astype(np.int64) @ B.astype(np.int64)
        dt = np.int32 if out == "Int32" else np.uint32
        info = np.iinfo(dt)
        assert acc.size == 0 or (acc.min() >= info.min and acc.max() <= info.max), "overflow"
        return acc.astype(dt)
    acc = A.astype(np.float64) @ B.astype(np.float64)
    return coopmat_convert(acc, out)


def gemm_tiled(A: np.ndarray, B: np.ndarray, out: str, BM: int = 128, BN: int = 128,
               BK: int = 64) -> np.ndarray:
    """The workgroup-tile algorithm of coopmat2_gemm_regs.comp (see module doc)."""
    M, K = A.shape
    _, N = B.shape
    integer = np.issubdtype(A.dtype, np.integer)
    if integer:
        acc_dt = np.int32 if out == "Int32" else np.uint32
        res = np.zeros((M, N), dtype=acc_dt)
    else:
        res = np.zeros((M, N), dtype=np.float32 if out != "Float16" else np.float16)
    for ir in range(0, M, BM):
        for ic in range(0, N, BN):
            s = np.zeros((BM, BN), dtype=np.int32 if integer and out == "Int32" else
                         (np.uint32 if integer else np.float32))
            for bk in range(0, K, BK):
                a = tensor_load_clamped(A, ir, bk, BM, BK)
                b = tensor_load_clamped(B, bk, ic, BK, BN)
                s = coopmat_muladd(a, b, s)
            tile = s if integer else coopmat_convert(s, out)
            tensor_store_clamped(res, ir, ic, tile)
    return res


def rel_frobenius(x: np.ndarray, ref: np.ndarray) -> float:
    x = np.asarray(x, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = np.linalg.norm(ref)
    return float(np.linalg.norm(x - ref) / den) if den > 0 else float(np.linalg.norm(x))


def max_abs(x: np.ndarray, ref: np.ndarray) -> float:
    d = np.abs(np.asarray(x, dtype=np.float64) - np.asarray(ref, dtype=np.float64))
    return float(d.max()) if d.size else 0.0


def ulp_distance_f16(x: np.ndarray, ref: np.ndarray) -> int:
    """Max distance in fp16 units-in-the-last-place between two float16 arrays."""
    def key(a):
        u = np.asarray(a, dtype=np.float16).view(np.uint16).astype(np.int32)
        return np.where(u & 0x8000, 0x8000 - u, u)   # monotone integer order
    d = np.abs(key(x) - key(ref))
    return int(d.max()) if d.size else 0


def ulp_distance_bf16(x_vals: np.ndarray, ref_vals: np.ndarray) -> int:
    """Same for bf16 values carried in float32."""
    def key(a):
        u = (np.asarray(a, dtype=np.float32).view(np.uint32) >> 16).astype(np.int32)
        return np.where(u & 0x8000, 0x8000 - u, u)
    d = np.abs(key(x_vals) - key(ref_vals))
    return int(d.max()) if d.size else 0


def sgemm_cpu(A32: np.ndarray, B32: np.ndarray) -> np.ndarray:
    """float32 matmul on the host BLAS (numpy's OpenBLAS) — the stand-in for Lava's
    reference CPU path (host Julia Float32 matmul, also OpenBLAS)."""
    return A32 @ B32


__all__ = ["gemm_ref", "gemm_tiled", "rel_frobenius", "max_abs", "ulp_distance_f16",
           "ulp_distance_bf16", "sgemm_cpu", "round_bf16", "to_float64"]


# ---- fused epilogue ------------------------------------------------------------------
# The per-element functions a GEMM applies to its accumulator with coopmat_perelement (or
# getcomp/setcomp over coopmat_length) before convert + copyto!
# (src/device/coopmat_intrinsics.jl:322-331,551-593), in float64.
def _erf(x: np.ndarray) -> np.ndarray:
    from scipy.special import erf
    return erf(x)


def _silu(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        return x / (1.0 + np.exp(-x))


ACTIVATIONS = {
    None: lambda x: x,
    "relu": lambda x: np.where(x < 0, 0.0, x),
    "gelu": lambda x: 0.5 * x * (1.0 + np.tanh(np.sqrt(2.0 / np.pi) * (x + 0.044715 * x ** 3))),
    "gelu_erf": lambda x: 0.5 * x * (1.0 + _erf(x / np.sqrt(2.0))),
    "silu": _silu,
}
ACTIVATION_SLOPE = {None: 1.0, "relu": 1.0, "gelu": 1.13, "gelu_erf": 1.13, "silu": 1.1}


def epilogue_init(M: int, N: int, bias=None, bias_axis: str = "col", residual=None) -> np.ndarray:
    """The accumulator a fused GEMM starts from: coopmat_add of the bias read at stride 0
    (per row: column-major load, every column reads the same M-vector; per column: row-major
    load) and the residual, both as Float32 accumulator matrices
    (src/device/coopmat_intrinsics.jl:435-447; src/compiler/spirv/coopmat.jl:873-878)."""
    init = np.zeros((M, N), dtype=np.float32)
    if bias is not None:
        b = np.asarray(bias, dtype=np.float32)
        smear = coopmat_load(b, 1, 0, M, N, rowmajor=(bias_axis == "col"))
        init = coopmat_add(init, smear)
    if residual is not None:
        init = coopmat_add(init, np.asarray(residual, dtype=np.float32))
    return init


def gemm_epilogue_ref(A: np.ndarray, B: np.ndarray, out: str, bias=None, bias_axis: str = "col",
                      residual=None, act=None, rounded: bool = True):
    """C = act(A·B + bias + residual): the product in float64 onto the Float32 initial
    accumulator (``epilogue_init``), the activation in float64, one conversion to ``out``
    (or the unrounded float64 value with ``rounded=False``). Bias and residual are given
    as the values of their stored type."""
    M, N = A.shape[0], B.shape[1]
    init = epilogue_init(M, N, bias, bias_axis, residual).astype(np.float64)
    pre = A.astype(np.float64) @ B.astype(np.float64) + init
    val = ACTIVATIONS[act](pre)
    return coopmat_convert(val, out) if rounded else val


# ---- clamped loads over a padded k extent, coopmat_mul and per-element programs ---------
def clamp_pad(X: np.ndarray, k_pad: int, axis: int, mode: str, value, T: str) -> np.ndarray:
    """``X`` (values of type T) extended along ``axis`` (its k axis) to ``k_pad`` entries, as
    a load through a tensor layout with clamp ``mode`` reads past the extent
    (src/vocabulary/tensor.jl:46-51; src/device/tensor_intrinsics.jl:139-148):
    "undefined" -> 0 (this library's choice), "constant" -> ``value`` in T's bits
    (tensor_clampbits, tensor.jl:83-85: rounded to the component type), "edge" -> the nearest
    element inside (index K-1)."""
    K = X.shape[axis]
    extra = k_pad - K
    if extra <= 0:
        return X
    shape = list(X.shape)
    shape[axis] = extra
    if mode == "edge":
        edge = np.take(X, [K - 1], axis=axis)
        pad = np.repeat(edge, extra, axis=axis)
    elif mode == "constant":
        if np.issubdtype(X.dtype, np.integer):
            v = int(value)
        else:
            v = coopmat_convert(np.array([float(value)]), T)[0] if T != "Float32" else float(value)
        pad = np.full(shape, v, dtype=X.dtype)
    else:
        pad = np.zeros(shape, dtype=X.dtype)
    return np.concatenate([X, pad], axis=axis)


def gemm_vocab_ref(A: np.ndarray, B: np.ndarray, out: str, T: str, bias=None,
                   bias_axis: str = "col", residual=None, act=None, mul=None, program=None,
                   extra=None, k_pad=None, a_clamp=("undefined", 0), b_clamp=("undefined", 0),
                   rounded: bool = True):
    """The fused GEMM with every epilogue step, as a Lava kernel would compose them:
    acc = coopmat_add(bias, residual) as the initial accumulator, muladd over the k extent
    (``k_pad`` columns with the clamped reads, float64 here), then coopmat_mul by ``mul``
    (coopmat_intrinsics.jl:402-464), the activation, the per-element ``program`` on fp32
    values with 0-based row/col and the ``extra`` matrix's element (oracle/perelement.py), and
    one conversion to ``out``. Integer pairs: the exact int64 product of the padded operands
    (the clamp modes are their only epilogue)."""
    M, N = A.shape[0], B.shape[1]
    if k_pad is not None and k_pad > A.shape[1]:
        A = clamp_pad(A, k_pad, 1, a_clamp[0], a_clamp[1], T)
        B = clamp_pad(B, k_pad, 0, b_clamp[0], b_clamp[1], T)
    if np.issubdtype(A.dtype, np.integer):
        return gemm_ref(A, B, out)
    init = epilogue_init(M, N, bias, bias_axis, residual).astype(np.float64)
    v = A.astype(np.float64) @ B.astype(np.float64) + init
    if mul is not None:
        v = v * np.asarray(mul, dtype=np.float64)
    v = ACTIVATIONS[act](v)
    if program is not None:
        from .perelement import pe_eval
        rows = np.arange(M)[:, None] * np.ones((1, N), dtype=np.int64)
        cols = np.ones((M, 1), dtype=np.int64) * np.arange(N)[None, :]
        ext = None if extra is None else np.asarray(extra, dtype=np.float32)
        v = pe_eval(program, v.astype(np.float32), rows, cols, ext).astype(np.float64)
    return coopmat_convert(v, out) if rounded else v
