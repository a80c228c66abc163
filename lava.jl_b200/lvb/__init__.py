"""lvb — Python host mirror of the LavaB200 Julia package, over liblvb's C ABI.

The Julia package (``lava.jl_b200/LavaB200``) is the drop-in for Lava.jl users; this module
exposes the same entry points to Python so the parity tests and the benchmark drive the
library exactly the way the Julia host does (``ccall`` ≙ ``ctypes``):

* capability vocabulary — ``MatrixShape``, ``DeviceCaps``, ``caps``, ``matrix_shapes``,
  ``supports``, ``bestshape``, ``wggranularity`` (Lava ``src/vocabulary/matrix.jl:88-172``,
  ``src/vocabulary/caps.jl:54-169``);
* ``gemm(C, A, B)`` — Lava's coopmat GEMM (``gemm!`` in Julia): ``C = A·B`` with the
  accumulation type of ``C``'s pair, layouts read from the tensors' strides (row-major
  ≙ ``Val(true)``, ``src/vocabulary/coopmat.jl:124-161``);
* ``attention(O, Q, K, V; causal, scale)`` — the flash-attention forward (``attention!``);
* ``device_status()`` — the exception-flag check Lava's host does after a sync
  (``src/compiler/entry_wrapper.jl:199-216``).

Errors are raised as ``LavaError(operation, message, suggestion)`` like Lava's
(``src/runtime/errors.jl:4-24``). There is no fallback: if ``liblvb.so`` is missing the
import fails, and a call on a machine without a B200 raises.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass, field
from pathlib import Path
from typing import Optional

_HERE = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("LVB_LIBRARY", _HERE.parent / "lib" / "liblvb.so"))

# ---- status / dtype enums (include/lvb.h) -------------------------------------------
LVB_OK, LVB_ERR_INVALID_ARG, LVB_ERR_UNSUPPORTED, LVB_ERR_CUDA = 0, 1, 2, 3
LVB_ERR_TIMEOUT, LVB_ERR_NCCL, LVB_ERR_NO_DEVICE = 4, 5, 6
F16, BF16, F32, I8, U8, I32, U32 = range(7)
ACT_NONE, ACT_RELU, ACT_GELU_TANH, ACT_GELU_ERF, ACT_SILU = range(5)
CLAMP_UNDEFINED, CLAMP_CONSTANT, CLAMP_TO_EDGE = range(3)
ACTIVATIONS = {None: ACT_NONE, "none": ACT_NONE, "relu": ACT_RELU, "gelu": ACT_GELU_TANH,
               "gelu_tanh": ACT_GELU_TANH, "gelu_erf": ACT_GELU_ERF, "silu": ACT_SILU}
BIAS_PER_ROW, BIAS_PER_COL = 0, 1
SUBGROUP_SCOPE, WORKGROUP_SCOPE = 0, 1
DTYPE_NAMES = {F16: "Float16", BF16: "BFloat16", F32: "Float32", I8: "Int8", U8: "UInt8",
               I32: "Int32", U32: "UInt32"}
DTYPE_SIZES = {F16: 2, BF16: 2, F32: 4, I8: 1, U8: 1, I32: 4, U32: 4}

# Symbols include/lvb.h declares; the CPU tests check the library exports each one.
EXPORTS = [
    "lvb_caps_sm100", "lvb_caps", "lvb_matrix_shapes", "lvb_bestshape",
    "lvb_gemm_check", "lvb_gemm_plan_for", "lvb_gemm", "lvb_gemm_noalloc",
    "lvb_gemm_noalloc_status", "lvb_gemm_noalloc_selftest_wait_timeout",
    "lvb_gemm_ex_check", "lvb_gemm_ex", "lvb_pe_program_check",
    "lvb_attention_check", "lvb_attention_plan_for", "lvb_attention_fwd",
    "lvb_abi_version", "lvb_last_error", "lvb_status_string", "lvb_device_count",
    "lvb_set_device", "lvb_malloc", "lvb_free", "lvb_memcpy_htod", "lvb_memcpy_dtoh",
    "lvb_stream_create", "lvb_stream_destroy", "lvb_stream_synchronize",
    "lvb_device_status", "lvb_set_wait_timeout_ms", "lvb_shard_range",
    "lvb_selftest_wait_timeout",
    "lvb_comm_unique_id", "lvb_comm_init", "lvb_comm_destroy", "lvb_comm_size", "lvb_allgather",
]


class LavaError(RuntimeError):
    """``LavaError(operation, message, suggestion)`` plus the lvb status code."""

    def __init__(self, status: int, text: str):
        self.status = status
        op, _, rest = text.partition(": ")
        msg, _, hint = rest.partition(" (")
        self.operation = op
        self.message = msg
        self.suggestion = hint[:-1] if hint.endswith(")") else hint
        super().__init__(f"[{STATUS_NAMES.get(status, status)}] {text}")


STATUS_NAMES = {0: "LVB_OK", 1: "LVB_ERR_INVALID_ARG", 2: "LVB_ERR_UNSUPPORTED",
                3: "LVB_ERR_CUDA", 4: "LVB_ERR_TIMEOUT", 5: "LVB_ERR_NCCL",
                6: "LVB_ERR_NO_DEVICE"}


# ---- C structs ------------------------------------------------------------------------
class lvb_matrix_shape(C.Structure):
    _fields_ = [("ab", C.c_int32), ("acc", C.c_int32), ("M", C.c_int32), ("N", C.c_int32),
                ("K", C.c_int32), ("scope", C.c_int32)]


class lvb_device_caps(C.Structure):
    _fields_ = [("coopmat", C.c_int32), ("tile", C.c_int32), ("subgroup", C.c_int32),
                ("coopmatsubgroup", C.c_int32), ("sharedbudget", C.c_int64),
                ("workgrouplimit", C.c_int32), ("cores", C.c_int32), ("warps", C.c_int32),
                ("n_wggran", C.c_int32), ("wggran", (C.c_int32 * 4) * 8),
                ("n_shapes", C.c_int32), ("cc_major", C.c_int32), ("cc_minor", C.c_int32)]


class lvb_gemm_desc(C.Structure):
    _fields_ = [("a_type", C.c_int32), ("b_type", C.c_int32), ("c_type", C.c_int32),
                ("a_rowmajor", C.c_int32), ("b_rowmajor", C.c_int32), ("c_rowmajor", C.c_int32),
                ("M", C.c_int64), ("N", C.c_int64), ("K", C.c_int64),
                ("lda", C.c_int64), ("ldb", C.c_int64), ("ldc", C.c_int64)]


class lvb_gemm_plan(C.Structure):
    _fields_ = [("swap_ab", C.c_int32), ("tile_m", C.c_int32), ("tile_n", C.c_int32),
                ("tile_k", C.c_int32), ("stages", C.c_int32), ("tiles", C.c_int32),
                ("ctas", C.c_int32), ("smem_bytes", C.c_int32), ("tmem_cols", C.c_int32),
                ("instr_m", C.c_int32), ("instr_n", C.c_int32), ("instr_k", C.c_int32),
                ("repack_a", C.c_int32), ("repack_b", C.c_int32), ("cta_pair", C.c_int32),
                ("a_mnmajor", C.c_int32), ("b_mnmajor", C.c_int32), ("gemv", C.c_int32),
                ("gemv_ksplit", C.c_int32), ("launches", C.c_int32)]


class lvb_attn_plan(C.Structure):
    _fields_ = [("kernel", C.c_int32), ("splits", C.c_int32), ("ctas", C.c_int32),
                ("launches", C.c_int32)]


class lvb_epilogue(C.Structure):
    _fields_ = [("bias", C.c_void_p), ("residual", C.c_void_p), ("ldr", C.c_int64),
                ("bias_type", C.c_int32), ("bias_axis", C.c_int32),
                ("residual_type", C.c_int32), ("activation", C.c_int32),
                ("mul", C.c_void_p), ("ldm", C.c_int64), ("mul_type", C.c_int32),
                ("extra_type", C.c_int32), ("extra", C.c_void_p), ("lde", C.c_int64),
                ("program", C.c_void_p), ("k_pad", C.c_int64),
                ("a_clamp", C.c_int32), ("b_clamp", C.c_int32),
                ("a_clamp_value", C.c_double), ("b_clamp_value", C.c_double)]


class lvb_attn_desc(C.Structure):
    _fields_ = [("dtype", C.c_int32), ("causal", C.c_int32),
                ("batch", C.c_int64), ("heads_q", C.c_int64), ("heads_kv", C.c_int64),
                ("seq_q", C.c_int64), ("seq_kv", C.c_int64), ("head_dim", C.c_int64),
                ("scale", C.c_float), ("reserved", C.c_int32),
                ("q_stride", C.c_int64 * 3), ("k_stride", C.c_int64 * 3),
                ("v_stride", C.c_int64 * 3), ("o_stride", C.c_int64 * 3)]


class lvb_comm_id(C.Structure):
    _fields_ = [("bytes", C.c_char * 128)]


def _load() -> C.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(f"liblvb.so not built at {LIB_PATH}; run python lava.jl_b200/build.py")
    lib = C.CDLL(str(LIB_PATH))
    P = C.c_void_p
    sig = {
        "lvb_caps_sm100": ([C.POINTER(lvb_device_caps)], C.c_int),
        "lvb_caps": ([C.c_int, C.POINTER(lvb_device_caps)], C.c_int),
        "lvb_matrix_shapes": ([C.POINTER(lvb_matrix_shape), C.c_int32, C.POINTER(C.c_int32)], C.c_int),
        "lvb_bestshape": ([C.c_int32, C.c_int32, C.c_int32, C.POINTER(lvb_matrix_shape)], C.c_int),
        "lvb_gemm_check": ([C.POINTER(lvb_gemm_desc)], C.c_int),
        "lvb_gemm_plan_for": ([C.POINTER(lvb_gemm_desc), C.c_int32, C.POINTER(lvb_gemm_plan)], C.c_int),
        "lvb_gemm": ([C.POINTER(lvb_gemm_desc), P, P, P, P], C.c_int),
        "lvb_gemm_noalloc": ([C.POINTER(lvb_gemm_desc), P, P, P, P], C.c_int),
        "lvb_gemm_noalloc_status": ([P, C.POINTER(C.c_int32), C.POINTER(C.c_int32),
                                     C.POINTER(C.c_int32)], C.c_int),
        "lvb_gemm_noalloc_selftest_wait_timeout": ([C.c_int32, P], C.c_int),
        "lvb_gemm_ex_check": ([C.POINTER(lvb_gemm_desc), C.POINTER(lvb_epilogue)], C.c_int),
        "lvb_pe_program_check": ([P], C.c_int),
        "lvb_gemm_ex": ([C.POINTER(lvb_gemm_desc), C.POINTER(lvb_epilogue), P, P, P, P], C.c_int),
        "lvb_attention_check": ([C.POINTER(lvb_attn_desc)], C.c_int),
        "lvb_attention_fwd": ([C.POINTER(lvb_attn_desc), P, P, P, P, P, P], C.c_int),
        "lvb_attention_plan_for": ([C.POINTER(lvb_attn_desc), C.c_int32, C.POINTER(lvb_attn_plan)], C.c_int),
        "lvb_abi_version": ([], C.c_int),
        "lvb_last_error": ([], C.c_char_p),
        "lvb_status_string": ([C.c_int], C.c_char_p),
        "lvb_device_count": ([C.POINTER(C.c_int32)], C.c_int),
        "lvb_set_device": ([C.c_int], C.c_int),
        "lvb_malloc": ([C.POINTER(P), C.c_size_t], C.c_int),
        "lvb_free": ([P], C.c_int),
        "lvb_memcpy_htod": ([P, P, C.c_size_t, P], C.c_int),
        "lvb_memcpy_dtoh": ([P, P, C.c_size_t, P], C.c_int),
        "lvb_stream_create": ([C.POINTER(P)], C.c_int),
        "lvb_stream_destroy": ([P], C.c_int),
        "lvb_stream_synchronize": ([P], C.c_int),
        "lvb_device_status": ([P, C.POINTER(C.c_int32), C.POINTER(C.c_int32), C.POINTER(C.c_int32)], C.c_int),
        "lvb_set_wait_timeout_ms": ([C.c_int64], C.c_int),
        "lvb_shard_range": ([C.c_int64, C.c_int32, C.c_int32, C.c_int64, C.POINTER(C.c_int64),
                             C.POINTER(C.c_int64)], C.c_int),
        "lvb_selftest_wait_timeout": ([C.c_int32, P], C.c_int),
        "lvb_comm_unique_id": ([C.POINTER(lvb_comm_id)], C.c_int),
        "lvb_comm_init": ([C.POINTER(P), C.POINTER(lvb_comm_id), C.c_int32, C.c_int32], C.c_int),
        "lvb_comm_destroy": ([P], C.c_int),
        "lvb_comm_size": ([P, C.POINTER(C.c_int32), C.POINTER(C.c_int32)], C.c_int),
        "lvb_allgather": ([P, P, P, C.c_size_t, P], C.c_int),
    }
    for name, (args, res) in sig.items():
        f = getattr(lib, name)
        f.argtypes = args
        f.restype = res
    return lib


lib = _load()


def check(status: int) -> None:
    if status != LVB_OK:
        raise LavaError(status, lib.lvb_last_error().decode())


# ---- capability vocabulary ----------------------------------------------------------
@dataclass(frozen=True)
class MatrixShape:
    """One (M, N, K) shape for operands ``ab`` accumulating into ``acc`` (matrix.jl:88-95)."""
    ab: int
    acc: int
    M: int
    N: int
    K: int
    scope: int = SUBGROUP_SCOPE

    def __str__(self):
        sc = "SubgroupScope" if self.scope == SUBGROUP_SCOPE else "WorkgroupScope"
        return (f"MatrixShape({DTYPE_NAMES[self.ab]}->{DTYPE_NAMES[self.acc]} "
                f"{self.M}x{self.N}x{self.K} {sc})")


@dataclass
class DeviceCaps:
    """Lava's DeviceCaps record (caps.jl:54-65) as a B200 answers it."""
    coopmat: bool
    tile: int
    subgroup: int
    coopmatsubgroup: int
    sharedbudget: int
    workgrouplimit: int
    cores: int
    warps: int
    wggran: list = field(default_factory=list)
    shapes: list = field(default_factory=list)


def _shape_table() -> list[MatrixShape]:
    n = C.c_int32()
    check(lib.lvb_matrix_shapes(None, 0, C.byref(n)))
    arr = (lvb_matrix_shape * n.value)()
    check(lib.lvb_matrix_shapes(arr, n.value, C.byref(n)))
    return [MatrixShape(s.ab, s.acc, s.M, s.N, s.K, s.scope) for s in arr]


def _caps_from(c: lvb_device_caps) -> DeviceCaps:
    shapes = [s for s in _shape_table() if s.scope == SUBGROUP_SCOPE]
    wg = [tuple(c.wggran[i]) for i in range(c.n_wggran)]
    return DeviceCaps(bool(c.coopmat), c.tile, c.subgroup, c.coopmatsubgroup, c.sharedbudget,
                      c.workgrouplimit, c.cores, c.warps, wg, shapes)


def caps(device: Optional[int] = None) -> DeviceCaps:
    """``Lava.caps(backend)``: the live device's answer; ``device=None`` gives the static
    sm_100a table (no GPU needed), the form Lava's copy constructor exists for."""
    c = lvb_device_caps()
    if device is None:
        check(lib.lvb_caps_sm100(C.byref(c)))
    else:
        check(lib.lvb_caps(device, C.byref(c)))
    return _caps_from(c)


def matrix_shapes(c: Optional[DeviceCaps] = None, scope: Optional[int] = None) -> list[MatrixShape]:
    """``matrix_shapes(c)``: empty when ``c.coopmat`` is false (caps.jl:158-159). With no
    caps, the whole table including the workgroup-scope (tcgen05 tile) shapes."""
    if c is not None:
        return list(c.shapes) if c.coopmat else []
    t = _shape_table()
    return [s for s in t if scope is None or s.scope == scope]


def supports(shapes_or_caps, s: MatrixShape) -> bool:
    shapes = matrix_shapes(shapes_or_caps) if isinstance(shapes_or_caps, DeviceCaps) else shapes_or_caps
    return any(x == s for x in shapes)


def _isbetter(a: MatrixShape, b: MatrixShape) -> bool:
    sa = abs(a.M - a.N) + abs(a.N - a.K)
    sb = abs(b.M - b.N) + abs(b.N - b.K)
    if sa != sb:
        return sa < sb
    return a.M * a.N * a.K > b.M * b.N * b.K


def bestshape(shapes_or_caps, ab: int, acc: int, scope: int = SUBGROUP_SCOPE) -> Optional[MatrixShape]:
    """Squarest, then largest (matrix.jl:155-172); None where Lava returns ``nothing``."""
    shapes = matrix_shapes(shapes_or_caps) if isinstance(shapes_or_caps, DeviceCaps) else shapes_or_caps
    best = None
    for s in shapes:
        if s.ab != ab or s.acc != acc or s.scope != scope:
            continue
        if best is None or _isbetter(s, best):
            best = s
    return best


def bestshape_native(ab: int, acc: int, scope: int = SUBGROUP_SCOPE) -> Optional[MatrixShape]:
    """The library's own bestshape over its full table (C ABI lvb_bestshape)."""
    out = lvb_matrix_shape()
    st = lib.lvb_bestshape(ab, acc, scope, C.byref(out))
    if st == LVB_ERR_UNSUPPORTED:
        return None
    check(st)
    return MatrixShape(out.ab, out.acc, out.M, out.N, out.K, out.scope)


def wggranularity(c: DeviceCaps, nt: int):
    """(M, N, K) multiples of a workgroup-scope matrix at ``nt`` invocations (caps.jl:140-145)."""
    for (n, m, nn, k) in c.wggran:
        if n == nt:
            return (m, nn, k)
    return None


# ---- tensors -> descriptors -----------------------------------------------------------
def _torch():
    import torch
    return torch


def dtype_of(t) -> int:
    torch = _torch()
    m = {torch.float16: F16, torch.bfloat16: BF16, torch.float32: F32, torch.int8: I8,
         torch.uint8: U8, torch.int32: I32}
    if hasattr(torch, "uint32"):
        m[torch.uint32] = U32
    if t.dtype not in m:
        raise LavaError(LVB_ERR_UNSUPPORTED, f"lvb: no component type for {t.dtype}")
    return m[t.dtype]


def _layout2d(t, name: str):
    """(rowmajor, ld) of a 2-D tensor: row-major when the column stride is 1."""
    if t.dim() != 2:
        raise LavaError(LVB_ERR_INVALID_ARG, f"lvb_gemm: {name} must be 2-D")
    r, c = t.shape
    s0, s1 = t.stride()
    if r == 0 or c == 0:            # an empty operand has no layout to read
        return 1, max(c, 1)
    if s1 == 1 and (r <= 1 or s0 >= max(c, 1)):
        return 1, max(s0, c, 1)
    if s0 == 1 and (c <= 1 or s1 >= max(r, 1)):
        return 0, max(s1, r, 1)
    raise LavaError(LVB_ERR_UNSUPPORTED, f"lvb_gemm: {name} has no unit stride "
                    "(make it contiguous or a transpose of a contiguous tensor)")


def gemm_desc(C_, A, B, c_type: Optional[int] = None) -> lvb_gemm_desc:
    M, K = A.shape
    K2, N = B.shape
    if K2 != K or tuple(C_.shape) != (M, N):
        raise LavaError(LVB_ERR_INVALID_ARG,
                        f"lvb_gemm: shapes {tuple(A.shape)} x {tuple(B.shape)} -> {tuple(C_.shape)}")
    d = lvb_gemm_desc()
    d.a_type, d.b_type = dtype_of(A), dtype_of(B)
    d.c_type = dtype_of(C_) if c_type is None else c_type
    d.a_rowmajor, d.lda = _layout2d(A, "A")
    d.b_rowmajor, d.ldb = _layout2d(B, "B")
    d.c_rowmajor, d.ldc = _layout2d(C_, "C")
    d.M, d.N, d.K = M, N, K
    return d


def _stream_ptr(stream) -> Optional[int]:
    if stream is None:
        torch = _torch()
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def _cmatrix(C_, t, what):
    """(pointer, type, leading dimension) of an M×N epilogue operand read in C's layout (a
    single row or column reads the same in either, whatever strides torch gave it)."""
    if tuple(t.shape) != tuple(C_.shape):
        raise LavaError(LVB_ERR_INVALID_ARG, f"lvb_gemm_ex: {what} must have C's shape")
    crm, _ = _layout2d(C_, "C")
    r, c = t.shape
    s0, s1 = t.stride()
    if crm:
        if c > 1 and s1 != 1:
            raise LavaError(LVB_ERR_UNSUPPORTED, f"lvb_gemm_ex: {what} must have C's layout")
        ld = s0 if r > 1 else max(c, 1)
    else:
        if r > 1 and s0 != 1:
            raise LavaError(LVB_ERR_UNSUPPORTED, f"lvb_gemm_ex: {what} must have C's layout")
        ld = s1 if c > 1 else max(r, 1)
    return t.data_ptr(), dtype_of(t), ld


def _clamp(spec):
    """A clamp given as None / "undefined", "edge", or a number (the constant)."""
    if spec is None or spec == "undefined":
        return CLAMP_UNDEFINED, 0.0
    if spec == "edge":
        return CLAMP_TO_EDGE, 0.0
    if isinstance(spec, (int, float)) and not isinstance(spec, bool):
        return CLAMP_CONSTANT, float(spec)
    raise LavaError(LVB_ERR_INVALID_ARG, f"lvb_gemm_ex: clamp {spec!r}: None, 'edge' or a number")


def epilogue(C_, bias=None, bias_axis: str = "col", residual=None, activation=None, mul=None,
             program=None, extra=None, k_pad=None, a_clamp=None, b_clamp=None) -> lvb_epilogue:
    """The ``lvb_epilogue`` for ``C = f(act((A·B + bias + residual) ⊙ mul))``: ``bias`` a
    contiguous vector added per column (``bias_axis="col"``, N elements) or per row (``"row"``,
    M elements); ``residual`` and ``mul`` M×N tensors in C's layout (the residual may be C
    itself); ``program`` a ``perelement.Program`` (or a Python function, traced) with
    ``extra`` its M×N matrix operand; ``k_pad`` the padded k extent whose reads past K take
    ``a_clamp`` / ``b_clamp`` (None, ``"edge"`` or a constant). The program structure is kept
    alive on the returned value (``e._keep``) for the duration of the call."""
    e = lvb_epilogue()
    if activation not in ACTIVATIONS:
        raise LavaError(LVB_ERR_INVALID_ARG, f"lvb_gemm_ex: unknown activation {activation!r}")
    e.activation = ACTIVATIONS[activation]
    if bias is not None:
        if bias.dim() != 1 or bias.stride(0) != 1:
            raise LavaError(LVB_ERR_INVALID_ARG, "lvb_gemm_ex: bias must be a contiguous vector")
        want = C_.shape[1] if bias_axis == "col" else C_.shape[0]
        if bias.shape[0] != want:
            raise LavaError(LVB_ERR_INVALID_ARG,
                            f"lvb_gemm_ex: bias has {bias.shape[0]} elements, needs {want}")
        e.bias = bias.data_ptr()
        e.bias_type = dtype_of(bias)
        e.bias_axis = BIAS_PER_COL if bias_axis == "col" else BIAS_PER_ROW
    if residual is not None:
        e.residual, e.residual_type, e.ldr = _cmatrix(C_, residual, "residual")
    if mul is not None:
        e.mul, e.mul_type, e.ldm = _cmatrix(C_, mul, "mul")
    e._keep = None
    if program is not None:
        from .perelement import Program, program as trace
        prog = program if isinstance(program, Program) else trace(program)
        st = prog.to_struct()
        e._keep = st
        e.program = C.addressof(st)
        if extra is not None:
            e.extra, e.extra_type, e.lde = _cmatrix(C_, extra, "extra")
    elif extra is not None:
        raise LavaError(LVB_ERR_INVALID_ARG, "lvb_gemm_ex: extra without a program")
    if k_pad is not None:
        e.k_pad = int(k_pad)
        e.a_clamp, e.a_clamp_value = _clamp(a_clamp)
        e.b_clamp, e.b_clamp_value = _clamp(b_clamp)
    return e


def gemm(C_, A, B, stream=None, c_type: Optional[int] = None, bias=None, bias_axis="col",
         residual=None, activation=None, mul=None, program=None, extra=None, k_pad=None,
         a_clamp=None, b_clamp=None):
    """``gemm!(C, A, B)``: C = A·B on the GPU (torch CUDA tensors, logical shapes
    (M,K)·(K,N) -> (M,N)); enqueued on ``stream`` (default: torch's current stream).
    ``c_type`` overrides the component type read from C (e.g. U32 held in an int32
    tensor). With any of the epilogue keywords the fused epilogue runs (``lvb_gemm_ex``, see
    ``epilogue``): C = program(act((A·B + bias + residual) ⊙ mul)), the product over
    ``k_pad`` columns with the clamp modes when given."""
    d = gemm_desc(C_, A, B, c_type)
    if (bias is None and residual is None and activation in (None, "none") and mul is None
            and program is None and k_pad is None):
        check(lib.lvb_gemm(C.byref(d), A.data_ptr(), B.data_ptr(), C_.data_ptr(),
                           _stream_ptr(stream)))
        return C_
    e = epilogue(C_, bias, bias_axis, residual, activation, mul, program, extra, k_pad,
                 a_clamp, b_clamp)
    check(lib.lvb_gemm_ex(C.byref(d), C.byref(e), A.data_ptr(), B.data_ptr(), C_.data_ptr(),
                          _stream_ptr(stream)))
    return C_


class GemmCall:
    """A GEMM validated and described once, launched many times: ``g = prepare_gemm(C, A, B,
    ...)`` then ``g()`` (or ``g(stream)``) enqueues ``lvb_gemm`` / ``lvb_gemm_ex`` with the
    prepared descriptor — one foreign call per launch, for small problems whose time is the
    host's. The tensors must stay alive and keep their storage while the object is used."""

    def __init__(self, C_, A, B, c_type=None, **epi):
        self.d = gemm_desc(C_, A, B, c_type)
        self.ptrs = (A.data_ptr(), B.data_ptr(), C_.data_ptr())
        self.keep = (C_, A, B)
        active = {k: v for k, v in epi.items() if v is not None and v != "none"}
        self.e = epilogue(C_, **epi) if active else None
        self._fn = lib.lvb_gemm if self.e is None else lib.lvb_gemm_ex
        self._d = C.byref(self.d)
        self._args = ((self._d,) if self.e is None else (self._d, C.byref(self.e))) + self.ptrs
        self._default_stream = None

    def __call__(self, stream=None):
        if stream is None:
            if self._default_stream is None:
                self._default_stream = _stream_ptr(None)
            s = self._default_stream
        else:
            s = _stream_ptr(stream)
        st = self._fn(*self._args, s)
        if st:
            check(st)


def prepare_gemm(C_, A, B, c_type=None, **epi) -> GemmCall:
    """See ``GemmCall``; keywords as ``gemm``'s epilogue keywords. The default stream is
    torch's current stream at the first call."""
    return GemmCall(C_, A, B, c_type, **epi)


def gemm_plan(M, N, K, a_type=F16, c_type=F32, c_rowmajor=False, sm_count=148,
              a_rowmajor=True, b_rowmajor=False) -> lvb_gemm_plan:
    lda = max(K if a_rowmajor else M, 1)
    ldb = max(N if b_rowmajor else K, 1)
    d = lvb_gemm_desc(a_type, a_type, c_type, int(a_rowmajor), int(b_rowmajor), int(c_rowmajor),
                      M, N, K, lda, ldb, max(N if c_rowmajor else M, 1))
    p = lvb_gemm_plan()
    check(lib.lvb_gemm_plan_for(C.byref(d), sm_count, C.byref(p)))
    return p


def _strides4(t):
    if t.dim() != 4 or t.stride(3) != 1:
        raise LavaError(LVB_ERR_UNSUPPORTED, "lvb_attention_fwd: tensors are [B][H][S][D] "
                        "with D contiguous")
    return (t.stride(0), t.stride(1), t.stride(2))


def attention_desc(O, Q, K, V, causal=True, scale=None) -> lvb_attn_desc:
    Bq, Hq, Sq, D = Q.shape
    Bk, Hkv, Skv, Dk = K.shape
    if tuple(V.shape) != tuple(K.shape) or Bk != Bq or Dk != D or tuple(O.shape) != tuple(Q.shape):
        raise LavaError(LVB_ERR_INVALID_ARG, "lvb_attention_fwd: shape mismatch")
    d = lvb_attn_desc()
    d.dtype = dtype_of(Q)
    if dtype_of(K) != d.dtype or dtype_of(V) != d.dtype or dtype_of(O) != d.dtype:
        raise LavaError(LVB_ERR_UNSUPPORTED, "lvb_attention_fwd: Q, K, V, O must share a dtype")
    d.causal = int(bool(causal))
    d.batch, d.heads_q, d.heads_kv, d.seq_q, d.seq_kv, d.head_dim = Bq, Hq, Hkv, Sq, Skv, D
    d.scale = float(scale) if scale is not None else float(D) ** -0.5
    for name, t in (("q_stride", Q), ("k_stride", K), ("v_stride", V), ("o_stride", O)):
        s = _strides4(t)
        arr = getattr(d, name)
        for i in range(3):
            arr[i] = s[i]
    return d


def attention(O, Q, K, V, causal=True, scale=None, lse=None, stream=None):
    """``attention!(O, Q, K, V; causal, scale)``: flash-attention forward on the GPU.
    Q/O [B][Hq][Sq][D], K/V [B][Hkv][Skv][D]; optional fp32 ``lse`` [B][Hq][Sq]."""
    d = attention_desc(O, Q, K, V, causal, scale)
    check(lib.lvb_attention_fwd(C.byref(d), Q.data_ptr(), K.data_ptr(), V.data_ptr(),
                                O.data_ptr(), lse.data_ptr() if lse is not None else None,
                                _stream_ptr(stream)))
    return O


class AttentionCall:
    """An attention forward described once, launched many times: ``a = prepare_attention(O,
    Q, K, V, ...)`` then ``a()`` (or ``a(stream)``) — one foreign call per launch. The tensors
    must stay alive and keep their storage while the object is used."""

    def __init__(self, O, Q, K, V, causal=True, scale=None, lse=None):
        self.d = attention_desc(O, Q, K, V, causal, scale)
        self.keep = (O, Q, K, V, lse)
        self._args = (C.byref(self.d), Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(),
                      lse.data_ptr() if lse is not None else None)
        self._default_stream = None

    def __call__(self, stream=None):
        if stream is None:
            if self._default_stream is None:
                self._default_stream = _stream_ptr(None)
            s = self._default_stream
        else:
            s = _stream_ptr(stream)
        st = lib.lvb_attention_fwd(*self._args, s)
        if st:
            check(st)


def prepare_attention(O, Q, K, V, causal=True, scale=None, lse=None) -> AttentionCall:
    """See ``AttentionCall``; arguments as ``attention``'s. The default stream is torch's
    current stream at the first call."""
    return AttentionCall(O, Q, K, V, causal, scale, lse)


ATTN_FLASH, ATTN_DECODE, ATTN_EMPTY = 0, 1, 2


def attention_plan(B, Hq, Hkv, Sq, Skv, D=128, dtype=BF16, causal=True,
                   sm_count=148) -> lvb_attn_plan:
    """The kernel lvb_attention_fwd picks for these extents (host only, no GPU)."""
    d = lvb_attn_desc()
    d.dtype, d.causal = dtype, int(bool(causal))
    d.batch, d.heads_q, d.heads_kv, d.seq_q, d.seq_kv, d.head_dim = B, Hq, Hkv, Sq, Skv, D
    d.scale = float(D) ** -0.5
    p = lvb_attn_plan()
    check(lib.lvb_attention_plan_for(C.byref(d), sm_count, C.byref(p)))
    return p


def attention_available() -> bool:
    return True


def device_status(stream=None):
    """Synchronise and read/clear the device status word: (code, where, block)."""
    code, where, block = C.c_int32(), C.c_int32(), C.c_int32()
    check(lib.lvb_device_status(_stream_ptr(stream), C.byref(code), C.byref(where), C.byref(block)))
    return code.value, where.value, block.value


def gemm_noalloc_status(stream=None):
    """Synchronise and read/clear lvb_gemm_noalloc's own status word: (code, where, block)."""
    code, where, block = C.c_int32(), C.c_int32(), C.c_int32()
    check(lib.lvb_gemm_noalloc_status(_stream_ptr(stream), C.byref(code), C.byref(where),
                                      C.byref(block)))
    return code.value, where.value, block.value


def selftest_wait_timeout(ms: int = 50, stream=None) -> None:
    """Enqueue the failure-path self-test (a wait nothing satisfies, limited to ``ms``)."""
    check(lib.lvb_selftest_wait_timeout(int(ms), _stream_ptr(stream)))


def set_wait_timeout_ms(ms: int) -> None:
    check(lib.lvb_set_wait_timeout_ms(int(ms)))


def abi_version() -> int:
    return lib.lvb_abi_version()
