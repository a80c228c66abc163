"""Per-element program oracle — TEST INFRASTRUCTURE (see ``oracle/__init__.py``).

Restates, in numpy, what the GEMM epilogue computes for a caller's per-element function
(Lava's ``coopmat_perelement(f, m, extras...)``, ``src/device/coopmat_intrinsics.jl:520-678``:
``f(row0, col0, elem, extras...)`` for every element, row and column 0-based UInt32,
``coopmat_intrinsics.jl:551-593``) when the function arrives as an ``lvb_pe_program`` (the
straight-line form the C ABI carries, ``include/lvb.h``): 8 registers of 32 bits, r0 = the
element (fp32), r1 = row, r2 = col (int32), r3 = the extra matrix's element (fp32), r4..r7 = 0;
the result is r0. Each opcode below follows its definition in the header; fp32 arithmetic is
numpy float32 (IEEE, round to nearest even), the transcendental functions are evaluated in
float64 and rounded once to fp32 (the device's are within a few ulp of that).
"""
from __future__ import annotations

import numpy as np

# lvb_pe_op values (include/lvb.h)
CONST, ICONST, MOV, FADD, FSUB, FMUL, FDIV, FMIN, FMAX, FFMA = range(10)
FNEG, FABS, FEXP, FEXP2, FLOG, FTANH, FSQRT, FRSQRT, FFLOOR, FERF = range(10, 20)
I2F, IADD, ISUB, IMUL, IMIN, IMAX = range(20, 26)
FLT, FLE, FEQ, ILT, ILE, IEQ, SELECT = range(26, 33)


def _f(u):
    return u.view(np.float32)


def _i(u):
    return u.view(np.int32)


def _u(x):
    return np.ascontiguousarray(x).view(np.uint32)


def _f64(fn):
    def g(a):
        with np.errstate(all="ignore"):
            return fn(_f(a).astype(np.float64)).astype(np.float32)
    return g


def _erf(x):
    from scipy.special import erf
    return erf(x)


UNARY = {
    FEXP: _f64(np.exp), FEXP2: _f64(np.exp2), FLOG: _f64(np.log), FTANH: _f64(np.tanh),
    FSQRT: lambda a: np.sqrt(_f(a)),
    FRSQRT: lambda a: np.float32(1.0) / np.sqrt(_f(a)),
    FFLOOR: lambda a: np.floor(_f(a)),
    FERF: _f64(_erf),
}


def pe_eval(code, x, row, col, ext=None):
    """Evaluate ``code`` (a list of (op, dst, a, b, imm)) for every element: x, ext fp32
    arrays, row, col int arrays of one shape. Returns the fp32 result array."""
    x = np.asarray(x, dtype=np.float32)
    shape = x.shape
    R = np.zeros((8,) + shape, dtype=np.uint32)
    R[0] = _u(x)
    R[1] = _u(np.asarray(row, dtype=np.int64).astype(np.int32) * np.ones(shape, np.int32))
    R[2] = _u(np.asarray(col, dtype=np.int64).astype(np.int32) * np.ones(shape, np.int32))
    if ext is not None:
        R[3] = _u(np.asarray(ext, dtype=np.float32) * np.ones(shape, np.float32))
    with np.errstate(all="ignore"):
        for op, dst, a, b, imm in code:
            A, B, D = R[a].copy(), R[b].copy(), R[dst].copy()
            if op == CONST or op == ICONST:
                out = np.full(shape, imm, dtype=np.uint32)
            elif op == MOV:
                out = A
            elif op == FADD:
                out = _u(_f(A) + _f(B))
            elif op == FSUB:
                out = _u(_f(A) - _f(B))
            elif op == FMUL:
                out = _u(_f(A) * _f(B))
            elif op == FDIV:
                out = _u(_f(A) / _f(B))
            elif op == FMIN:
                out = _u(np.fmin(_f(A), _f(B)))
            elif op == FMAX:
                out = _u(np.fmax(_f(A), _f(B)))
            elif op == FFMA:
                # a·b is exact in float64; the sum rounded to float64 and then to fp32
                out = _u((_f(A).astype(np.float64) * _f(B) + _f(D)).astype(np.float32))
            elif op == FNEG:
                out = A ^ np.uint32(0x80000000)
            elif op == FABS:
                out = A & np.uint32(0x7FFFFFFF)
            elif op in UNARY:
                out = _u(UNARY[op](A).astype(np.float32))
            elif op == I2F:
                out = _u(_i(A).astype(np.float32))
            elif op == IADD:
                out = A + B
            elif op == ISUB:
                out = A - B
            elif op == IMUL:
                out = A * B
            elif op == IMIN:
                out = _u(np.minimum(_i(A), _i(B)))
            elif op == IMAX:
                out = _u(np.maximum(_i(A), _i(B)))
            elif op in (FLT, FLE, FEQ):
                fa, fb = _f(A), _f(B)
                c = fa < fb if op == FLT else (fa <= fb if op == FLE else fa == fb)
                out = c.astype(np.uint32)
            elif op in (ILT, ILE, IEQ):
                ia, ib = _i(A), _i(B)
                c = ia < ib if op == ILT else (ia <= ib if op == ILE else ia == ib)
                out = c.astype(np.uint32)
            elif op == SELECT:
                out = np.where(A != 0, B, D)
            else:
                raise ValueError(f"unknown opcode {op}")
            R[dst] = out.astype(np.uint32)
    return _f(R[0]).copy()
