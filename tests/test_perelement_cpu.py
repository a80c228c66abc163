"""CPU tier: the host side of the vocabulary epilogue — per-element programs (the opcode
table against include/lvb.h, the Python tracer against direct numpy evaluation of the same
functions, the C ABI's program and epilogue validation) and the clamp restatement of the
oracle against hand-worked values. No GPU."""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

from oracle import perelement as ope
from oracle.gemm import clamp_pad, gemm_vocab_ref

HEADER = Path(__file__).resolve().parents[1] / "include" / "lvb.h"


def header_ops():
    txt = HEADER.read_text()
    return {m.group(1): int(m.group(2)) for m in re.finditer(r"LVB_PE_([A-Z0-9_]+) = (\d+)", txt)}


def test_opcode_tables_match_the_header(lvb):
    from lvb.perelement import OPS, NUM_OPS, MAX_INSTR, REGS, lvb_pe_program
    h = header_ops()
    assert h.pop("NUM_OPS") == NUM_OPS
    assert h == OPS
    for name, v in OPS.items():
        assert getattr(ope, name) == v, name
    assert C.sizeof(lvb_pe_program) == 4 + 8 * MAX_INSTR and REGS == 8
    assert C.sizeof(lvb.lvb_epilogue) == 120


def _grid(M=6, N=9, seed=0):
    g = np.random.default_rng(seed)
    x = g.standard_normal((M, N)).astype(np.float32) * 4
    e = g.standard_normal((M, N)).astype(np.float32)
    row = np.arange(M)[:, None] * np.ones((1, N), np.int64)
    col = np.ones((M, 1), np.int64) * np.arange(N)[None, :]
    return x, row, col, e


def test_traced_programs_equal_direct_evaluation(lvb):
    from lvb.perelement import (program, where, exp, exp2, tanh, maximum, minimum, fma, floor,
                                eq, sqrt, rsqrt, log, erf)
    from scipy.special import erf as serf
    x, row, col, e = _grid()
    rf, cf = row.astype(np.float32), col.astype(np.float32)
    f32 = np.float32
    cases = [
        (lambda x, r, c, e: where(c > r, float("-inf"), 0.125 * x - 0.5 * (r - c)),
         np.where(col > row, -np.inf, f32(0.125) * x - f32(0.5) * (rf - cf))),
        (lambda x, r, c, e: x * e + r, x * e + rf),
        (lambda x, r, c, e: maximum(minimum(x, 1.5), -1.0) + tanh(e) * exp(0.1 * x),
         np.maximum(np.minimum(x, f32(1.5)), f32(-1)) + np.tanh(e.astype(np.float64)).astype(f32)
         * np.exp((f32(0.1) * x).astype(np.float64)).astype(f32)),
        (lambda x, r, c, e: where(eq(r + c - floor(0.5 * (r + c)) * 2, 0), x, -x),
         np.where((rf + cf - np.floor(f32(0.5) * (rf + cf)) * 2) == 0, x, -x)),
        (lambda x, r, c, e: 3, np.full_like(x, 3)),
        (lambda x, r, c, e: (r - c) * (r + 2 * c), ((row - col) * (row + 2 * col)).astype(f32)),
        (lambda x, r, c, e: exp2(-abs(x)) + rsqrt(abs(e) + 1.0) - sqrt(abs(x)) + log(2.0 + e * e)
         + erf(e),
         (np.exp2(-np.abs(x).astype(np.float64)).astype(f32)
          + f32(1) / np.sqrt(np.abs(e) + f32(1)) - np.sqrt(np.abs(x))
          + np.log((f32(2) + e * e).astype(np.float64)).astype(f32)
          + serf(e.astype(np.float64)).astype(f32))),
        (lambda x, r, c, e: fma(x, e, 1.0) / (1 + abs(x)),
         (x.astype(np.float64) * e + 1).astype(f32) / (f32(1) + np.abs(x))),
    ]
    for fn, want in cases:
        p = program(fn)
        got = ope.pe_eval(p.code, x, row, col, e)
        assert np.allclose(got, want.astype(f32), rtol=2e-6, atol=2e-6, equal_nan=True), p


def test_tracer_errors(lvb):
    from lvb.perelement import program, ProgramError, where, exp
    with pytest.raises(ProgramError):                       # Python truth of a traced value
        program(lambda x, r, c, e: x if x > 0 else -x)
    with pytest.raises(ProgramError):                       # condition must be a comparison
        program(lambda x, r, c, e: where(x, x, e))
    with pytest.raises(ProgramError):                       # nine values live at once
        def wide(x, r, c, e):
            vs = [exp(x * float(i + 1)) for i in range(9)]
            acc = vs[0]
            for v in vs[1:]:
                acc = acc + v * vs[0]
            return acc + sum(vs[1:], vs[0])
        program(wide)
    with pytest.raises(ProgramError):                       # more than 32 instructions
        def long(x, r, c, e):
            for i in range(40):
                x = x * 1.0001 + float(i)
            return x
        program(long)


def test_pe_program_check_through_the_abi(lvb):
    from lvb.perelement import program, lvb_pe_program, lvb_pe_instr
    p = program(lambda x, r, c, e: x * 2.0 + c).to_struct()
    assert lvb.lib.lvb_pe_program_check(C.addressof(p)) == 0
    bad = lvb_pe_program()
    bad.n = 1
    bad.code[0] = lvb_pe_instr(40, 0, 0, 0, 0)
    assert lvb.lib.lvb_pe_program_check(C.addressof(bad)) == lvb.LVB_ERR_INVALID_ARG
    bad.code[0] = lvb_pe_instr(3, 9, 0, 0, 0)
    assert lvb.lib.lvb_pe_program_check(C.addressof(bad)) == lvb.LVB_ERR_INVALID_ARG
    bad.n = 33
    assert lvb.lib.lvb_pe_program_check(C.addressof(bad)) == lvb.LVB_ERR_INVALID_ARG
    assert lvb.lib.lvb_pe_program_check(None) == lvb.LVB_ERR_INVALID_ARG


def _desc(lvb, M, N, K, ab, out):
    t = {"Float16": lvb.F16, "Int8": lvb.I8, "Float32": lvb.F32, "Int32": lvb.I32}
    return lvb.lvb_gemm_desc(t[ab], t[ab], t[out], 1, 0, 0, M, N, K, K, K, M)


def test_gemm_ex_check_vocab_fields(lvb):
    from lvb.perelement import program
    ok = lvb.LVB_OK
    d = _desc(lvb, 64, 32, 100, "Float16", "Float32")
    e = lvb.lvb_epilogue()
    e.k_pad, e.a_clamp, e.a_clamp_value, e.b_clamp = 128, lvb.CLAMP_CONSTANT, 1.0, lvb.CLAMP_TO_EDGE
    assert lvb.lib.lvb_gemm_ex_check(C.byref(d), C.byref(e)) == ok
    e.k_pad = 64                                        # below K
    assert lvb.lib.lvb_gemm_ex_check(C.byref(d), C.byref(e)) == lvb.LVB_ERR_INVALID_ARG
    e.k_pad, e.a_clamp = 128, 7                          # unknown mode
    assert lvb.lib.lvb_gemm_ex_check(C.byref(d), C.byref(e)) == lvb.LVB_ERR_INVALID_ARG
    # TO_EDGE with K == 0 has no edge element
    d0 = _desc(lvb, 64, 32, 0, "Float16", "Float32")
    e0 = lvb.lvb_epilogue()
    e0.k_pad, e0.a_clamp = 16, lvb.CLAMP_TO_EDGE
    assert lvb.lib.lvb_gemm_ex_check(C.byref(d0), C.byref(e0)) == lvb.LVB_ERR_INVALID_ARG
    # 8-bit operands: integer clamp values in range; the clamp is their only epilogue
    d8 = _desc(lvb, 64, 32, 100, "Int8", "Int32")
    e8 = lvb.lvb_epilogue()
    e8.k_pad, e8.a_clamp, e8.a_clamp_value = 128, lvb.CLAMP_CONSTANT, -128
    assert lvb.lib.lvb_gemm_ex_check(C.byref(d8), C.byref(e8)) == ok
    e8.a_clamp_value = 0.5
    assert lvb.lib.lvb_gemm_ex_check(C.byref(d8), C.byref(e8)) == lvb.LVB_ERR_INVALID_ARG
    e8.a_clamp_value = 128
    assert lvb.lib.lvb_gemm_ex_check(C.byref(d8), C.byref(e8)) == lvb.LVB_ERR_INVALID_ARG
    e8.a_clamp_value = 1
    p = program(lambda x, r, c, e: x + 1.0).to_struct()
    e8.program = C.addressof(p)
    assert lvb.lib.lvb_gemm_ex_check(C.byref(d8), C.byref(e8)) == lvb.LVB_ERR_UNSUPPORTED
    # an extra matrix needs a program; mul needs a float type and a leading dimension >= M
    e2 = lvb.lvb_epilogue()
    e2.extra, e2.extra_type, e2.lde = 256, lvb.F32, 64
    assert lvb.lib.lvb_gemm_ex_check(C.byref(d), C.byref(e2)) == lvb.LVB_ERR_INVALID_ARG
    e3 = lvb.lvb_epilogue()
    e3.mul, e3.mul_type, e3.ldm = 256, lvb.I32, 64
    assert lvb.lib.lvb_gemm_ex_check(C.byref(d), C.byref(e3)) == lvb.LVB_ERR_UNSUPPORTED
    e3.mul_type, e3.ldm = lvb.F16, 10
    assert lvb.lib.lvb_gemm_ex_check(C.byref(d), C.byref(e3)) == lvb.LVB_ERR_INVALID_ARG
    e3.ldm = 64
    assert lvb.lib.lvb_gemm_ex_check(C.byref(d), C.byref(e3)) == ok


def test_clamp_pad_known_values():
    """Hand-worked reads past the extent (tensor.jl:46-51): constant rounded to the
    component type (tensor_clampbits, tensor.jl:83-85), the edge element, zero."""
    A = np.array([[1, 2, 3], [4, 5, 6]], dtype=np.float16)
    assert clamp_pad(A, 5, 1, "constant", 0.1, "Float16").tolist() == \
        [[1, 2, 3, np.float16(0.1), np.float16(0.1)], [4, 5, 6, np.float16(0.1), np.float16(0.1)]]
    assert clamp_pad(A, 5, 1, "edge", 0, "Float16").tolist() == [[1, 2, 3, 3, 3], [4, 5, 6, 6, 6]]
    assert clamp_pad(A.T, 4, 0, "undefined", 0, "Float16").tolist() == [[1, 4], [2, 5], [3, 6], [0, 0]]
    I = np.array([[1, -2]], dtype=np.int8)
    assert clamp_pad(I, 4, 1, "constant", -7, "Int8").tolist() == [[1, -2, -7, -7]]
    # an exact int8 product over the padded extent: [1,-2,-7,-7]·[3,4,4,4]ᵀ (B to edge)
    B = np.array([[3], [4]], dtype=np.int8)
    got = gemm_vocab_ref(I, B, "Int32", "Int8", k_pad=4, a_clamp=("constant", -7),
                         b_clamp=("edge", 0))
    assert got.tolist() == [[3 - 8 - 28 - 28]]
