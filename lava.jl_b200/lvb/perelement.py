"""Per-element programs — the caller-supplied function of Lava's
``coopmat_perelement(f, m, extras...)`` (``src/device/coopmat_intrinsics.jl:520-678``) for the
GEMM's fused epilogue.

Lava compiles ``f`` into the kernel. Across this library's C ABI the function travels as a
short straight-line program over 8 registers (``lvb_pe_program`` in ``include/lvb.h``) that
the epilogue evaluates for every element of C, with the element's 0-based row and column
(``coopmat_intrinsics.jl:551-593``) and the element of an optional second matrix at the same
position (the matrix-operand form). ``program(f)`` builds one by calling ``f`` once on
symbolic values::

    from lvb.perelement import program, where, exp
    # a causal mask with an ALiBi-style slope, on the scaled scores
    p = program(lambda x, row, col, e: where(col > row, float("-inf"), 0.125 * x - 0.5 * (row - col)))

``x`` and ``e`` are fp32 values, ``row`` and ``col`` int32; arithmetic between an int and a
float converts the int (``I2F``), comparisons give int 0/1, ``where(c, a, b)`` selects. The
result is converted to fp32. Supported: ``+ - * /``, unary ``-``, ``abs``, ``< <= > >=``,
``eq``, ``minimum``, ``maximum``, ``exp``, ``exp2``, ``log``, ``tanh``, ``sqrt``, ``rsqrt``,
``floor``, ``erf``, ``fma``, ``where``.
"""
from __future__ import annotations

import ctypes as C
import struct
from typing import Callable

MAX_INSTR, REGS = 32, 8

# opcodes (include/lvb.h, lvb_pe_op)
OPS = {
    "CONST": 0, "ICONST": 1, "MOV": 2, "FADD": 3, "FSUB": 4, "FMUL": 5, "FDIV": 6, "FMIN": 7,
    "FMAX": 8, "FFMA": 9, "FNEG": 10, "FABS": 11, "FEXP": 12, "FEXP2": 13, "FLOG": 14,
    "FTANH": 15, "FSQRT": 16, "FRSQRT": 17, "FFLOOR": 18, "FERF": 19, "I2F": 20, "IADD": 21,
    "ISUB": 22, "IMUL": 23, "IMIN": 24, "IMAX": 25, "FLT": 26, "FLE": 27, "FEQ": 28,
    "ILT": 29, "ILE": 30, "IEQ": 31, "SELECT": 32,
}
NUM_OPS = 33


class lvb_pe_instr(C.Structure):
    _fields_ = [("op", C.c_uint8), ("dst", C.c_uint8), ("a", C.c_uint8), ("b", C.c_uint8),
                ("imm", C.c_uint32)]


class lvb_pe_program(C.Structure):
    _fields_ = [("n", C.c_int32), ("code", lvb_pe_instr * MAX_INSTR)]


def f32_bits(v: float) -> int:
    return struct.unpack("<I", struct.pack("<f", v))[0]


class ProgramError(ValueError):
    pass


class Program:
    """A straight-line program: a list of ``(op, dst, a, b, imm)`` tuples."""

    def __init__(self, code):
        code = [tuple(int(v) for v in ins) for ins in code]
        if len(code) > MAX_INSTR:
            raise ProgramError(f"program needs {len(code)} instructions, at most {MAX_INSTR}")
        for i, (op, dst, a, b, imm) in enumerate(code):
            if not 0 <= op < NUM_OPS:
                raise ProgramError(f"instruction {i}: unknown opcode {op}")
            if not all(0 <= r < REGS for r in (dst, a, b)):
                raise ProgramError(f"instruction {i}: register outside r0..r7")
            if not 0 <= imm < 2 ** 32:
                raise ProgramError(f"instruction {i}: immediate outside 32 bits")
        self.code = code

    def __len__(self):
        return len(self.code)

    def to_struct(self) -> lvb_pe_program:
        s = lvb_pe_program()
        s.n = len(self.code)
        for i, (op, dst, a, b, imm) in enumerate(self.code):
            s.code[i] = lvb_pe_instr(op, dst, a, b, imm)
        return s

    def __repr__(self):
        names = {v: k for k, v in OPS.items()}
        return "Program([" + ", ".join(f"({names[o]}, r{d}, r{a}, r{b}, {i:#x})"
                                       for o, d, a, b, i in self.code) + "])"


# ---- tracing ------------------------------------------------------------------------------
class Value:
    """A symbolic fp32 ('f') or int32 ('i') value produced while tracing a program."""
    __slots__ = ("tr", "id", "kind")
    __hash__ = None  # comparisons build nodes, so values are not dict keys

    def __init__(self, tr, nid, kind):
        self.tr, self.id, self.kind = tr, nid, kind

    # arithmetic
    def __add__(self, o): return self.tr.binary("ADD", self, o)
    def __radd__(self, o): return self.tr.binary("ADD", o, self)
    def __sub__(self, o): return self.tr.binary("SUB", self, o)
    def __rsub__(self, o): return self.tr.binary("SUB", o, self)
    def __mul__(self, o): return self.tr.binary("MUL", self, o)
    def __rmul__(self, o): return self.tr.binary("MUL", o, self)
    def __truediv__(self, o): return self.tr.binary("DIV", self, o)
    def __rtruediv__(self, o): return self.tr.binary("DIV", o, self)
    def __neg__(self): return self.tr.unary_f("FNEG", self) if self.kind == "f" else 0 - self
    def __abs__(self): return self.tr.unary_f("FABS", self) if self.kind == "f" else maximum(self, -self)
    # comparisons (int 0/1)
    def __lt__(self, o): return self.tr.compare("LT", self, o)
    def __le__(self, o): return self.tr.compare("LE", self, o)
    def __gt__(self, o): return self.tr.compare("LT", o, self)
    def __ge__(self, o): return self.tr.compare("LE", o, self)

    def __bool__(self):
        raise ProgramError("a traced value has no truth value: use where(cond, a, b)")


class Tracer:
    def __init__(self):
        # node: (op name, arg node ids, imm, kind); nodes 0..3 are the inputs x, row, col, e
        self.nodes = [("IN", (), 0, "f"), ("IN", (), 0, "i"), ("IN", (), 0, "i"), ("IN", (), 0, "f")]
        self.consts = {}

    def node(self, op, args, imm, kind) -> Value:
        self.nodes.append((op, tuple(args), imm, kind))
        return Value(self, len(self.nodes) - 1, kind)

    def lift(self, v, kind) -> Value:
        """A Python number as a constant node of `kind` (cached)."""
        if isinstance(v, Value):
            if v.tr is not self:
                raise ProgramError("values of two different traces mixed")
            return v
        if isinstance(v, bool) or not isinstance(v, (int, float)):
            raise ProgramError(f"unsupported constant {v!r}")
        if kind == "i" and isinstance(v, int):
            if not -2 ** 31 <= v < 2 ** 31:
                raise ProgramError(f"integer constant {v} outside int32")
            key = ("i", v)
            if key not in self.consts:
                self.consts[key] = self.node("ICONST", (), v & 0xFFFFFFFF, "i")
            return self.consts[key]
        key = ("f", f32_bits(float(v)))
        if key not in self.consts:
            self.consts[key] = self.node("CONST", (), key[1], "f")
        return self.consts[key]

    def to_f(self, v: Value) -> Value:
        return v if v.kind == "f" else self.node("I2F", (v.id,), 0, "f")

    def unify(self, a, b):
        """Both operands as Values of one kind: int only if both are ints."""
        ka = a.kind if isinstance(a, Value) else ("i" if isinstance(a, int) and not isinstance(a, bool) else "f")
        kb = b.kind if isinstance(b, Value) else ("i" if isinstance(b, int) and not isinstance(b, bool) else "f")
        kind = "i" if ka == kb == "i" else "f"
        a, b = self.lift(a, kind), self.lift(b, kind)
        if kind == "f":
            a, b = self.to_f(a), self.to_f(b)
        return a, b, kind

    def binary(self, name, a, b) -> Value:
        if name == "DIV":
            a, b, _ = self.unify(a, b)
            a, b = self.to_f(a), self.to_f(b)
            return self.node("FDIV", (a.id, b.id), 0, "f")
        a, b, kind = self.unify(a, b)
        return self.node(("I" if kind == "i" else "F") + name, (a.id, b.id), 0, kind)

    def compare(self, name, a, b) -> Value:
        a, b, kind = self.unify(a, b)
        return self.node(("I" if kind == "i" else "F") + name, (a.id, b.id), 0, "i")

    def unary_f(self, op, a) -> Value:
        a = self.to_f(self.lift(a, "f"))
        return self.node(op, (a.id,), 0, "f")


def _tracer_of(*vals):
    for v in vals:
        if isinstance(v, Value):
            return v.tr
    raise ProgramError("at least one operand must be a traced value")


def where(cond, a, b):
    """``cond ? a : b`` element-wise; ``cond`` a comparison (int 0/1)."""
    tr = _tracer_of(cond, a, b)
    c = tr.lift(cond, "i")
    if c.kind != "i":
        raise ProgramError("where: the condition must be a comparison (int 0/1)")
    a, b, kind = tr.unify(a, b)
    return tr.node("SELECT", (c.id, a.id, b.id), 0, kind)


def minimum(a, b):
    tr = _tracer_of(a, b)
    a, b, kind = tr.unify(a, b)
    return tr.node("IMIN" if kind == "i" else "FMIN", (a.id, b.id), 0, kind)


def maximum(a, b):
    tr = _tracer_of(a, b)
    a, b, kind = tr.unify(a, b)
    return tr.node("IMAX" if kind == "i" else "FMAX", (a.id, b.id), 0, kind)


def eq(a, b):
    tr = _tracer_of(a, b)
    a, b, kind = tr.unify(a, b)
    return tr.node("IEQ" if kind == "i" else "FEQ", (a.id, b.id), 0, "i")


def fma(a, b, c):
    """a·b + c with one rounding (fp32)."""
    tr = _tracer_of(a, b, c)
    a, b, c = (tr.to_f(tr.lift(v, "f")) for v in (a, b, c))
    return tr.node("FFMA", (a.id, b.id, c.id), 0, "f")


def _unary(op):
    def f(a):
        if not isinstance(a, Value):
            raise ProgramError(f"{op.lower()}: the operand must be a traced value")
        return a.tr.unary_f(op, a)
    f.__name__ = op[1:].lower()
    return f


exp, exp2, log, tanh = _unary("FEXP"), _unary("FEXP2"), _unary("FLOG"), _unary("FTANH")
sqrt, rsqrt, floor, erf = _unary("FSQRT"), _unary("FRSQRT"), _unary("FFLOOR"), _unary("FERF")


def program(fn: Callable) -> Program:
    """Trace ``fn(x, row, col, e)`` into a Program (see the module docstring)."""
    tr = Tracer()
    ins = [Value(tr, i, tr.nodes[i][3]) for i in range(4)]
    out = fn(*ins)
    if not isinstance(out, Value):
        out = tr.lift(out, "f")
    out = tr.to_f(out)
    return _compile(tr, out.id)


def _compile(tr: Tracer, out: int) -> Program:
    nodes = tr.nodes
    # live nodes: reachable from the output
    live = set()
    stack = [out]
    while stack:
        n = stack.pop()
        if n in live:
            continue
        live.add(n)
        stack.extend(nodes[n][1])
    order = [n for n in range(len(nodes)) if n in live]
    last = {n: -1 for n in order}
    for n in order:
        for a in nodes[n][1]:
            last[a] = max(last[a], n)
    last[out] = len(nodes)                    # the result stays until the final move
    reg = {}
    free = list(range(REGS))
    for i in range(4):                       # the inputs arrive in r0..r3
        if i in live:
            reg[i] = i
            free.remove(i)
    code = []

    def take():
        if not free:
            raise ProgramError("the program needs more than 8 registers at once")
        return free.pop(0)

    def release_after(n):
        for a in set(nodes[n][1]):
            if last[a] == n and a in reg:
                free.append(reg[a])
                free.sort()

    for n in order:
        op, args, imm, kind = nodes[n]
        if op == "IN":
            continue
        if op == "SELECT":
            c, t, f = args
            if last[f] == n and f != c and f != t:
                dst = reg[f]                 # the else operand's register becomes the result
                del reg[f]
                release_after(n)
            else:
                release_after(n)
                dst = take()
                code.append((OPS["MOV"], dst, reg[f], 0, 0))
            code.append((OPS["SELECT"], dst, reg[c], reg[t], 0))
            reg[n] = dst
            continue
        if op == "FFMA":
            a, b, c = args
            if last[c] == n and c != a and c != b:
                dst = reg[c]
                del reg[c]
                release_after(n)
            else:
                release_after(n)
                dst = take()
                code.append((OPS["MOV"], dst, reg[c], 0, 0))
            code.append((OPS["FFMA"], dst, reg[a], reg[b], 0))
            reg[n] = dst
            continue
        ra = reg[args[0]] if len(args) > 0 else 0
        rb = reg[args[1]] if len(args) > 1 else 0
        release_after(n)
        dst = take()
        code.append((OPS[op], dst, ra, rb, imm))
        reg[n] = dst
    if reg[out] != 0:
        code.append((OPS["MOV"], 0, reg[out], 0, 0))
    return Program(code)


__all__ = ["Program", "ProgramError", "program", "where", "minimum", "maximum", "eq", "fma",
           "exp", "exp2", "log", "tanh", "sqrt", "rsqrt", "floor", "erf", "OPS",
           "lvb_pe_program", "lvb_pe_instr", "f32_bits"]
