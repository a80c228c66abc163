# Per-element programs: the function of Lava's `coopmat_perelement(f, m, extras...)`
# (src/device/coopmat_intrinsics.jl:520-678) carried across the C ABI as the straight-line
# program `lvb_pe_program` (include/lvb.h) that the GEMM epilogue evaluates for every element:
# registers r0 = the element (Float32), r1 = row, r2 = col (0-based Int32), r3 = the `extra`
# matrix's element (Float32), r4..r7 = 0; the result is r0. `pe_program(f)` calls `f` once on
# symbolic values and records what it does — the counterpart of Lava compiling `f` into the
# kernel. The same tracer exists in Python (lava.jl_b200/lvb/perelement.py).

struct PeInstr
    op::UInt8; dst::UInt8; a::UInt8; b::UInt8
    imm::UInt32
end

struct PeProgram
    n::Int32
    code::NTuple{32,PeInstr}
end

const PE_OPS = Dict{Symbol,UInt8}(
    :CONST => 0, :ICONST => 1, :MOV => 2, :FADD => 3, :FSUB => 4, :FMUL => 5, :FDIV => 6,
    :FMIN => 7, :FMAX => 8, :FFMA => 9, :FNEG => 10, :FABS => 11, :FEXP => 12, :FEXP2 => 13,
    :FLOG => 14, :FTANH => 15, :FSQRT => 16, :FRSQRT => 17, :FFLOOR => 18, :FERF => 19,
    :I2F => 20, :IADD => 21, :ISUB => 22, :IMUL => 23, :IMIN => 24, :IMAX => 25, :FLT => 26,
    :FLE => 27, :FEQ => 28, :ILT => 29, :ILE => 30, :IEQ => 31, :SELECT => 32)

mutable struct PeTracer
    nodes::Vector{Tuple{Symbol,Vector{Int},UInt32,Symbol}}   # (op, args, imm, kind :f/:i)
    consts::Dict{Tuple{Symbol,UInt32},Int}
end

"""A symbolic Float32 (`:f`) or Int32 (`:i`) value while a per-element function is traced."""
struct PeVal
    tr::PeTracer
    id::Int
    kind::Symbol
end

function pe_node!(tr::PeTracer, op::Symbol, args::Vector{Int}, imm::UInt32, kind::Symbol)
    push!(tr.nodes, (op, args, imm, kind))
    return PeVal(tr, length(tr.nodes), kind)
end

pe_lift(tr::PeTracer, v::PeVal, ::Symbol) = v
function pe_lift(tr::PeTracer, v::Integer, kind::Symbol)
    kind === :f && return pe_lift(tr, Float32(v), :f)
    typemin(Int32) <= v <= typemax(Int32) || throw(ArgumentError("pe_program: $v outside Int32"))
    bits = reinterpret(UInt32, Int32(v))
    return PeVal(tr, get!(() -> pe_node!(tr, :ICONST, Int[], bits, :i).id, tr.consts, (:i, bits)), :i)
end
function pe_lift(tr::PeTracer, v::Real, ::Symbol)
    bits = reinterpret(UInt32, Float32(v))
    return PeVal(tr, get!(() -> pe_node!(tr, :CONST, Int[], bits, :f).id, tr.consts, (:f, bits)), :f)
end

pe_f(tr, v::PeVal) = v.kind === :f ? v : pe_node!(tr, :I2F, [v.id], UInt32(0), :f)
kindof(v::PeVal) = v.kind
kindof(v::Integer) = :i
kindof(v::Real) = :f

function pe_unify(tr, a, b)
    kind = kindof(a) === :i && kindof(b) === :i ? :i : :f
    x, y = pe_lift(tr, a, kind), pe_lift(tr, b, kind)
    kind === :f && ((x, y) = (pe_f(tr, x), pe_f(tr, y)))
    return x, y, kind
end

tracer(a::PeVal, rest...) = a.tr
tracer(a::Real, b::PeVal, rest...) = b.tr
tracer(a::Real, b::Real, c::PeVal) = c.tr

function pe_binary(name::Symbol, a, b)
    tr = tracer(a, b)
    x, y, kind = pe_unify(tr, a, b)
    op = Symbol(kind === :i ? "I" : "F", name)
    return pe_node!(tr, op, [x.id, y.id], UInt32(0), kind)
end
function pe_compare(name::Symbol, a, b)
    tr = tracer(a, b)
    x, y, kind = pe_unify(tr, a, b)
    return pe_node!(tr, Symbol(kind === :i ? "I" : "F", name), [x.id, y.id], UInt32(0), :i)
end
function pe_unary(op::Symbol, a::PeVal)
    x = pe_f(a.tr, a)
    return pe_node!(a.tr, op, [x.id], UInt32(0), :f)
end

for (f, name) in ((:+, :ADD), (:-, :SUB), (:*, :MUL))
    @eval Base.$f(a::PeVal, b::PeVal) = pe_binary($(QuoteNode(name)), a, b)
    @eval Base.$f(a::PeVal, b::Real) = pe_binary($(QuoteNode(name)), a, b)
    @eval Base.$f(a::Real, b::PeVal) = pe_binary($(QuoteNode(name)), a, b)
end
function pe_div(a, b)
    tr = tracer(a, b)
    x, y, _ = pe_unify(tr, a, b)
    return pe_node!(tr, :FDIV, [pe_f(tr, x).id, pe_f(tr, y).id], UInt32(0), :f)
end
Base.:/(a::PeVal, b::PeVal) = pe_div(a, b)
Base.:/(a::PeVal, b::Real) = pe_div(a, b)
Base.:/(a::Real, b::PeVal) = pe_div(a, b)
Base.:-(a::PeVal) = a.kind === :f ? pe_unary(:FNEG, a) : 0 - a
Base.abs(a::PeVal) = a.kind === :f ? pe_unary(:FABS, a) : max(a, -a)
for (f, name) in ((:<, :LT), (:<=, :LE))
    @eval Base.$f(a::PeVal, b::PeVal) = pe_compare($(QuoteNode(name)), a, b)
    @eval Base.$f(a::PeVal, b::Real) = pe_compare($(QuoteNode(name)), a, b)
    @eval Base.$f(a::Real, b::PeVal) = pe_compare($(QuoteNode(name)), a, b)
end
Base.:>(a::PeVal, b::Union{PeVal,Real}) = b < a
Base.:>(a::Real, b::PeVal) = b < a
Base.:>=(a::PeVal, b::Union{PeVal,Real}) = b <= a
Base.:>=(a::Real, b::PeVal) = b <= a
"""`pe_eq(a, b)`: element-wise equality (Int32 0/1), since `==` must stay a Bool in Julia."""
pe_eq(a, b) = pe_compare(:EQ, a, b)
for (f, name) in ((:min, :MIN), (:max, :MAX))
    @eval Base.$f(a::PeVal, b::PeVal) = pe_binary($(QuoteNode(name)), a, b)
    @eval Base.$f(a::PeVal, b::Real) = pe_binary($(QuoteNode(name)), a, b)
    @eval Base.$f(a::Real, b::PeVal) = pe_binary($(QuoteNode(name)), a, b)
end
for (f, op) in ((:exp, :FEXP), (:exp2, :FEXP2), (:log, :FLOG), (:tanh, :FTANH), (:sqrt, :FSQRT),
                (:floor, :FFLOOR))
    @eval Base.$f(a::PeVal) = pe_unary($(QuoteNode(op)), a)
end
"""`pe_rsqrt(x)` = 1/sqrt(x) and `pe_erf(x)` = erf(x) on traced values."""
pe_rsqrt(a::PeVal) = pe_unary(:FRSQRT, a)
pe_erf(a::PeVal) = pe_unary(:FERF, a)
function Base.fma(a::PeVal, b::Union{PeVal,Real}, c::Union{PeVal,Real})
    tr = a.tr
    x, y, z = (pe_f(tr, pe_lift(tr, v, :f)) for v in (a, b, c))
    return pe_node!(tr, :FFMA, [x.id, y.id, z.id], UInt32(0), :f)
end
# `ifelse` is a builtin (no methods can be added), so the traced select has its own name.
"""`pe_ifelse(c, a, b)`: `c ? a : b` element-wise, `c` a comparison of traced values."""
function pe_ifelse(c::PeVal, a, b)
    c.kind === :i || throw(ArgumentError("pe_program: pe_ifelse needs a comparison as its condition"))
    tr = c.tr
    x, y, kind = pe_unify(tr, a, b)
    return pe_node!(tr, :SELECT, [c.id, x.id, y.id], UInt32(0), kind)
end
Base.Bool(::PeVal) = throw(ArgumentError("pe_program: a traced value has no truth value; use pe_ifelse"))  # Bool(v); `if v` is a TypeError

"""
    pe_program(f) -> PeProgram

Trace `f(x, row, col, e)` — `x`, `e` Float32, `row`, `col` 0-based Int32 — into the library's
per-element program. Supported: `+ - * /`, unary `-`, `abs`, `< <= > >=`, `pe_eq`, `min`,
`max`, `exp`, `exp2`, `log`, `tanh`, `sqrt`, `floor`, `fma`, `pe_ifelse`, `pe_rsqrt`, `pe_erf`.
At most 32 instructions and 8 values alive at once.
"""
function pe_program(f)
    tr = PeTracer([(:IN, Int[], UInt32(0), :f), (:IN, Int[], UInt32(0), :i),
                   (:IN, Int[], UInt32(0), :i), (:IN, Int[], UInt32(0), :f)],
                  Dict{Tuple{Symbol,UInt32},Int}())
    ins = [PeVal(tr, i, tr.nodes[i][4]) for i in 1:4]
    out = f(ins...)
    out = out isa PeVal ? out : pe_lift(tr, out, :f)
    return pe_compile(tr, pe_f(tr, out).id)
end

function pe_compile(tr::PeTracer, out::Int)
    nodes = tr.nodes
    live = Set{Int}()
    stack = [out]
    while !isempty(stack)
        n = pop!(stack)
        n in live && continue
        push!(live, n)
        append!(stack, nodes[n][2])
    end
    order = sort!(collect(live))
    last = Dict(n => 0 for n in order)
    for n in order, a in nodes[n][2]
        last[a] = max(last[a], n)
    end
    last[out] = typemax(Int)
    reg = Dict{Int,Int}()
    free = collect(0:7)
    for i in 1:4
        i in live && (reg[i] = i - 1; filter!(!=(i - 1), free))
    end
    code = PeInstr[]
    take!() = isempty(free) ? throw(ArgumentError("pe_program: more than 8 values alive at once")) :
              popfirst!(free)
    function release!(n)
        for a in unique(nodes[n][2])
            if last[a] == n && haskey(reg, a)
                push!(free, reg[a]); sort!(free)
            end
        end
    end
    emit!(op, dst, a = 0, b = 0, imm = UInt32(0)) =
        push!(code, PeInstr(PE_OPS[op], UInt8(dst), UInt8(a), UInt8(b), imm))
    for n in order
        op, args, imm, kind = nodes[n]
        op === :IN && continue
        if op === :SELECT || op === :FFMA
            # the third operand (the else value / the addend) must sit in the result register
            x, y, z = args
            if last[z] == n && z != x && z != y
                dst = reg[z]; delete!(reg, z); release!(n)
            else
                release!(n); dst = take!(); emit!(:MOV, dst, reg[z])
            end
            emit!(op, dst, reg[x], reg[y])
            reg[n] = dst
            continue
        end
        ra = length(args) >= 1 ? reg[args[1]] : 0
        rb = length(args) >= 2 ? reg[args[2]] : 0
        release!(n)
        dst = take!()
        emit!(op, dst, ra, rb, imm)
        reg[n] = dst
    end
    reg[out] != 0 && emit!(:MOV, 0, reg[out])
    length(code) <= 32 || throw(ArgumentError("pe_program: $(length(code)) instructions, at most 32"))
    pad = ntuple(i -> i <= length(code) ? code[i] : PeInstr(0, 0, 0, 0, 0), 32)
    return PeProgram(Int32(length(code)), pad)
end
