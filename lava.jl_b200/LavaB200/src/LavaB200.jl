"""
    LavaB200

The B200 (sm_100a) execution path for Lava.jl's cooperative-matrix GEMM and
flash-attention: a kernel author's `gemm!` / `attention!` call, and the backend's answer to
`Lava.caps`, go through `ccall` into `liblvb.so` (hand-written tcgen05/TMA kernels behind a
C ABI, `include/lvb.h`) instead of compiling a coopmat kernel to SPIR-V and dispatching it
through Vulkan.

* `gemm!(C, A, B)` — `C = A·B` accumulated in the pair's accumulator type (Float32 for
  Float16/BFloat16, Int32 for Int8, UInt32 for UInt8), converted to `eltype(C)` with
  round-to-nearest-even — Lava's `muladd` + `convert` + `copyto!`
  (src/vocabulary/coopmat.jl:150-203). Column-major device matrices are Julia's default;
  a row-major operand is the `transpose` of a column-major one (`Val(true)` in Lava's load).
  Keywords `bias`, `residual`, `activation` fuse the epilogue `act(A·B + bias + residual)`.
* `attention!(O, Q, K, V; causal, scale)` — Q/O `(E, Lq, Hq, B)`, K/V `(E, Lk, Hkv, B)`
  column-major (Lava's layout, src/device/sharedmemory.jl:73-76); GQA by head grouping.
* `B200Array` — an owning device buffer (`lvb_malloc`/`lvb_free`); any value with
  `pointer` and `size` (e.g. `Lava.LavaDeviceArray`, a non-owning `(ptr, dims)`,
  src/device/devicearray.jl:35-38) is accepted by the ops.
* Errors: `LavaB200Error(operation, message, suggestion)`, Lava's `LavaError` triad
  (src/runtime/errors.jl:4-24).

Loading `Lava` alongside activates `LavaB200LavaExt`, which answers `Lava.caps`,
`Lava.supports_*` for `B200Backend` with Lava's own `DeviceCaps` and `MatrixShape`.
"""
module LavaB200

using Libdl
using LinearAlgebra: Transpose, transpose
# Lava's backend-form queries (`matrix_shapes(backend)`, `supports(backend, s)`,
# `bestshape(backend, ab, acc)`, src/vocabulary/caps.jl:158-169, matrix.jl:138-141) dispatch
# on `backend::KI.Backend` and call `caps(backend)`; B200Backend subtypes it so they resolve.
import KernelInterface as KI

export B200Backend, B200Array, gemm!, attention!, device_status, caps_raw, matrix_shapes_raw,
       pe_program, PeProgram, pe_ifelse, pe_eq, pe_rsqrt, pe_erf,
       LavaB200Error, BFloat16, shard_range, comm_unique_id, Comm, allgather!

const libpath = Ref{String}("")
const libhandle = Ref{Ptr{Cvoid}}(C_NULL)

default_lib() = get(ENV, "LVB_LIBRARY",
                    normpath(joinpath(@__DIR__, "..", "..", "lib", "liblvb.so")))

function __init__()
    p = default_lib()
    isfile(p) || error("liblvb.so not found at $p — build it with `python lava.jl_b200/build.py`")
    libpath[] = p
    libhandle[] = Libdl.dlopen(p, Libdl.RTLD_GLOBAL)
end

sym(name::Symbol) = Libdl.dlsym(libhandle[], name)

# ---- enums (include/lvb.h) --------------------------------------------------------------
const LVB_OK = 0
const LVB_ERR_UNSUPPORTED = 2
const STATUS = Dict(0 => :LVB_OK, 1 => :LVB_ERR_INVALID_ARG, 2 => :LVB_ERR_UNSUPPORTED,
                    3 => :LVB_ERR_CUDA, 4 => :LVB_ERR_TIMEOUT, 5 => :LVB_ERR_NCCL,
                    6 => :LVB_ERR_NO_DEVICE)
const F16, BF16, F32, I8, U8, I32, U32 = Int32.(0:6)
const SUBGROUP, WORKGROUP = Int32(0), Int32(1)

"""16-bit brain float storage type (bit-compatible with BFloat16s.jl's)."""
primitive type BFloat16 <: AbstractFloat 16 end

dtype(::Type{Float16}) = F16
dtype(::Type{BFloat16}) = BF16
dtype(::Type{Float32}) = F32
dtype(::Type{Int8}) = I8
dtype(::Type{UInt8}) = U8
dtype(::Type{Int32}) = I32
dtype(::Type{UInt32}) = U32
function dtype(::Type{T}) where {T}
    # BFloat16s.BFloat16 (if the caller uses that package) has the same bits.
    nameof(T) === :BFloat16 && sizeof(T) == 2 && return BF16
    throw(LavaB200Error("lvb", "no component type for $T", "", 2))
end

struct LavaB200Error <: Exception
    operation::String
    message::String
    suggestion::String
    status::Int
end
Base.showerror(io::IO, e::LavaB200Error) =
    print(io, "LavaB200Error(", STATUS[e.status], ") in ", e.operation, ": ", e.message,
          isempty(e.suggestion) ? "" : " — " * e.suggestion)

function check(st::Integer)
    st == LVB_OK && return nothing
    msg = unsafe_string(ccall(sym(:lvb_last_error), Cstring, ()))
    op, rest = occursin(": ", msg) ? split(msg, ": "; limit = 2) : ("lvb", msg)
    m, hint = occursin(" (", rest) ? split(rest, " ("; limit = 2) : (rest, ")")
    throw(LavaB200Error(String(op), String(m), String(chop(hint)), Int(st)))
end

# ---- C structs ----------------------------------------------------------------------------
struct MatrixShapeC
    ab::Int32; acc::Int32; M::Int32; N::Int32; K::Int32; scope::Int32
end

struct DeviceCapsC
    coopmat::Int32; tile::Int32; subgroup::Int32; coopmatsubgroup::Int32
    sharedbudget::Int64
    workgrouplimit::Int32; cores::Int32; warps::Int32
    n_wggran::Int32
    wggran::NTuple{32,Int32}
    n_shapes::Int32; cc_major::Int32; cc_minor::Int32
end

struct GemmDesc
    a_type::Int32; b_type::Int32; c_type::Int32
    a_rowmajor::Int32; b_rowmajor::Int32; c_rowmajor::Int32
    M::Int64; N::Int64; K::Int64
    lda::Int64; ldb::Int64; ldc::Int64
end

struct Epilogue
    bias::Ptr{Cvoid}; residual::Ptr{Cvoid}
    ldr::Int64
    bias_type::Int32; bias_axis::Int32; residual_type::Int32; activation::Int32
    mul::Ptr{Cvoid}; ldm::Int64; mul_type::Int32; extra_type::Int32
    extra::Ptr{Cvoid}; lde::Int64
    program::Ptr{Cvoid}; k_pad::Int64
    a_clamp::Int32; b_clamp::Int32
    a_clamp_value::Float64; b_clamp_value::Float64
end

# tensor clamp modes (src/vocabulary/tensor.jl:46-51) as `gemm!` takes them
const CLAMPS = Dict{Symbol,Int32}(:undefined => 0, :constant => 1, :edge => 2)
clampspec(::Nothing) = (Int32(0), 0.0)
clampspec(s::Symbol) = s === :edge ? (Int32(2), 0.0) :
    s === :undefined ? (Int32(0), 0.0) : throw(ArgumentError("clamp: :edge, :undefined or a number"))
clampspec(v::Real) = (Int32(1), Float64(v))

include("perelement.jl")

const ACTIVATIONS = Dict{Symbol,Int32}(:none => 0, :relu => 1, :gelu => 2, :gelu_tanh => 2,
                                       :gelu_erf => 3, :silu => 4)

struct AttnDesc
    dtype::Int32; causal::Int32
    batch::Int64; heads_q::Int64; heads_kv::Int64; seq_q::Int64; seq_kv::Int64; head_dim::Int64
    scale::Float32; reserved::Int32
    q_stride::NTuple{3,Int64}; k_stride::NTuple{3,Int64}
    v_stride::NTuple{3,Int64}; o_stride::NTuple{3,Int64}
end

# ---- capabilities ----------------------------------------------------------------------
"""
The backend type a kernel library dispatches on to reach this library: a
`KernelInterface.Backend`, so Lava's backend-form queries (`Lava.matrix_shapes(b)`,
`Lava.supports(b, s)`, `Lava.bestshape(b, ab, acc)`) reach `Lava.caps(b)`, which the Lava
extension answers.
"""
struct B200Backend <: KI.Backend
    device::Int
end
B200Backend() = B200Backend(0)

"""`caps_raw(device)` — the C record; `nothing` device gives the static sm_100a table."""
function caps_raw(device::Union{Nothing,Integer} = nothing)
    r = Ref{DeviceCapsC}()
    if device === nothing
        check(ccall(sym(:lvb_caps_sm100), Cint, (Ptr{DeviceCapsC},), r))
    else
        check(ccall(sym(:lvb_caps), Cint, (Cint, Ptr{DeviceCapsC}), device, r))
    end
    c = r[]
    wg = [ntuple(j -> Int(c.wggran[4(i - 1) + j]), 4) for i in 1:c.n_wggran]
    return (coopmat = c.coopmat != 0, tile = Int(c.tile), subgroup = Int(c.subgroup),
            coopmatsubgroup = Int(c.coopmatsubgroup), sharedbudget = Int(c.sharedbudget),
            workgrouplimit = Int(c.workgrouplimit), cores = Int(c.cores), warps = Int(c.warps),
            wggran = wg)
end

function matrix_shapes_raw()
    n = Ref{Int32}(0)
    check(ccall(sym(:lvb_matrix_shapes), Cint, (Ptr{MatrixShapeC}, Int32, Ptr{Int32}), C_NULL, 0, n))
    v = Vector{MatrixShapeC}(undef, n[])
    check(ccall(sym(:lvb_matrix_shapes), Cint, (Ptr{MatrixShapeC}, Int32, Ptr{Int32}), v, n[], n))
    return v
end

const JULIA_TYPE = Dict(F16 => Float16, BF16 => BFloat16, F32 => Float32, I8 => Int8,
                        U8 => UInt8, I32 => Int32, U32 => UInt32)

# ---- device buffers -----------------------------------------------------------------------
"""
    B200Array{T,N}

An owning, column-major device buffer. `B200Array(host)` uploads, `Array(a)` downloads,
`pointer(a)`/`size(a)` make it usable wherever a `LavaDeviceArray` would be.
"""
mutable struct B200Array{T,N}
    ptr::Ptr{T}
    dims::NTuple{N,Int}
    function B200Array{T,N}(::UndefInitializer, dims::NTuple{N,Int}) where {T,N}
        p = Ref{Ptr{Cvoid}}(C_NULL)
        nbytes = max(prod(dims; init = 1) * sizeof(T), 1)
        check(ccall(sym(:lvb_malloc), Cint, (Ptr{Ptr{Cvoid}}, Csize_t), p, nbytes))
        a = new{T,N}(Ptr{T}(p[]), dims)
        finalizer(a) do x
            x.ptr == C_NULL || ccall(sym(:lvb_free), Cint, (Ptr{Cvoid},), x.ptr)
            x.ptr = C_NULL
        end
        return a
    end
end
B200Array{T}(::UndefInitializer, dims::Integer...) where {T} =
    B200Array{T,length(dims)}(undef, Int.(dims))
function B200Array(h::Array{T,N}) where {T,N}
    a = B200Array{T,N}(undef, size(h))
    copyto!(a, h)
    return a
end
Base.size(a::B200Array) = a.dims
Base.size(a::B200Array, i::Integer) = i <= length(a.dims) ? a.dims[i] : 1
Base.pointer(a::B200Array) = a.ptr
Base.eltype(::B200Array{T}) where {T} = T
Base.length(a::B200Array) = prod(a.dims; init = 1)

function Base.copyto!(a::B200Array{T}, h::Array{T}; stream = C_NULL) where {T}
    length(h) == length(a) || throw(DimensionMismatch("sizes differ"))
    GC.@preserve h check(ccall(sym(:lvb_memcpy_htod), Cint, (Ptr{Cvoid}, Ptr{Cvoid}, Csize_t, Ptr{Cvoid}),
                               a.ptr, pointer(h), sizeof(h), stream))
    check(ccall(sym(:lvb_stream_synchronize), Cint, (Ptr{Cvoid},), stream))
    return a
end
function Base.copyto!(h::Array{T}, a::B200Array{T}; stream = C_NULL) where {T}
    length(h) == length(a) || throw(DimensionMismatch("sizes differ"))
    GC.@preserve h check(ccall(sym(:lvb_memcpy_dtoh), Cint, (Ptr{Cvoid}, Ptr{Cvoid}, Csize_t, Ptr{Cvoid}),
                               pointer(h), a.ptr, sizeof(h), stream))
    check(ccall(sym(:lvb_stream_synchronize), Cint, (Ptr{Cvoid},), stream))
    return h
end
Base.Array(a::B200Array{T,N}) where {T,N} = copyto!(Array{T,N}(undef, a.dims), a)

# ---- operand layout -----------------------------------------------------------------------
# (pointer, rows, cols, rowmajor, ld) of a matrix operand. A plain device matrix is
# column-major with ld = size(x, 1); `transpose(x)` of a column-major (cols × rows) matrix is
# the row-major (rows × cols) operand with ld = size(x, 1).
layout(x) = (pointer(x), size(x, 1), size(x, 2), Int32(0), max(size(x, 1), 1))
function layout(x::Transpose)
    p = parent(x)
    return (pointer(p), size(p, 2), size(p, 1), Int32(1), max(size(p, 1), 1))
end
elt(x) = eltype(x)
elt(x::Transpose) = eltype(parent(x))

"""
    gemm!(C, A, B; bias = nothing, bias_axis = :row, residual = nothing, activation = :none,
          mul = nothing, perelement = nothing, extra = nothing, k_pad = nothing,
          a_clamp = nothing, b_clamp = nothing, stream = C_NULL) -> C

`C = activation(A·B + bias + residual)` on the GPU. Any layout: a plain device matrix is
column-major, its `transpose` row-major (Lava's `Val(true)` load); A column-major / B row-major
are read MN-major by the tensor core (16-bit types) — Lava's transposing tensor view.

The epilogue is optional: `bias` a device vector added per row (`bias_axis = :row`, length M,
Lava's stride-0 accumulator load) or per column (`:col`, length N); `residual` an M×N device
matrix in C's layout (may be `C` itself); `activation` one of `:none, :relu, :gelu`
(tanh form), `:gelu_erf, :silu` — the accumulator initialised with `coopmat_add(bias,
residual)` and finished with `coopmat_perelement` (src/device/coopmat_intrinsics.jl:
435-447,551-593). Floating-point outputs only.

More of the vocabulary on the same epilogue: `mul` an M×N matrix in C's layout multiplying
the accumulator element-wise (`coopmat_mul`, src/device/coopmat_intrinsics.jl:402-464);
`perelement` a function `(x, row, col, e) -> value` applied to every element with its 0-based
row and column and the element `e` of the optional matrix `extra` (`coopmat_perelement`,
coopmat_intrinsics.jl:520-678), traced once into the library's per-element program
(`pe_program`); `k_pad` a padded k extent whose reads past `K` take `a_clamp` / `b_clamp`
(`nothing`, `:edge` or a constant: TENSOR_CLAMP_TO_EDGE / TENSOR_CLAMP_CONSTANT,
src/vocabulary/tensor.jl:46-51). The result is
`perelement(activation((A·B + bias + residual) .* mul))`.

A device vector as `B` and `C` (N == 1), or a 1×K `A` (M == 1), is a matrix-vector product:
it runs on the library's HBM-bound streaming kernel — `dot4x8` for Int8/UInt8 operands
(src/vocabulary/vocabulary.jl:18-35), fp32 multiply-adds for Float16/BFloat16 — with the
same results and epilogue.
"""
function gemm!(C, A, B; bias = nothing, bias_axis::Symbol = :row, residual = nothing,
               activation::Symbol = :none, mul = nothing, perelement = nothing,
               extra = nothing, k_pad = nothing, a_clamp = nothing, b_clamp = nothing,
               stream::Ptr{Cvoid} = C_NULL)
    pa, M, K, ra, lda = layout(A)
    pb, K2, N, rb, ldb = layout(B)
    pc, M2, N2, rc, ldc = layout(C)
    (K2 == K && M2 == M && N2 == N) ||
        throw(DimensionMismatch("gemm!: ($M×$K)·($K2×$N) -> ($M2×$N2)"))
    d = GemmDesc(dtype(elt(A)), dtype(elt(B)), dtype(elt(C)), ra, rb, rc, M, N, K, lda, ldb, ldc)
    if bias === nothing && residual === nothing && activation === :none && mul === nothing &&
       perelement === nothing && k_pad === nothing
        check(ccall(sym(:lvb_gemm), Cint,
                    (Ref{GemmDesc}, Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}),
                    d, pa, pb, pc, stream))
        return C
    end
    haskey(ACTIVATIONS, activation) ||
        throw(ArgumentError("gemm!: activation must be one of $(collect(keys(ACTIVATIONS)))"))
    bias_axis in (:row, :col) || throw(ArgumentError("gemm!: bias_axis must be :row or :col"))
    pbias, tbias = C_NULL, Int32(2)
    if bias !== nothing
        length(bias) == (bias_axis === :row ? M : N) ||
            throw(DimensionMismatch("gemm!: bias of length $(length(bias)) for $bias_axis of ($M×$N)"))
        pbias, tbias = pointer(bias), dtype(eltype(bias))
    end
    # an M×N epilogue operand in C's layout: (pointer, type, leading dimension)
    function cmatrix(x, what)
        px, Mx, Nx, rx, ldx = layout(x)
        (Mx == M && Nx == N && rx == rc) ||
            throw(DimensionMismatch("gemm!: $what must be ($M×$N) in C's layout"))
        return Ptr{Cvoid}(px), dtype(elt(x)), Int64(ldx)
    end
    pres, tres, ldr = residual === nothing ? (C_NULL, Int32(2), Int64(0)) : cmatrix(residual, "residual")
    pmul, tmul, ldm = mul === nothing ? (C_NULL, Int32(2), Int64(0)) : cmatrix(mul, "mul")
    prog = perelement === nothing ? nothing :
           perelement isa PeProgram ? perelement : pe_program(perelement)
    pext, text, lde = extra === nothing ? (C_NULL, Int32(2), Int64(0)) : cmatrix(extra, "extra")
    (extra === nothing || prog !== nothing) ||
        throw(ArgumentError("gemm!: extra is the perelement function's matrix operand"))
    ca, va = clampspec(a_clamp)
    cb, vb = clampspec(b_clamp)
    progref = Ref(prog === nothing ? PeProgram(Int32(0), ntuple(_ -> PeInstr(0, 0, 0, 0, 0), 32)) : prog)
    GC.@preserve progref begin
        pprog = prog === nothing ? C_NULL : Ptr{Cvoid}(Base.unsafe_convert(Ptr{PeProgram}, progref))
        e = Epilogue(pbias, pres, ldr, tbias, Int32(bias_axis === :row ? 0 : 1), tres,
                     ACTIVATIONS[activation], pmul, ldm, tmul, text, pext, lde, pprog,
                     k_pad === nothing ? Int64(0) : Int64(k_pad), ca, cb, va, vb)
        check(ccall(sym(:lvb_gemm_ex), Cint,
                    (Ref{GemmDesc}, Ref{Epilogue}, Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}),
                    d, e, pa, pb, pc, stream))
    end
    return C
end

"""
    attention!(O, Q, K, V; causal = true, scale = 1/sqrt(E), lse = nothing, stream = C_NULL)

Flash-attention forward. Q, O: `(E, Lq, Hq, B)`; K, V: `(E, Lk, Hkv, B)` (column-major,
dense); `lse` (optional, Float32 `(Lq, Hq, B)`) receives the natural-log row log-sum-exp.
With at most 32 query rows per KV head (`Lq · Hq/Hkv <= 32`, E = 128) — decoding against a
KV cache — the library streams the cache once, split over the keys, instead.
"""
function attention!(O, Q, K, V; causal::Bool = true, scale::Real = inv(sqrt(size(Q, 1))),
                    lse = nothing, stream::Ptr{Cvoid} = C_NULL)
    E, Lq, Hq, Bq = size(Q, 1), size(Q, 2), size(Q, 3), size(Q, 4)
    E2, Lk, Hkv, Bk = size(K, 1), size(K, 2), size(K, 3), size(K, 4)
    (E2 == E && Bk == Bq && size(V) == size(K) && size(O) == size(Q)) ||
        throw(DimensionMismatch("attention!: Q $(size(Q)) K $(size(K)) V $(size(V)) O $(size(O))"))
    z = (0, 0, 0)
    d = AttnDesc(dtype(eltype(Q)), Int32(causal), Bq, Hq, Hkv, Lq, Lk, E, Float32(scale), 0,
                 z, z, z, z)
    pl = lse === nothing ? C_NULL : pointer(lse)
    check(ccall(sym(:lvb_attention_fwd), Cint,
                (Ref{AttnDesc}, Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}),
                d, pointer(Q), pointer(K), pointer(V), pointer(O), pl, stream))
    return O
end

"""Synchronise `stream` and read/clear the device status word: `(code, where, block)`."""
function device_status(stream::Ptr{Cvoid} = C_NULL)
    c, w, b = Ref{Int32}(0), Ref{Int32}(0), Ref{Int32}(0)
    check(ccall(sym(:lvb_device_status), Cint, (Ptr{Cvoid}, Ptr{Int32}, Ptr{Int32}, Ptr{Int32}),
                stream, c, w, b))
    return (Int(c[]), Int(w[]), Int(b[]))
end

function synchronize(stream::Ptr{Cvoid} = C_NULL)
    check(ccall(sym(:lvb_stream_synchronize), Cint, (Ptr{Cvoid},), stream))
end

function device_count()
    n = Ref{Int32}(0)
    check(ccall(sym(:lvb_device_count), Cint, (Ptr{Int32},), n))
    return Int(n[])
end

# ---- several GPUs: shards and the optional all-gather -----------------------------------
# Lava's runtime is single-device; the units of this path are independent (GEMM output rows
# with B replicated, attention (batch, KV head) groups), so each process computes its share
# on its own GPU and nothing is exchanged unless the caller wants the whole output on every
# GPU (include/lvb.h: lvb_shard_range, lvb_comm_*, lvb_allgather).

"""
    shard_range(total, world, rank; align = 1) -> (first, count)

`rank`'s contiguous share of `total` units (0-based `first`), made of whole chunks of
`align` units; for GEMM rows use `align = 128` (one tile of rows).
"""
function shard_range(total::Integer, world::Integer, rank::Integer; align::Integer = 1)
    b, n = Ref{Int64}(0), Ref{Int64}(0)
    check(ccall(sym(:lvb_shard_range), Cint, (Int64, Int32, Int32, Int64, Ptr{Int64}, Ptr{Int64}),
                total, world, rank, align, b, n))
    return (Int(b[]), Int(n[]))
end

"""
    comm_unique_id() -> Vector{UInt8}

A fresh 128-byte communicator id, made on one process (rank 0) and handed to the others by
the host's own channel (a file, MPI, a socket).
"""
function comm_unique_id()
    id = zeros(UInt8, 128)
    GC.@preserve id check(ccall(sym(:lvb_comm_unique_id), Cint, (Ptr{UInt8},), id))
    return id
end

"""
    Comm(id, nranks, rank)

Join the communicator `id` as `rank` of `nranks` on the current device (NCCL over
NVLink/NVSwitch underneath); every rank must construct it. Released by `close` or the GC.
"""
mutable struct Comm
    handle::Ptr{Cvoid}
    nranks::Int
    rank::Int
    function Comm(id::AbstractVector{UInt8}, nranks::Integer, rank::Integer)
        length(id) == 128 || throw(ArgumentError("a communicator id has 128 bytes"))
        buf = Vector{UInt8}(id)
        h = Ref{Ptr{Cvoid}}(C_NULL)
        GC.@preserve buf check(ccall(sym(:lvb_comm_init), Cint,
                                     (Ptr{Ptr{Cvoid}}, Ptr{UInt8}, Int32, Int32),
                                     h, buf, nranks, rank))
        c = new(h[], Int(nranks), Int(rank))
        finalizer(c) do x          # no exceptions from a finalizer: the status is dropped
            if x.handle != C_NULL
                ccall(sym(:lvb_comm_destroy), Cint, (Ptr{Cvoid},), x.handle)
                x.handle = C_NULL
            end
        end
        return c
    end
end

function Base.close(c::Comm)
    if c.handle != C_NULL
        h, c.handle = c.handle, C_NULL
        check(ccall(sym(:lvb_comm_destroy), Cint, (Ptr{Cvoid},), h))
    end
    return nothing
end

"""
    allgather!(recv, send, comm; stream = C_NULL)

Enqueue on `stream`: `recv` (nranks × the bytes of `send`) receives every rank's `send` in
rank order. `recv` and `send` are any device values with `pointer`, `length` and `eltype`
(a `B200Array`, a `Lava.LavaDeviceArray`). Shards of equal size: pad a short last shard. With column-major Julia arrays a
gather of row shards is a gather of the shards of Cᵀ (compute Cᵀ = BᵀAᵀ per shard, or
shard by output columns).
"""
function allgather!(recv, send, comm::Comm; stream = C_NULL)
    T = eltype(send)
    eltype(recv) === T || throw(ArgumentError("allgather!: recv and send element types differ"))
    nb = sizeof(T) * length(send)
    sizeof(T) * length(recv) == nb * comm.nranks ||
        throw(DimensionMismatch("recv must hold nranks × the elements of send"))
    check(ccall(sym(:lvb_allgather), Cint, (Ptr{Cvoid}, Ptr{Cvoid}, Ptr{Cvoid}, Csize_t, Ptr{Cvoid}),
                comm.handle, pointer(send), pointer(recv), nb, stream))
    return recv
end

end # module
