"""
The bridge to Lava.jl's vocabulary, loaded when `Lava` is: `Lava.caps(::B200Backend)`
answers with Lava's own `DeviceCaps` (src/vocabulary/caps.jl:54-82) and `MatrixShape`
table (src/vocabulary/matrix.jl:88-95), so `matrix_shapes`, `supports`, `bestshape` and
`wggranularity` work unchanged; the `supports_*` predicates answer for the fused kernels.
`gemm!` / `attention!` accept `Lava.LavaDeviceArray` directly (it has `pointer`/`size`).
"""
module LavaB200LavaExt

using LavaB200
import Lava

const TYPES = Dict(LavaB200.F16 => Float16, LavaB200.BF16 => LavaB200.BFloat16,
                   LavaB200.F32 => Float32, LavaB200.I8 => Int8, LavaB200.U8 => UInt8,
                   LavaB200.I32 => Int32, LavaB200.U32 => UInt32)

function lava_shapes(scope)
    out = Lava.MatrixShape[]
    for s in LavaB200.matrix_shapes_raw()
        s.scope == scope || continue
        sc = s.scope == LavaB200.SUBGROUP ? Lava.SubgroupScope() : Lava.WorkgroupScope()
        push!(out, Lava.MatrixShape(TYPES[s.ab], TYPES[s.acc], Int(s.M), Int(s.N), Int(s.K), sc))
    end
    return out
end

function Lava.caps(b::LavaB200.B200Backend)
    c = LavaB200.caps_raw(b.device)
    return Lava.DeviceCaps(c.coopmat, c.tile, c.subgroup, c.coopmatsubgroup, c.sharedbudget,
                           c.workgrouplimit, c.cores, c.warps, c.wggran,
                           lava_shapes(LavaB200.SUBGROUP))
end

# The fused kernels implement per-element application, row reduction and clamped tensor
# addressing (ragged edges) on this device.
Lava.supports_coopmat_perelement(::LavaB200.B200Backend) = true
Lava.supports_coopmat_reduce(::LavaB200.B200Backend) = true
Lava.supports_tensor_addressing(::LavaB200.B200Backend) = true
Lava.supports_flexible_coopmat_shapes(::LavaB200.B200Backend) = true

end # module
