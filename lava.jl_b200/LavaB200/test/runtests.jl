# LavaB200 tests. Tier 1 (no GPU): the library loads, caps/shape answers, argument errors.
# Tier 2 (GPU, when a B200 is visible): gemm!/attention! against a host reference.
using Test
using LavaB200
using LinearAlgebra

@testset "LavaB200" begin
    @testset "caps (no GPU)" begin
        c = caps_raw()
        @test c.coopmat && c.tile == 16 && c.subgroup == 32 && c.cores == 148
        shapes = matrix_shapes_raw()
        @test any(s -> s.M == 16 && s.N == 16 && s.K == 16 && s.ab == LavaB200.F16 &&
                       s.acc == LavaB200.F32, shapes)
    end

    @testset "argument errors surface as LavaB200Error" begin
        d = LavaB200.GemmDesc(LavaB200.F16, LavaB200.F16, LavaB200.I32, 1, 0, 0, 64, 64, 64,
                              64, 64, 64)
        st = ccall(LavaB200.sym(:lvb_gemm_check), Cint, (Ref{LavaB200.GemmDesc},), d)
        @test st == LavaB200.LVB_ERR_UNSUPPORTED
        err = try
            LavaB200.check(st)
        catch e
            e
        end
        @test err isa LavaB200Error && err.operation == "lvb_gemm"
    end

    @testset "B200Backend is a KernelInterface.Backend (no GPU)" begin
        @test B200Backend() isa LavaB200.KI.Backend
    end

    # Lava's backend-form queries dispatch on `backend::KI.Backend` and reach `Lava.caps`
    # (src/vocabulary/caps.jl:158-169, src/vocabulary/matrix.jl:138-141); with the extension
    # loaded they answer for a B200 from the library's static sm_100a table.
    if Base.find_package("Lava") !== nothing
        @eval using Lava
        @testset "Lava backend-form queries (no GPU)" begin
            b = B200Backend()
            shapes = Lava.matrix_shapes(b)
            @test !isempty(shapes)
            s = Lava.bestshape(b, Float16, Float32)
            @test s isa Lava.MatrixShape && s.M == 16 && s.N == 16 && s.K == 16
            @test Lava.supports(b, s)
            @test Lava.bestshape(b, Int8, Int32) isa Lava.MatrixShape
            @test Lava.bestshape(b, Float32, Float32) === nothing
        end
    else
        @info "Lava not installed: backend-form query tests not run"
    end

    @testset "per-element programs are traced (no GPU)" begin
        p = pe_program((x, r, c, e) -> x * 2.0f0 + c)
        ops = [p.code[i].op for i in 1:p.n]
        @test LavaB200.PE_OPS[:FMUL] in ops && LavaB200.PE_OPS[:I2F] in ops &&
              LavaB200.PE_OPS[:FADD] in ops && p.n <= 32
        q = pe_program((x, r, c, e) -> pe_ifelse(c > r, -Inf32, 0.125f0 * x))
        @test LavaB200.PE_OPS[:SELECT] in [q.code[i].op for i in 1:q.n]
        st = ccall(LavaB200.sym(:lvb_pe_program_check), Cint, (Ref{PeProgram},), q)
        @test st == 0
        @test_throws TypeError pe_program((x, r, c, e) -> x > 0 ? x : -x)   # non-Bool condition
    end

    @testset "shards and communicator ids (no GPU)" begin
        @test [shard_range(1000, 2, r; align = 128) for r in 0:1] == [(0, 512), (512, 488)]
        id = comm_unique_id()
        @test length(id) == 128 && id != comm_unique_id()
        @test_throws LavaB200Error Comm(zeros(UInt8, 128), 2, 2)
    end

    if LavaB200.device_count() > 0
        @testset "gemm! Float16 -> Float32 (GPU)" begin
            M, N, K = 300, 200, 136
            A = Float16.(rand(Float32, K, M) .* 2 .- 1)    # storage of row-major A (M×K)
            B = Float16.(rand(Float32, K, N) .* 2 .- 1)    # column-major B (K×N)
            dA, dB = B200Array(A), B200Array(B)
            dC = B200Array{Float32}(undef, M, N)
            gemm!(dC, transpose(dA), dB)
            C = Array(dC)
            ref = Float64.(transpose(A)) * Float64.(B)
            @test maximum(abs.(C .- ref)) <= 1e-2
            @test device_status() == (0, 0, 0)
        end
        @testset "gemm! column-major A, fused bias + residual + relu (GPU)" begin
            M, N, K = 256, 192, 320
            A = Float16.(rand(Float32, M, K) .* 2 .- 1)    # column-major A: read MN-major
            B = Float16.(rand(Float32, K, N) .* 2 .- 1)
            bias = rand(Float32, M) .- 0.5f0
            R = rand(Float32, M, N) .- 0.5f0
            dC = B200Array(copy(R))                        # residual = C itself
            gemm!(dC, B200Array(A), B200Array(B); bias = B200Array(bias), bias_axis = :row,
                  residual = dC, activation = :relu)
            ref = max.(Float64.(A) * Float64.(B) .+ Float64.(bias) .+ Float64.(R), 0.0)
            @test maximum(abs.(Array(dC) .- ref)) <= 1e-2
            @test device_status() == (0, 0, 0)
        end
        @testset "gemm! coopmat_mul, per-element function, clamps (GPU)" begin
            M, N, K = 200, 136, 100
            A = Float16.(rand(Float32, M, K) .* 2 .- 1)
            B = Float16.(rand(Float32, K, N) .* 2 .- 1)
            S = rand(Float32, M, N) .* 2 .- 1
            E = rand(Float32, M, N) .- 0.5f0
            dC = B200Array{Float32}(undef, M, N)
            gemm!(dC, B200Array(A), B200Array(B); mul = B200Array(S), extra = B200Array(E),
                  perelement = (x, r, c, e) -> pe_ifelse(c > r, -Inf32, 0.5f0 * x + e))
            P = (Float64.(A) * Float64.(B)) .* S
            ref = [j - 1 > i - 1 ? -Inf : 0.5 * P[i, j] + E[i, j] for i in 1:M, j in 1:N]
            got = Array(dC)
            @test all(isinf.(got) .== isinf.(ref))
            fin = .!isinf.(ref)
            @test maximum(abs.(got[fin] .- ref[fin])) <= 1e-2
            # TO_EDGE on A and the constant 0.5 on B over k_pad = 128
            gemm!(dC, B200Array(A), B200Array(B); k_pad = 128, a_clamp = :edge, b_clamp = 0.5)
            Ap = hcat(Float64.(A), repeat(Float64.(A[:, end]), 1, 28))
            Bp = vcat(Float64.(B), fill(0.5, 28, N))
            @test maximum(abs.(Array(dC) .- Ap * Bp)) <= 1e-2
            @test device_status() == (0, 0, 0)
        end
        @testset "gemm! Int8 exact (GPU)" begin
            M, N, K = 130, 70, 256
            A = rand(Int8, K, M); B = rand(Int8, K, N)
            dC = B200Array{Int32}(undef, M, N)
            gemm!(dC, transpose(B200Array(A)), B200Array(B))
            @test Array(dC) == Int32.(transpose(Int64.(A)) * Int64.(B))
        end
        @testset "attention! causal GQA (GPU)" begin
            E, L, Hq, Hkv, Bt = 128, 256, 4, 2, 1
            Q = Float16.(randn(Float32, E, L, Hq, Bt))
            K = Float16.(randn(Float32, E, L, Hkv, Bt))
            V = Float16.(randn(Float32, E, L, Hkv, Bt))
            dO = B200Array{Float16}(undef, E, L, Hq, Bt)
            attention!(dO, B200Array(Q), B200Array(K), B200Array(V); causal = true)
            O = Float64.(Array(dO))
            g = Hq ÷ Hkv
            for h in 1:Hq
                q = Float64.(Q[:, :, h, 1]); k = Float64.(K[:, :, (h - 1) ÷ g + 1, 1])
                v = Float64.(V[:, :, (h - 1) ÷ g + 1, 1])
                s = (k' * q) ./ sqrt(E)                       # (Lk, Lq)
                for i in 1:L, j in 1:L
                    j > i && (s[j, i] = -Inf)
                end
                p = exp.(s .- maximum(s; dims = 1))
                ref = v * (p ./ sum(p; dims = 1))
                @test maximum(abs.(O[:, :, h, 1] .- ref)) <= 1e-2
            end
        end
    else
        @info "no GPU visible: GPU tier not run"
    end
end
