// epilogue.cuh — per-element device helpers shared by the GEMM and GEMV kernels: operand
// loads converted to fp32, and the activation a Lava GEMM applies to its accumulator with
// coopmat_perelement (src/device/coopmat_intrinsics.jl:322-331,551-593).
#pragma once

#include "sm100.cuh"
#include "lvb.h"

namespace lvb {

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

__device__ __forceinline__ float load_as_f32(const void* p, int kind, long long i) {
  if (kind == LVB_F32) return reinterpret_cast<const float*>(p)[i];
  if (kind == LVB_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}

// The per-element function of the epilogue (coopmat_perelement with a fixed callback).
// gelu-tanh 0.5x(1 + tanh(u)) and silu are evaluated as x·sigmoid(t) = x / (1 + e^-t)
// (t = 2u and t = x): the same functions, with no cancellation for negative arguments
// (1 + tanh(u) -> 0) and a limit of -0 where e^-t overflows. gelu-erf as 0.5x·erfc(-x/√2),
// which equals 0.5x(1 + erf(x/√2)) without the same cancellation.
template <int ACT>
__device__ __forceinline__ float act_fn(float v) {
  if constexpr (ACT == LVB_ACT_RELU) {
    return v < 0.f ? 0.f : v;  // NaN passes through, as max(x, 0) does in Julia
  } else if constexpr (ACT == LVB_ACT_GELU_TANH) {
    const float t = 1.5957691216057308f * fmaf(0.044715f * v, v * v, v);  // 2·sqrt(2/pi)·(...)
    return __fdividef(v, 1.f + __expf(-t));
  } else if constexpr (ACT == LVB_ACT_GELU_ERF) {
    return 0.5f * v * erfcf(-0.7071067811865476f * v);
  } else if constexpr (ACT == LVB_ACT_SILU) {
    return __fdividef(v, 1.f + __expf(-v));
  } else {
    return v;
  }
}

__device__ __forceinline__ float act_any(int act, float v) {
  switch (act) {
    case LVB_ACT_RELU: return act_fn<LVB_ACT_RELU>(v);
    case LVB_ACT_GELU_TANH: return act_fn<LVB_ACT_GELU_TANH>(v);
    case LVB_ACT_GELU_ERF: return act_fn<LVB_ACT_GELU_ERF>(v);
    case LVB_ACT_SILU: return act_fn<LVB_ACT_SILU>(v);
  }
  return v;
}

// ---------------------------------------------------------------------------------------
// Caller-supplied per-element programs (lvb_pe_program): coopmat_perelement(f, m, extras...)
// with a function the caller writes, evaluated W elements at a time. The program is the same
// for every thread (it sits in the kernel's parameters), so every switch below branches
// uniformly; the 8 registers of the W elements stay in registers because each is named by a
// constant index inside a case.
// ---------------------------------------------------------------------------------------
struct PeProgram {
  int n;
  lvb_pe_instr code[LVB_PE_MAX_INSTR];
};

template <int W>
__device__ __forceinline__ void pe_get(const uint32_t (&R)[LVB_PE_REGS][W], int r,
                                       uint32_t (&o)[W]) {
  switch (r) {
#define LVB_PE_GET(i) \
  case i:             \
    _Pragma("unroll") for (int e = 0; e < W; ++e) o[e] = R[i][e]; break;
    LVB_PE_GET(0) LVB_PE_GET(1) LVB_PE_GET(2) LVB_PE_GET(3)
    LVB_PE_GET(4) LVB_PE_GET(5) LVB_PE_GET(6) LVB_PE_GET(7)
#undef LVB_PE_GET
  }
}

template <int W>
__device__ __forceinline__ void pe_set(uint32_t (&R)[LVB_PE_REGS][W], int r,
                                       const uint32_t (&v)[W]) {
  switch (r) {
#define LVB_PE_SET(i) \
  case i:             \
    _Pragma("unroll") for (int e = 0; e < W; ++e) R[i][e] = v[e]; break;
    LVB_PE_SET(0) LVB_PE_SET(1) LVB_PE_SET(2) LVB_PE_SET(3)
    LVB_PE_SET(4) LVB_PE_SET(5) LVB_PE_SET(6) LVB_PE_SET(7)
#undef LVB_PE_SET
  }
}

__device__ __forceinline__ float pe_f(uint32_t u) { return __uint_as_float(u); }
__device__ __forceinline__ uint32_t pe_u(float f) { return __float_as_uint(f); }

// x[e] <- f(x[e], row[e], col[e], ext[e]) for W elements.
template <int W>
__device__ __forceinline__ void pe_run(const PeProgram& pg, float (&x)[W], const int (&row)[W],
                                       const int (&col)[W], const float (&ext)[W]) {
  uint32_t R[LVB_PE_REGS][W];
#pragma unroll
  for (int e = 0; e < W; ++e) {
    R[0][e] = pe_u(x[e]);
    R[1][e] = (uint32_t)row[e];
    R[2][e] = (uint32_t)col[e];
    R[3][e] = pe_u(ext[e]);
#pragma unroll
    for (int r = 4; r < LVB_PE_REGS; ++r) R[r][e] = 0u;
  }
#pragma unroll 1
  for (int i = 0; i < pg.n; ++i) {
    const lvb_pe_instr I = pg.code[i];
    uint32_t A[W], B[W], D[W];
    pe_get<W>(R, I.a, A);
    pe_get<W>(R, I.b, B);
    if (I.op == LVB_PE_FFMA || I.op == LVB_PE_SELECT) pe_get<W>(R, I.dst, D);
#define LVB_PE_EACH(expr) \
  _Pragma("unroll") for (int e = 0; e < W; ++e) D[e] = (expr); break;
    switch (I.op) {
      case LVB_PE_CONST: LVB_PE_EACH(I.imm)
      case LVB_PE_ICONST: LVB_PE_EACH(I.imm)
      case LVB_PE_MOV: LVB_PE_EACH(A[e])
      case LVB_PE_FADD: LVB_PE_EACH(pe_u(pe_f(A[e]) + pe_f(B[e])))
      case LVB_PE_FSUB: LVB_PE_EACH(pe_u(pe_f(A[e]) - pe_f(B[e])))
      case LVB_PE_FMUL: LVB_PE_EACH(pe_u(pe_f(A[e]) * pe_f(B[e])))
      case LVB_PE_FDIV: LVB_PE_EACH(pe_u(pe_f(A[e]) / pe_f(B[e])))
      case LVB_PE_FMIN: LVB_PE_EACH(pe_u(fminf(pe_f(A[e]), pe_f(B[e]))))
      case LVB_PE_FMAX: LVB_PE_EACH(pe_u(fmaxf(pe_f(A[e]), pe_f(B[e]))))
      case LVB_PE_FFMA: LVB_PE_EACH(pe_u(fmaf(pe_f(A[e]), pe_f(B[e]), pe_f(D[e]))))
      case LVB_PE_FNEG: LVB_PE_EACH(A[e] ^ 0x80000000u)
      case LVB_PE_FABS: LVB_PE_EACH(A[e] & 0x7fffffffu)
      case LVB_PE_FEXP: LVB_PE_EACH(pe_u(expf(pe_f(A[e]))))
      case LVB_PE_FEXP2: LVB_PE_EACH(pe_u(exp2f(pe_f(A[e]))))
      case LVB_PE_FLOG: LVB_PE_EACH(pe_u(logf(pe_f(A[e]))))
      case LVB_PE_FTANH: LVB_PE_EACH(pe_u(tanhf(pe_f(A[e]))))
      case LVB_PE_FSQRT: LVB_PE_EACH(pe_u(sqrtf(pe_f(A[e]))))
      case LVB_PE_FRSQRT: LVB_PE_EACH(pe_u(1.f / sqrtf(pe_f(A[e]))))
      case LVB_PE_FFLOOR: LVB_PE_EACH(pe_u(floorf(pe_f(A[e]))))
      case LVB_PE_FERF: LVB_PE_EACH(pe_u(erff(pe_f(A[e]))))
      case LVB_PE_I2F: LVB_PE_EACH(pe_u(__int2float_rn((int)A[e])))
      case LVB_PE_IADD: LVB_PE_EACH(A[e] + B[e])
      case LVB_PE_ISUB: LVB_PE_EACH(A[e] - B[e])
      case LVB_PE_IMUL: LVB_PE_EACH(A[e] * B[e])
      case LVB_PE_IMIN: LVB_PE_EACH((uint32_t)min((int)A[e], (int)B[e]))
      case LVB_PE_IMAX: LVB_PE_EACH((uint32_t)max((int)A[e], (int)B[e]))
      case LVB_PE_FLT: LVB_PE_EACH(pe_f(A[e]) < pe_f(B[e]) ? 1u : 0u)
      case LVB_PE_FLE: LVB_PE_EACH(pe_f(A[e]) <= pe_f(B[e]) ? 1u : 0u)
      case LVB_PE_FEQ: LVB_PE_EACH(pe_f(A[e]) == pe_f(B[e]) ? 1u : 0u)
      case LVB_PE_ILT: LVB_PE_EACH((int)A[e] < (int)B[e] ? 1u : 0u)
      case LVB_PE_ILE: LVB_PE_EACH((int)A[e] <= (int)B[e] ? 1u : 0u)
      case LVB_PE_IEQ: LVB_PE_EACH(A[e] == B[e] ? 1u : 0u)
      case LVB_PE_SELECT: LVB_PE_EACH(A[e] ? B[e] : D[e])
      default: LVB_PE_EACH(0u)
    }
#undef LVB_PE_EACH
    pe_set<W>(R, I.dst, D);
  }
#pragma unroll
  for (int e = 0; e < W; ++e) x[e] = pe_f(R[0][e]);
}

// An operand element as int32 (8-bit operands) or fp32 (16-bit ones) for the clamp term.
__device__ __forceinline__ float operand_f32(const void* p, int ab, long long i) {
  if (ab == 0) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}
__device__ __forceinline__ int operand_i32(const void* p, int ab, long long i) {
  if (ab == 2) return (int)reinterpret_cast<const int8_t*>(p)[i];
  return (int)reinterpret_cast<const uint8_t*>(p)[i];
}

}  // namespace lvb
