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

}  // namespace lvb
