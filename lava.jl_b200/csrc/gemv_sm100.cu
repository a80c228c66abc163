// gemv_sm100.cu — matrix-vector products for B200 (sm_100a): lvb_gemm / lvb_gemm_ex with
// N == 1 (y = A·x) or M == 1 (yᵀ = xᵀ·B).
//
// A product with one output column reads every matrix element once and does one
// multiply-add with it, so it is bound by HBM bandwidth, not by the tensor core: a 128-row
// tcgen05 tile would waste 127/128 of its work and, worse, serialise the matrix stream behind
// one output column. These kernels stream the matrix with 16-byte loads and do the
// multiply-adds on the CUDA cores:
//   * int8 / uint8: dot4x8 — four 8-bit products summed exactly into 32 bits in one
//     instruction (dp4a), Lava's `dot4x8` (src/vocabulary/vocabulary.jl:18-35) whose stated
//     purpose is exactly this int8 matrix-vector product;
//   * fp16 / bf16: widened to fp32 and accumulated in fp32, as coopmat_muladd does
//     (src/vocabulary/coopmat.jl:190-203).
// The output goes through the same fused epilogue as the GEMM (bias + residual accumulator
// initialisation, activation, round-to-nearest-even conversion).
//
// Two layouts of the matrix W (R rows of K elements):
//   * K-contiguous (A row-major, or Bᵀ of a column-major B): one warp per row, lanes stride
//     along k, a shuffle reduction at the end;
//   * R-contiguous (A column-major — Julia's default — or Bᵀ of a row-major B): a CTA owns
//     8·E consecutive rows (E elements per 16 bytes); 8 threads cover them with 16-byte
//     loads and 32 threads split k; a shared-memory reduction over the k threads.
// When the rows alone cannot fill the GPU, k is split across CTAs as well: each split
// writes fp32 / int32 partial sums to a stream-ordered workspace and a second kernel adds the
// splits in a fixed order (deterministic results) and applies the epilogue.
#include <algorithm>
#include <cstdint>
#include <type_traits>

#include "epilogue.cuh"
#include "lvb_internal.h"

namespace lvb {

namespace {

enum GvAb { GV_F16 = 0, GV_BF16 = 1, GV_S8 = 2, GV_U8 = 3 };
enum GvOut { GV_OUT_F32 = 0, GV_OUT_F16 = 1, GV_OUT_BF16 = 2, GV_OUT_I32 = 3 };

constexpr int kGvThreads = 256;

struct GemvParams {
  const void* W;
  long long sr, sk;       // W[r*sr + k*sk] (elements); sk == 1 or sr == 1
  const void* X;
  long long sx;           // x[k*sx]
  void* Y;
  long long sy;           // y[r*sy]
  int R, K;
  int ksplit, kchunk;     // k range of split s: [s*kchunk, min(K, (s+1)*kchunk))
  uint32_t* ws;           // [ksplit][R] partial sums (fp32 / int32 bits) when ksplit > 1
  int epi, act;
  const void* bias;
  int bias_kind, bias_on_r;  // bias[r] (1) or bias[0] (0)
  const void* res;
  int res_kind;
  long long sres;            // residual element of row r at res[r*sres]
};

template <int AB>
struct GvType;
template <> struct GvType<GV_F16> { using T = __half; using Acc = float; };
template <> struct GvType<GV_BF16> { using T = __nv_bfloat16; using Acc = float; };
template <> struct GvType<GV_S8> { using T = int8_t; using Acc = int32_t; };
template <> struct GvType<GV_U8> { using T = uint8_t; using Acc = uint32_t; };

template <int AB>
__device__ __forceinline__ typename GvType<AB>::Acc gv_mul(typename GvType<AB>::T w,
                                                           typename GvType<AB>::T x) {
  if constexpr (AB == GV_S8 || AB == GV_U8)
    return (typename GvType<AB>::Acc)w * (typename GvType<AB>::Acc)x;
  else
    return to_f32(w) * to_f32(x);
}

// Multiply-add of two 16-byte vectors into acc.
template <int AB>
__device__ __forceinline__ void gv_dot16(const uint4& w, const uint4& x,
                                         typename GvType<AB>::Acc& acc) {
  const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
  const uint32_t xv[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (AB == GV_S8) {
      acc = __dp4a((int)wv[i], (int)xv[i], acc);
    } else if constexpr (AB == GV_U8) {
      acc = __dp4a(wv[i], xv[i], acc);
    } else if constexpr (AB == GV_F16) {
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&wv[i]));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&xv[i]));
      acc = fmaf(a.x, b.x, acc);
      acc = fmaf(a.y, b.y, acc);
    } else {
      const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wv[i]));
      const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&xv[i]));
      acc = fmaf(a.x, b.x, acc);
      acc = fmaf(a.y, b.y, acc);
    }
  }
}

template <typename Acc>
__device__ __forceinline__ uint32_t acc_bits(Acc a) {
  if constexpr (std::is_same<Acc, float>::value) return __float_as_uint(a);
  else return (uint32_t)a;
}

// The epilogue of row r (floating-point outputs), conversion and store.
template <int OUT>
__device__ __forceinline__ void gv_store(const GemvParams& p, int r, uint32_t bits) {
  if constexpr (OUT != GV_OUT_I32) {
    if (p.epi) {
      float init = 0.f;
      if (p.bias) init += load_as_f32(p.bias, p.bias_kind, p.bias_on_r ? r : 0);
      if (p.res) init += load_as_f32(p.res, p.res_kind, (long long)r * p.sres);
      bits = __float_as_uint(act_any(p.act, __uint_as_float(bits) + init));
    }
  }
  const long long i = (long long)r * p.sy;
  if constexpr (OUT == GV_OUT_F32 || OUT == GV_OUT_I32) {
    reinterpret_cast<uint32_t*>(p.Y)[i] = bits;
  } else if constexpr (OUT == GV_OUT_F16) {
    reinterpret_cast<__half*>(p.Y)[i] = __float2half_rn(__uint_as_float(bits));
  } else {
    reinterpret_cast<__nv_bfloat16*>(p.Y)[i] = __float2bfloat16_rn(__uint_as_float(bits));
  }
}

template <int OUT>
__device__ __forceinline__ void gv_finish_row(const GemvParams& p, int r, int split,
                                              uint32_t bits) {
  if (p.ksplit > 1)
    p.ws[(long long)split * p.R + r] = bits;
  else
    gv_store<OUT>(p, r, bits);
}

// ---- K-contiguous: one warp per row ----------------------------------------------------
// VEC: rows and x start on 16-byte boundaries and x is contiguous, so both stream as
// 16-byte vectors; otherwise element by element.
template <int AB, int OUT, bool VEC>
__global__ void __launch_bounds__(kGvThreads)
    gemv_kc_kernel(const GemvParams p) {
  using T = typename GvType<AB>::T;
  using Acc = typename GvType<AB>::Acc;
  constexpr int E = 16 / (int)sizeof(T);   // elements per 16 bytes
  const int lane = threadIdx.x & 31;
  const int warps = kGvThreads / 32;
  const int split = blockIdx.y;
  const int k0 = split * p.kchunk;
  const int k1 = min(p.K, k0 + p.kchunk);
  const T* W = reinterpret_cast<const T*>(p.W);
  const T* X = reinterpret_cast<const T*>(p.X);
  for (int r = blockIdx.x * warps + (threadIdx.x >> 5); r < p.R; r += gridDim.x * warps) {
    const T* row = W + (long long)r * p.sr;
    Acc acc[4] = {0, 0, 0, 0};
    int k = k0;
    if constexpr (VEC) {
      // k0 is a multiple of 32·E (the split size is), so every vector is aligned.
      const int kv_end = k0 + (k1 - k0) / E * E;
      int kk = k0 + lane * E;
      for (; kk + 3 * 32 * E < kv_end; kk += 4 * 32 * E) {
        uint4 w[4], x[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          w[u] = ldg_stream_v4(row + kk + u * 32 * E);
          x[u] = __ldg(reinterpret_cast<const uint4*>(X + kk + u * 32 * E));
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) gv_dot16<AB>(w[u], x[u], acc[u]);
      }
      for (; kk < kv_end; kk += 32 * E) {
        const uint4 w = ldg_stream_v4(row + kk);
        const uint4 x = __ldg(reinterpret_cast<const uint4*>(X + kk));
        gv_dot16<AB>(w, x, acc[0]);
      }
      k = kv_end;
    }
    for (int kk = k + lane; kk < k1; kk += 32)
      acc[1] += gv_mul<AB>(row[kk], X[(long long)kk * p.sx]);
    Acc a = (acc[0] + acc[1]) + (acc[2] + acc[3]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
    if (lane == 0) gv_finish_row<OUT>(p, r, split, acc_bits<Acc>(a));
  }
}

// ---- R-contiguous: 8 threads × 16 bytes of rows, 32 threads along k ----------------------
template <int AB, int OUT, bool VEC>
__global__ void __launch_bounds__(kGvThreads)
    gemv_rc_kernel(const GemvParams p) {
  using T = typename GvType<AB>::T;
  using Acc = typename GvType<AB>::Acc;
  constexpr int E = 16 / (int)sizeof(T);
  constexpr int TR = 8, TK = kGvThreads / TR;
  constexpr int RB = TR * E;               // rows per CTA
  __shared__ Acc red[TK][RB + 1];
  const int tr = threadIdx.x % TR;
  const int tk = threadIdx.x / TR;
  const int split = blockIdx.y;
  const int k0 = split * p.kchunk;
  const int k1 = min(p.K, k0 + p.kchunk);
  const T* W = reinterpret_cast<const T*>(p.W);
  const T* X = reinterpret_cast<const T*>(p.X);
  for (int rb = blockIdx.x; rb * RB < p.R; rb += gridDim.x) {
    const int r0 = rb * RB + tr * E;
    Acc acc[E];
#pragma unroll
    for (int e = 0; e < E; ++e) acc[e] = 0;
    if (VEC && r0 + E <= p.R) {
      int k = k0 + tk;
      for (; k + 3 * TK < k1; k += 4 * TK) {
        uint4 w[4];
        T x[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          w[u] = ldg_stream_v4(W + (long long)(k + u * TK) * p.sk + r0);
          x[u] = X[(long long)(k + u * TK) * p.sx];
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const T* wv = reinterpret_cast<const T*>(&w[u]);
#pragma unroll
          for (int e = 0; e < E; ++e) acc[e] += gv_mul<AB>(wv[e], x[u]);
        }
      }
      for (; k < k1; k += TK) {
        const uint4 w = ldg_stream_v4(W + (long long)k * p.sk + r0);
        const T x = X[(long long)k * p.sx];
        const T* wv = reinterpret_cast<const T*>(&w);
#pragma unroll
        for (int e = 0; e < E; ++e) acc[e] += gv_mul<AB>(wv[e], x);
      }
    } else {
      for (int k = k0 + tk; k < k1; k += TK) {
        const T x = X[(long long)k * p.sx];
#pragma unroll
        for (int e = 0; e < E; ++e)
          if (r0 + e < p.R) acc[e] += gv_mul<AB>(W[(long long)k * p.sk + (long long)(r0 + e) * p.sr], x);
      }
    }
#pragma unroll
    for (int e = 0; e < E; ++e) red[tk][tr * E + e] = acc[e];
    __syncthreads();
    for (int i = threadIdx.x; i < RB; i += kGvThreads) {
      Acc a = 0;
#pragma unroll 8
      for (int j = 0; j < TK; ++j) a += red[j][i];
      const int r = rb * RB + i;
      if (r < p.R) gv_finish_row<OUT>(p, r, split, acc_bits<Acc>(a));
    }
    __syncthreads();
  }
}

// ---- the k splits added in a fixed order, then the epilogue -----------------------------
template <int OUT, bool INT>
__global__ void gemv_splits_kernel(const GemvParams p) {
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < p.R; r += gridDim.x * blockDim.x) {
    uint32_t bits;
    if constexpr (INT) {
      uint32_t a = 0;
      for (int s = 0; s < p.ksplit; ++s) a += p.ws[(long long)s * p.R + r];
      bits = a;
    } else {
      float a = 0.f;
      for (int s = 0; s < p.ksplit; ++s) a += __uint_as_float(p.ws[(long long)s * p.R + r]);
      bits = __float_as_uint(a);
    }
    gv_store<OUT>(p, r, bits);
  }
}

int gv_ab(int dt) {
  switch (dt) {
    case LVB_F16: return GV_F16;
    case LVB_BF16: return GV_BF16;
    case LVB_I8: return GV_S8;
    case LVB_U8: return GV_U8;
  }
  return -1;
}
int gv_out(int dt) {
  switch (dt) {
    case LVB_F32: return GV_OUT_F32;
    case LVB_F16: return GV_OUT_F16;
    case LVB_BF16: return GV_OUT_BF16;
    case LVB_I32:
    case LVB_U32: return GV_OUT_I32;
  }
  return -1;
}

template <int AB, int OUT>
int gv_launch_t(const GemvParams& p, bool kc, bool vec, dim3 grid, cudaStream_t s) {
  if (kc) {
    if (vec) gemv_kc_kernel<AB, OUT, true><<<grid, kGvThreads, 0, s>>>(p);
    else gemv_kc_kernel<AB, OUT, false><<<grid, kGvThreads, 0, s>>>(p);
  } else {
    if (vec) gemv_rc_kernel<AB, OUT, true><<<grid, kGvThreads, 0, s>>>(p);
    else gemv_rc_kernel<AB, OUT, false><<<grid, kGvThreads, 0, s>>>(p);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail_cuda(e, "lvb_gemm", "gemv launch");
  if (p.ksplit > 1) {
    const int blocks = (p.R + 255) / 256;
    constexpr bool kInt = AB == GV_S8 || AB == GV_U8;
    gemv_splits_kernel<OUT, kInt><<<std::min(blocks, 4096), 256, 0, s>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail_cuda(e, "lvb_gemm", "gemv split launch");
  }
  return LVB_OK;
}

// The pairs lvb_gemm_check admits: 16-bit operands -> F32 / F16 / BF16, 8-bit -> 32-bit int.
template <int AB>
int gv_launch_ab(int out, const GemvParams& p, bool kc, bool vec, dim3 grid, cudaStream_t s) {
  if constexpr (AB == GV_S8 || AB == GV_U8) {
    if (out == GV_OUT_I32) return gv_launch_t<AB, GV_OUT_I32>(p, kc, vec, grid, s);
  } else {
    switch (out) {
      case GV_OUT_F32: return gv_launch_t<AB, GV_OUT_F32>(p, kc, vec, grid, s);
      case GV_OUT_F16: return gv_launch_t<AB, GV_OUT_F16>(p, kc, vec, grid, s);
      case GV_OUT_BF16: return gv_launch_t<AB, GV_OUT_BF16>(p, kc, vec, grid, s);
    }
  }
  return fail(LVB_ERR_UNSUPPORTED, "lvb_gemm", "gemv output type");
}

}  // namespace

bool gemv_applies(const lvb_gemm_desc* d) { return d->K > 0 && (d->N == 1 || d->M == 1); }

int gemv_plan(const lvb_gemm_desc* d, int sm_count, GemvPlan* out) {
  const int es = dtype_size(d->a_type);
  const bool n1 = d->N == 1;
  const int64_t R = n1 ? d->M : d->N;
  // K-contiguous when the matrix (A for N == 1, Bᵀ for M == 1) runs along k.
  const bool kc = n1 ? (d->a_rowmajor != 0 || d->K == 1) : (d->b_rowmajor == 0 || d->K == 1);
  const int E = 16 / es;
  int64_t ctas_r, min_k;
  if (kc) {
    ctas_r = (R + kGvThreads / 32 - 1) / (kGvThreads / 32);
    min_k = 4LL * 32 * E;             // one unrolled sweep of a warp
  } else {
    ctas_r = (R + 8LL * E - 1) / (8LL * E);
    min_k = 4LL * (kGvThreads / 8);   // four k rows per thread
  }
  const int64_t want = 4LL * std::max(1, sm_count);
  int64_t ksplit = 1;
  if (ctas_r < want) ksplit = std::min<int64_t>((want + ctas_r - 1) / ctas_r, (d->K + min_k - 1) / min_k);
  ksplit = std::max<int64_t>(1, std::min<int64_t>(ksplit, 1024));
  const int64_t unit = kc ? 32LL * E : 1;   // split boundaries keep 16-byte vectors aligned
  int64_t kchunk = (d->K + ksplit - 1) / ksplit;
  kchunk = (kchunk + unit - 1) / unit * unit;
  ksplit = (d->K + kchunk - 1) / kchunk;
  out->k_contiguous = kc ? 1 : 0;
  out->ksplit = (int32_t)ksplit;
  out->kchunk = (int64_t)kchunk;
  out->ctas = (int32_t)std::min<int64_t>(ctas_r, 64LL * std::max(1, sm_count));
  out->workspace_bytes = ksplit > 1 ? (int64_t)ksplit * R * 4 : 0;
  return LVB_OK;
}

int gemv_launch(const lvb_gemm_desc* d, const lvb_epilogue* e, const void* A, const void* B,
                void* C, cudaStream_t stream, DeviceState* dev, bool allow_workspace) {
  const int es = dtype_size(d->a_type);
  GemvPlan plan;
  gemv_plan(d, dev->sm_count, &plan);
  if (!allow_workspace) {
    plan.ksplit = 1;
    plan.kchunk = d->K;
    plan.workspace_bytes = 0;
  }
  const bool n1 = d->N == 1;
  GemvParams p = {};
  if (n1) {
    p.W = A;
    p.R = (int)d->M;
    p.sr = d->a_rowmajor ? d->lda : 1;
    p.sk = d->a_rowmajor ? 1 : d->lda;
    p.X = B;
    p.sx = d->b_rowmajor ? d->ldb : 1;
    p.sy = d->c_rowmajor ? d->ldc : 1;
  } else {
    p.W = B;
    p.R = (int)d->N;
    p.sr = d->b_rowmajor ? 1 : d->ldb;
    p.sk = d->b_rowmajor ? d->ldb : 1;
    p.X = A;
    p.sx = d->a_rowmajor ? 1 : d->lda;
    p.sy = d->c_rowmajor ? 1 : d->ldc;
  }
  if (d->K == 1) {   // one element per row: either kernel; take the K-contiguous one
    p.sk = 1;
  }
  p.Y = C;
  p.K = (int)d->K;
  p.ksplit = plan.ksplit;
  p.kchunk = (int)plan.kchunk;
  p.act = LVB_ACT_NONE;
  if (e) {
    p.act = e->activation;
    p.bias = e->bias;
    p.bias_kind = e->bias_type;
    p.bias_on_r = n1 ? (e->bias_axis == LVB_BIAS_PER_ROW) : (e->bias_axis == LVB_BIAS_PER_COL);
    p.res = e->residual;
    p.res_kind = e->residual_type;
    p.sres = n1 ? (d->c_rowmajor ? e->ldr : 1) : (d->c_rowmajor ? 1 : e->ldr);
    p.epi = (p.act != LVB_ACT_NONE || p.bias || p.res) ? 1 : 0;
  }
  const bool kc = plan.k_contiguous != 0;
  const bool vec = kc ? ((uintptr_t)p.W % 16 == 0 && (p.sr * es) % 16 == 0 && p.sx == 1 &&
                         (uintptr_t)p.X % 16 == 0)
                      : ((uintptr_t)p.W % 16 == 0 && (p.sk * es) % 16 == 0);
  dim3 grid((unsigned)plan.ctas, (unsigned)plan.ksplit);
  const int ab = gv_ab(d->a_type), out = gv_out(d->c_type);
  void* ws = nullptr;
  if (plan.ksplit > 1) {
    cudaError_t ce = workspace_alloc(dev, &ws, (size_t)plan.workspace_bytes, stream);
    if (ce != cudaSuccess) return fail_cuda(ce, "lvb_gemm", "gemv workspace cudaMallocAsync");
    p.ws = reinterpret_cast<uint32_t*>(ws);
  }
  int st;
  switch (ab) {
    case GV_F16: st = gv_launch_ab<GV_F16>(out, p, kc, vec, grid, stream); break;
    case GV_BF16: st = gv_launch_ab<GV_BF16>(out, p, kc, vec, grid, stream); break;
    case GV_S8: st = gv_launch_ab<GV_S8>(out, p, kc, vec, grid, stream); break;
    case GV_U8: st = gv_launch_ab<GV_U8>(out, p, kc, vec, grid, stream); break;
    default: st = fail(LVB_ERR_UNSUPPORTED, "lvb_gemm", "gemv operand type");
  }
  if (ws) {
    cudaError_t ce = cudaFreeAsync(ws, stream);
    if (st == LVB_OK && ce != cudaSuccess) return fail_cuda(ce, "lvb_gemm", "gemv workspace cudaFreeAsync");
  }
  return st;
}

}  // namespace lvb
