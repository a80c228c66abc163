// gemm_sm100.cu — persistent warp-specialised tcgen05 GEMM for B200 (sm_100a).
//
// What it computes is Lava's coopmat GEMM (the k-loop of test/glsl/coopmat2_gemm_regs.comp:
// 53-83, and the vocabulary path AcceleratedMatrix load -> muladd -> convert -> copyto!,
// src/vocabulary/coopmat.jl:124-203): D[m,n] = sum_k A[m,k]·B[n,k] accumulated in fp32
// (kind::f16) or int32 (kind::i8), converted with round-to-nearest-even to the output type
// and stored with ragged edges clamped.
//
// Optionally with the fused epilogue D = act(A·B + (bias + R)): the accumulator started from
// bias + residual as coopmat_add builds it, then a per-element activation
// (src/device/coopmat_intrinsics.jl:322-331,435-447,551-593).
//
// How (kernel space; the host swaps A and B when the caller wants a row-major C):
//   * operands are K-contiguous ("K-major"), or, for 16-bit types, MN-contiguous and read
//     MN-major in place (Lava's transposing tensor view); a CTA owns a 128 × BN output tile;
//   * warp 0 lane 0: TMA producer. Streams 128×128-byte A and BN×128-byte B boxes
//     (128B swizzle, zero fill past the edges) into a STAGES-deep mbarrier ring;
//   * warp 1: MMA issuer (the converged warp waits, an elected lane issues). Four
//     tcgen05.mma (128×BN×16 f16 / ×32 i8) per stage into one of two TMEM accumulators,
//     tcgen05.commit frees the stage;
//   * warp 2: allocates / frees TMEM (2·BN columns);
//   * warps 4-7: epilogue. tcgen05.ld 32 columns at a time; lane = output row, so each
//     store of one column by a warp writes 32 consecutive m (coalesced, D is m-contiguous),
//     or, with D n-contiguous, 32 × 128-byte boxes staged in shared memory go out as TMA
//     tensor stores; the accumulator is handed back as soon as it has been read, so the
//     next tile's MMAs overlap this tile's stores.
//   * persistent grid (one CTA per SM), tiles visited in groups of GROUP_M row-tiles so the
//     ~148 tiles in flight share A rows and B columns in L2.
#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "epilogue.cuh"
#include "lvb_internal.h"

namespace lvb {

enum AbKind { AB_F16 = 0, AB_BF16 = 1, AB_S8 = 2, AB_U8 = 3 };
enum OutKind { OUT_F32 = 0, OUT_F16 = 1, OUT_BF16 = 2, OUT_I32 = 3 };

constexpr int kBM = 128;
constexpr int kMaxDevices = 128;
constexpr int kRowBytes = 128;                 // K bytes per stage row (64 f16 / 128 i8)
constexpr int kAStageBytes = kBM * kRowBytes;  // 16 KB
constexpr int kThreads = 256;

struct GemmParams {
  int M, N, K;            // kernel space
  int tiles_m, tiles_n, num_kb;
  int total_tiles;
  int group_m;            // row-tiles per raster group
  int l2_mode;            // 0: A and B evict_last, 1: A evict_last / B evict_first, 2: no hint
  int a_mn, b_mn;         // operand staged MN-major (16-bit types only): the transposed view
  int d_nmajor;           // D[m*ldd + n] (n contiguous) instead of D[m + n*ldd]
  int stage_out;          // 1 (with d_nmajor): interior 32×32 boxes written by TMA tensor stores
  void* D;
  long long ldd;
  // Fused epilogue (kernel space): D = act(acc + (bias + R)).
  int epi;                // any of the below present
  int act;                // lvb_activation
  const void* bias;       // nullable
  int bias_kind;          // lvb_dtype of bias (F32 / F16 / BF16)
  int bias_on_m;          // 1: bias[m] (one value per TMEM lane), 0: bias[n]
  const void* res;        // nullable; R[m + n*ldr], may be D itself
  int res_kind;
  long long ldr;
  // coopmat_mul operand S and the per-element program's matrix operand E, both M×N in D's
  // layout (kernel space, like R); the program runs when prog.n > 0.
  const void* mul;
  int mul_kind;
  long long ldm;
  const void* ext;
  int ext_kind;
  long long lde;
  int prog_swap;          // 1: the caller's row is kernel n (the product runs as Cᵀ = BᵀAᵀ)
  PeProgram prog;
  // Clamped k tail over the padded extent: acc += kx · u[m] · v[n], with u the value kernel A
  // reads past its last column (row m) and v the one kernel B reads (row n).
  int kx;                 // k_pad - K (0: none)
  int cu_mode, cv_mode;   // 1: the clamp constant, 2: the row's element K-1 (to edge)
  float cu_f, cv_f;       // constants for 16-bit operands
  int cu_i, cv_i;         // constants for 8-bit operands
  const void* cu_ptr;     // kernel A / B and their layout, for the edge elements
  long long cu_ld;
  int cu_mn;
  const void* cv_ptr;
  long long cv_ld;
  int cv_mn;
  DevStatus* status;
  unsigned long long timeout_ns;
};

// Stage geometry of an MN-major 16-bit operand: 64-element (128-byte) MN chunks of 64 K
// rows, each one TMA box; consecutive chunks 8 KB apart (the descriptor's leading byte
// offset), 8-row K groups 1 KB apart (its stride byte offset).
constexpr int kMnChunkBytes = 64 * 128;

// Output staging for TMA stores: per epilogue warp two 32×32 sub-tiles of up to 4-byte
// elements.
constexpr int kStoreBufBytes = 32 * 32 * 4;
constexpr int kStoreBytes = 4 * 2 * kStoreBufBytes;

// out[j] += X[i0 + j*stride] for j < nv. The 32 loads form one basic block ahead of the
// conversions, so their latencies overlap.
template <typename T>
__device__ __forceinline__ void add_loaded32(const void* base, long long i0, long long stride,
                                             int nv, float (&out)[32]) {
  const T* x = reinterpret_cast<const T*>(base) + i0;
  if (stride == 1 && nv == 32 && (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    // A contiguous run (a bias slice, or a residual row when D is n-contiguous): 16-byte
    // loads marked for streaming (evict-first), so the residual does not push the A and B
    // panels the next tiles re-read out of L2.
    constexpr int E = 16 / (int)sizeof(T);
    uint4 w[32 / E];
#pragma unroll
    for (int i = 0; i < 32 / E; ++i) w[i] = __ldcs(reinterpret_cast<const uint4*>(x) + i);
#pragma unroll
    for (int i = 0; i < 32 / E; ++i) {
      const T* e = reinterpret_cast<const T*>(&w[i]);
#pragma unroll
      for (int k = 0; k < E; ++k) out[i * E + k] += to_f32(e[k]);
    }
    return;
  }
  T v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = j < nv ? x[j * stride] : T(0.f);
#pragma unroll
  for (int j = 0; j < 32; ++j) out[j] += to_f32(v[j]);
}

__device__ __forceinline__ void add_loaded32(int kind, const void* base, long long i0,
                                             long long stride, int nv, float (&out)[32]) {
  if (kind == LVB_F32) add_loaded32<float>(base, i0, stride, nv, out);
  else if (kind == LVB_F16) add_loaded32<__half>(base, i0, stride, nv, out);
  else add_loaded32<__nv_bfloat16>(base, i0, stride, nv, out);
}

// acc + (bias + R), then the activation, for one element: the accumulator started from
// bias + residual as coopmat_add builds it (src/device/coopmat_intrinsics.jl:435-447), then
// perelement.
__device__ __forceinline__ float epi_value(const GemmParams& p, float acc, int m, int n,
                                           float bias_m) {
  float init = bias_m;
  if (p.bias && !p.bias_on_m) init += load_as_f32(p.bias, p.bias_kind, n);
  if (p.res) init += load_as_f32(p.res, p.res_kind, (long long)n * p.ldr + m);
  if (p.kx) init += (float)p.kx * p.cu_f * p.cv_f;   // K == 0: constant clamps only
  float x = acc + init;
  if (p.mul) x *= load_as_f32(p.mul, p.mul_kind, (long long)n * p.ldm + m);
  x = act_any(p.act, x);
  if (p.prog.n) {
    float xs[1] = {x};
    const int rows[1] = {p.prog_swap ? n : m}, cols[1] = {p.prog_swap ? m : n};
    const float es[1] = {p.ext ? load_as_f32(p.ext, p.ext_kind, (long long)n * p.lde + m) : 0.f};
    pe_run<1>(p.prog, xs, rows, cols, es);
    x = xs[0];
  }
  return x;
}

// The clamp term's per-row value u (kernel A's read past column K-1 of row m) and per-column
// values v (kernel B's, rows n0..n0+nv-1), as fp32 for 16-bit operands.
template <int AB>
__device__ __forceinline__ float clamp_u_f(const GemmParams& p, int m) {
  if (p.cu_mode == 1) return p.cu_f;
  const long long i = p.cu_mn ? (long long)(p.K - 1) * p.cu_ld + m : (long long)m * p.cu_ld + p.K - 1;
  return operand_f32(p.cu_ptr, AB, i);
}
template <int AB>
__device__ __forceinline__ float clamp_v_f(const GemmParams& p, int n) {
  if (p.cv_mode == 1) return p.cv_f;
  const long long i = p.cv_mn ? (long long)(p.K - 1) * p.cv_ld + n : (long long)n * p.cv_ld + p.K - 1;
  return operand_f32(p.cv_ptr, AB, i);
}
template <int AB>
__device__ __forceinline__ int clamp_u_i(const GemmParams& p, int m) {
  if (p.cu_mode == 1) return p.cu_i;
  const long long i = p.cu_mn ? (long long)(p.K - 1) * p.cu_ld + m : (long long)m * p.cu_ld + p.K - 1;
  return operand_i32(p.cu_ptr, AB, i);
}
template <int AB>
__device__ __forceinline__ int clamp_v_i(const GemmParams& p, int n) {
  if (p.cv_mode == 1) return p.cv_i;
  const long long i = p.cv_mn ? (long long)(p.K - 1) * p.cv_ld + n : (long long)n * p.cv_ld + p.K - 1;
  return operand_i32(p.cv_ptr, AB, i);
}

// 8 elements of an M×N operand in D's layout at row m, columns n0..n0+7 (nv of them inside).
__device__ __forceinline__ void load8(const GemmParams& p, int kind, const void* base,
                                      long long ld, int m, int n0, int nv, float (&out)[8]) {
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const long long i = p.d_nmajor ? (long long)m * ld + n0 + e : (long long)(n0 + e) * ld + m;
    out[e] = e < nv ? load_as_f32(base, kind, i) : 0.f;
  }
}

__device__ __forceinline__ uint64_t policy_for(int mode, bool is_a) {
  if (mode == 2) return 0;
  if (mode == 1 && !is_a) return policy_evict_first();
  return policy_evict_last();
}

// TMA load with the raster's cache policy (mode 2: plain load).
__device__ __forceinline__ void tma_load_2d_pol(void* dst, const CUtensorMap* tm, int32_t c0,
                                                int32_t c1, uint64_t* bar, int mode, uint64_t pol) {
  if (mode == 2)
    tma_load_2d(dst, tm, c0, c1, bar);
  else
    tma_load_2d_hint(dst, tm, c0, c1, bar, pol);
}

template <int BN>
struct GemmCfg {
  static constexpr int kBStageBytes = BN * kRowBytes;
  static constexpr int kStageBytes = kAStageBytes + kBStageBytes;
  static constexpr int kStages = BN == 256 ? 4 : (BN == 128 ? 6 : 8);
  static constexpr int kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;
  static constexpr int kBarBytes = 256;
  static constexpr int kSmemBytes = kStages * kStageBytes + kStoreBytes + kBarBytes + 1024;
};

__device__ __forceinline__ void tile_coords(int t, const GemmParams& p, int& tm, int& tn) {
  const int per_group = p.group_m * p.tiles_n;
  const int g = t / per_group;
  const int first_m = g * p.group_m;
  const int gsize = min(p.tiles_m - first_m, p.group_m);
  const int r = t - g * per_group;
  tm = first_m + r % gsize;
  tn = r / gsize;
}

// Wait that ignores the abort flag: used only while draining on the way out.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity, uint64_t timeout_ns) {
  const uint32_t a = smem_u32(bar);
  const uint64_t t0 = global_ns();
  while (!bar_try_wait(a, parity)) {
    if (global_ns() - t0 > timeout_ns) return;
  }
}

template <int OUT>
__device__ __forceinline__ void store_out(void* D, long long idx, uint32_t bits) {
  if constexpr (OUT == OUT_F32 || OUT == OUT_I32) {
    reinterpret_cast<uint32_t*>(D)[idx] = bits;
  } else if constexpr (OUT == OUT_F16) {
    reinterpret_cast<__half*>(D)[idx] = __float2half_rn(__uint_as_float(bits));
  } else {
    reinterpret_cast<__nv_bfloat16*>(D)[idx] = __float2bfloat16_rn(__uint_as_float(bits));
  }
}

// Output conversion: fp32 / int32 bits -> the bits stored (RNE for 16-bit outputs).
template <int OUT>
__device__ __forceinline__ uint32_t cvt_out(uint32_t bits) {
  if constexpr (OUT == OUT_F32 || OUT == OUT_I32) {
    return bits;
  } else if constexpr (OUT == OUT_F16) {
    return __half_as_ushort(__float2half_rn(__uint_as_float(bits)));
  } else {
    return __bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(bits)));
  }
}

// r[j] = act(acc[j] + init[j]) for the 32 columns: straight-line code over independent
// elements.
template <int ACT>
__device__ __forceinline__ void act32(uint32_t (&r)[32], const float (&init)[32]) {
#pragma unroll
  for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(act_fn<ACT>(__uint_as_float(r[j]) + init[j]));
}

// x[j] <- f(act(x[j] · S[m, n0+j])) for the 32 columns n0.. of row m (x already holds
// acc + bias + R): coopmat_mul, the activation and the caller's program, eight columns at a
// time.
__device__ __noinline__ void epi_generic(const GemmParams& p, float* x, int m, int n0, int nv) {
#pragma unroll 1
  for (int g = 0; g < 4; ++g) {
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = x[8 * g + e];
    const int nvg = nv - 8 * g;
    if (p.mul) {
      float s8[8];
      load8(p, p.mul_kind, p.mul, p.ldm, m, n0 + 8 * g, nvg, s8);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] *= s8[e];
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = act_any(p.act, v[e]);
    if (p.prog.n) {
      float e8[8];
      if (p.ext) {
        load8(p, p.ext_kind, p.ext, p.lde, m, n0 + 8 * g, nvg, e8);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) e8[e] = 0.f;
      }
      int rows[8], cols[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int n = n0 + 8 * g + e;
        rows[e] = p.prog_swap ? n : m;
        cols[e] = p.prog_swap ? m : n;
      }
      pe_run<8>(p.prog, v, rows, cols, e8);
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) x[8 * g + e] = v[e];
  }
}

// The fused epilogue on one tcgen05.ld worth (32 columns n0.. of row m), in place. `nv`
// columns are inside the matrix (0 for a row past M: nothing is loaded for it).
template <int OUT, int AB>
__device__ __forceinline__ void apply_epilogue(const GemmParams& p, uint32_t (&r)[32], int m,
                                               int n0, int nv, float bias_m) {
  if constexpr (OUT == OUT_I32) {
    // Integer outputs take only the clamp term, in wrapping int32 like the accumulation.
    if (p.kx && nv) {
      const int u = clamp_u_i<AB>(p, m);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int v = j < nv ? clamp_v_i<AB>(p, n0 + j) : 0;
        r[j] = (uint32_t)((int)r[j] + (int)((unsigned)p.kx * (unsigned)u * (unsigned)v));
      }
    }
  } else {
    float init[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) init[j] = bias_m;
    if (p.bias && !p.bias_on_m) add_loaded32(p.bias_kind, p.bias, n0, 1, nv, init);
    if (p.res) {
      if (p.d_nmajor)
        add_loaded32(p.res_kind, p.res, (long long)m * p.ldr + n0, 1, nv, init);
      else
        add_loaded32(p.res_kind, p.res, (long long)n0 * p.ldr + m, p.ldr, nv, init);
    }
    if (p.kx && nv) {
      const float u = (float)p.kx * clamp_u_f<AB>(p, m);
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < nv) init[j] = fmaf(u, clamp_v_f<AB>(p, n0 + j), init[j]);
    }
    if (!p.mul && !p.prog.n) {
      switch (p.act) {
        case LVB_ACT_RELU: act32<LVB_ACT_RELU>(r, init); break;
        case LVB_ACT_GELU_TANH: act32<LVB_ACT_GELU_TANH>(r, init); break;
        case LVB_ACT_GELU_ERF: act32<LVB_ACT_GELU_ERF>(r, init); break;
        case LVB_ACT_SILU: act32<LVB_ACT_SILU>(r, init); break;
        default: act32<LVB_ACT_NONE>(r, init); break;
      }
      return;
    }
    // coopmat_mul and / or the caller's per-element program, out of line: the values go
    // through a local array so the common path above keeps its registers.
    float x[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) x[j] = __uint_as_float(r[j]) + init[j];
    epi_generic(p, x, m, n0, nv);
#pragma unroll
    for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(x[j]);
  }
}

// Direct store of 32 columns n0.. of row m, clamped to N. With D m-contiguous, lanes hold
// consecutive m and every column is one warp store of 32 consecutive elements; with D
// n-contiguous (edge boxes only) each thread writes its own run of up to 32 elements.
template <int OUT>
__device__ __forceinline__ void store_direct(const GemmParams& p, const uint32_t (&r)[32], int m,
                                             int n0) {
  if (p.d_nmajor) {
    const long long base = (long long)m * p.ldd + n0;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (n0 + j < p.N) store_out<OUT>(p.D, base + j, r[j]);
    return;
  }
  if (n0 + 32 <= p.N) {
#pragma unroll
    for (int j = 0; j < 32; ++j) store_out<OUT>(p.D, (long long)(n0 + j) * p.ldd + m, r[j]);
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (n0 + j < p.N) store_out<OUT>(p.D, (long long)(n0 + j) * p.ldd + m, r[j]);
  }
}

template <int OUT>
__device__ __forceinline__ uint32_t pack_out2(uint32_t a, uint32_t b) {
  if constexpr (OUT == OUT_F16) {
    __half2 v = __floats2half2_rn(__uint_as_float(a), __uint_as_float(b));
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __nv_bfloat162 v = __floats2bfloat162_rn(__uint_as_float(a), __uint_as_float(b));
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

// Staged store (D n-contiguous) of 32-bit outputs: the warp's 32 (m) × 32 (n) sub-tile goes
// to shared memory as [m][n] — each lane's 32 values are one contiguous 128-byte row, written
// as 16-byte vectors with the tensor map's 128B swizzle (16-byte chunk c of row r at
// c ^ (r & 7)), so the 32 lanes' vector stores hit distinct banks — and one TMA tensor store of
// the box {32 n, 32 m} at (n0, m0w) writes it out. Only boxes wholly inside the matrix take
// this path (the store's clipping at the innermost edge is not exact to the element: a
// 333-row matrix inside a 400-row buffer had rows 333.. overwritten), edge boxes use the
// predicated direct stores. Two buffers per warp: a buffer is rewritten only after the store
// issued from it two chunks earlier has finished reading it.
template <int OUT>
__device__ __forceinline__ void store_staged(const CUtensorMap* tmD, const uint32_t (&r)[32],
                                             uint32_t sbase, uint32_t& cnt, int m0w, int n0) {
  static_assert(OUT == OUT_F32 || OUT == OUT_I32, "16-bit outputs are staged in pairs");
  const uint32_t lane = lane_id();
  const uint32_t buf = sbase + (cnt & 1) * kStoreBufBytes;
  if (lane == 0) bulk_wait_group_read<1>();
  __syncwarp();
  const uint32_t row = buf + lane * 128;
#pragma unroll
  for (int c = 0; c < 8; ++c)
    st_shared_v4(row + ((c ^ (lane & 7)) << 4), r[4 * c], r[4 * c + 1], r[4 * c + 2],
                 r[4 * c + 3]);
  fence_proxy_async_smem();  // this thread's writes -> visible to the TMA (async proxy)
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(tmD, buf, n0, m0w);
    bulk_commit_group();
  }
  ++cnt;
}

// Staged store of a pair of chunks for 16-bit outputs: the warp's 32 (m) × 64 (n) sub-tile
// is one 4 KB box {64 n, 32 m} of 128-byte rows (128B swizzle: 16-byte chunk j of row r at
// j ^ (r & 7)), one fence and one TMA tensor store for two chunks. The first chunk fills the
// left half of each row, the second the right half. Two 4 KB buffers per warp.
template <int OUT>
__device__ __forceinline__ void stage_half16(const uint32_t (&r)[32], uint32_t sbase,
                                             uint32_t cnt, int half) {
  const uint32_t lane = lane_id();
  const uint32_t buf = sbase + (cnt & 1) * kStoreBufBytes;
  if (half == 0) {
    if (lane == 0) bulk_wait_group_read<1>();
    __syncwarp();
  }
  const uint32_t row = buf + lane * 128;
#pragma unroll
  for (int c = 0; c < 4; ++c)
    st_shared_v4(row + (((4 * half + c) ^ (lane & 7)) << 4), pack_out2<OUT>(r[8 * c], r[8 * c + 1]),
                 pack_out2<OUT>(r[8 * c + 2], r[8 * c + 3]),
                 pack_out2<OUT>(r[8 * c + 4], r[8 * c + 5]),
                 pack_out2<OUT>(r[8 * c + 6], r[8 * c + 7]));
}

__device__ __forceinline__ void commit_pair16(const CUtensorMap* tmD, uint32_t sbase,
                                              uint32_t& cnt, int m0w, int n0) {
  const uint32_t buf = sbase + (cnt & 1) * kStoreBufBytes;
  fence_proxy_async_smem();  // this thread's writes -> visible to the TMA (async proxy)
  __syncwarp();
  if (lane_id() == 0) {
    tma_store_2d(tmD, buf, n0, m0w);
    bulk_commit_group();
  }
  ++cnt;
}

// Drains this warp's 32 TMEM lanes of one accumulator (NCH chunks of 32 columns): the
// tcgen05.ld of chunk c+1 is in flight while chunk c goes through the epilogue and its
// stores, so the TMEM round trip is hidden. `release` hands the accumulator back as soon as
// every chunk is in registers.
template <int OUT, int AB, int NCH, typename Release>
__device__ __forceinline__ void drain_acc(const GemmParams& p, const CUtensorMap* tmD,
                                          uint32_t t_row, int m, int m0w, int n_base,
                                          float bias_m, uint32_t s_out, uint32_t& n_staged,
                                          Release release) {
  constexpr bool k16 = OUT == OUT_F16 || OUT == OUT_BF16;
  static_assert(NCH % 2 == 0 || !k16, "16-bit outputs are stored in pairs of chunks");
  const bool m_ok = m < p.M;
  uint32_t ra[32], rb[32];
  auto handle = [&](uint32_t (&r)[32], int c) {
    const int n0 = n_base + c * 32;
    if (p.epi) apply_epilogue<OUT, AB>(p, r, m, n0, m_ok ? min(32, p.N - n0) : 0, bias_m);
    if constexpr (k16) {
      // 16-bit outputs go out as 32 x 64 boxes: chunk c (even) and c + 1 share one store
      const int np = n_base + (c & ~1) * 32;
      if (p.stage_out && m0w + 32 <= p.M && np + 64 <= p.N) {
        stage_half16<OUT>(r, s_out, n_staged, c & 1);
        if (c & 1) commit_pair16(tmD, s_out, n_staged, m0w, np);
      } else if (m_ok) {
        store_direct<OUT>(p, r, m, n0);
      }
    } else {
      if (p.stage_out && m0w + 32 <= p.M && n0 + 32 <= p.N)
        store_staged<OUT>(tmD, r, s_out, n_staged, m0w, n0);
      else if (m_ok)
        store_direct<OUT>(p, r, m, n0);
    }
    __syncwarp();  // tcgen05.ld / wait are .sync.aligned: reconverge after the stores
  };
  tmem_ld32(t_row, ra);
  tmem_wait_ld(ra);
#pragma unroll 1
  for (int c = 0; c < NCH; c += 2) {
    if constexpr (NCH % 2 == 1) {
      if (c + 1 == NCH) {   // the odd last chunk: already in registers
        release();
        handle(ra, c);
        break;
      }
    }
    tmem_ld32(t_row + (c + 1) * 32, rb);
    handle(ra, c);
    tmem_wait_ld(rb);
    if (c + 2 < NCH)
      tmem_ld32(t_row + (c + 2) * 32, ra);
    else
      release();
    handle(rb, c + 1);
    if (c + 2 < NCH) tmem_wait_ld(ra);
  }
}

// Shared-memory descriptor of one operand stage and its advance per MMA, in 16-byte units.
// K-major: rows of 128 K-bytes, 8-row groups 1 KB apart; the next MMA's K slice starts
// kMmaK elements further along the row. MN-major: 64-element MN chunks 8 KB apart, the next
// K slice starts 16 rows (2 KB) further down.
__device__ __forceinline__ uint64_t stage_desc(uint32_t saddr, int mn_major) {
  return mn_major ? sdesc_sw128(saddr, kMnChunkBytes, 1024) : sdesc_sw128(saddr, 16, 1024);
}

template <int AB, int OUT, int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmD, const __grid_constant__ GemmParams p) {
  using Cfg = GemmCfg<BN>;
  constexpr int S = Cfg::kStages;
  constexpr bool kInt = (AB == AB_S8 || AB == AB_U8);
  constexpr int kElemsPerRow = kInt ? 128 : 64;  // K elements per stage
  constexpr int kMmaK = kInt ? 32 : 16;          // K per tcgen05.mma
  constexpr int kMmasPerStage = kElemsPerRow / kMmaK;  // 4
  constexpr uint32_t kDescStep = (kMmaK * (kInt ? 1 : 2)) >> 4;  // 32 bytes -> 2
  constexpr uint32_t kIdesc =
      kInt ? make_idesc(2, AB == AB_S8 ? 1 : 0, AB == AB_S8 ? 1 : 0, 0, 0, kBM, BN)
           : make_idesc(1, AB == AB_BF16 ? 1 : 0, AB == AB_BF16 ? 1 : 0, 0, 0, kBM, BN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_1024(smem_raw);
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * kAStageBytes;
  uint8_t* sStore = smem + S * Cfg::kStageBytes;   // [4 epilogue warps][2][32×32 elements]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sStore + kStoreBytes);
  uint64_t* full = bars;            // [S]  TMA -> MMA
  uint64_t* empty = bars + S;       // [S]  MMA -> TMA
  uint64_t* tfull = bars + 2 * S;   // [2]  MMA -> epilogue
  uint64_t* tempty = tfull + 2;     // [2]  epilogue -> MMA
  uint64_t* drain = tempty + 2;     // [1]  MMA drain on exit
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      bar_init(&full[s], 1);
      bar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      bar_init(&tfull[b], 1);
      bar_init(&tempty[b], 128);
    }
    bar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const WaitGuard g{p.status, abort_flag, p.timeout_ns};
  // Launched with programmatic stream serialization: the setup above may have run while the
  // previous kernel of the stream was finishing; global memory is touched only after it has
  // completed. The next GEMM may start its own setup now (this grid is all resident already).
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer ----------------
    int stage = 0;
    uint32_t phase = 0;
    uint32_t filled_mask = 0;       // stages filled at least once
    uint32_t last_phase[8] = {0};
    bool ok = true;
    const uint64_t pol_a = policy_for(p.l2_mode, true);
    const uint64_t pol_b = policy_for(p.l2_mode, false);
    for (int t = blockIdx.x; t < p.total_tiles && ok; t += gridDim.x) {
      int tm, tn;
      tile_coords(t, p, tm, tn);
      for (int kb = 0; kb < p.num_kb; ++kb) {
        if (!wait_bar(&empty[stage], phase ^ 1, g, 1, t)) { ok = false; break; }
        bar_arrive_expect_tx(&full[stage], Cfg::kStageBytes);
        uint8_t* a_dst = sA + stage * kAStageBytes;
        uint8_t* b_dst = sB + stage * Cfg::kBStageBytes;
        if (!p.a_mn) {
          tma_load_2d_pol(a_dst, &tmA, kb * kElemsPerRow, tm * kBM, &full[stage], p.l2_mode, pol_a);
        } else {
          for (int c = 0; c < kBM / 64; ++c)
            tma_load_2d_pol(a_dst + c * kMnChunkBytes, &tmA, tm * kBM + 64 * c, kb * 64,
                            &full[stage], p.l2_mode, pol_a);
        }
        if (!p.b_mn) {
          tma_load_2d_pol(b_dst, &tmB, kb * kElemsPerRow, tn * BN, &full[stage], p.l2_mode, pol_b);
        } else {
          for (int c = 0; c < BN / 64; ++c)
            tma_load_2d_pol(b_dst + c * kMnChunkBytes, &tmB, tn * BN + 64 * c, kb * 64,
                            &full[stage], p.l2_mode, pol_b);
        }
        filled_mask |= 1u << stage;
        last_phase[stage] = phase;
        if (++stage == S) { stage = 0; phase ^= 1; }
      }
    }
    if (!ok) {
      // Let every copy this thread started land before the CTA's shared memory goes away.
      for (int s = 0; s < S; ++s)
        if (filled_mask & (1u << s)) drain_wait(&full[s], last_phase[s], p.timeout_ns);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: the warp waits, one elected lane issues ----------------
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    const uint32_t a_base = smem_u32(sA);
    const uint32_t b_base = smem_u32(sB);
    // MN-major operands (16-bit only): the transpose bits of the instruction descriptor.
    const uint32_t idesc = kIdesc | ((uint32_t)p.a_mn << 15) | ((uint32_t)p.b_mn << 16);
    const uint32_t a_step = p.a_mn ? (16 * 128) >> 4 : kDescStep;
    const uint32_t b_step = p.b_mn ? (16 * 128) >> 4 : kDescStep;
    for (int t = blockIdx.x; t < p.total_tiles && ok; t += gridDim.x) {
      if (!wait_bar_warp(&tempty[acc], acc_phase ^ 1, g, 2, t)) { ok = false; break; }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * BN;
      for (int kb = 0; kb < p.num_kb; ++kb) {
        if (!wait_bar_warp(&full[stage], phase, g, 3, t)) { ok = false; break; }
        tc_fence_after();
        const uint64_t adesc = stage_desc(a_base + stage * kAStageBytes, p.a_mn);
        const uint64_t bdesc = stage_desc(b_base + stage * Cfg::kBStageBytes, p.b_mn);
#pragma unroll
        for (int k = 0; k < kMmasPerStage; ++k) {
          const uint32_t accum = (kb > 0 || k > 0) ? 1u : 0u;
          if (elect_one()) {
            if constexpr (kInt)
              mma_i8_ss(d_tmem, adesc + k * kDescStep, bdesc + k * kDescStep, kIdesc, accum);
            else
              mma_f16_ss(d_tmem, adesc + k * a_step, bdesc + k * b_step, idesc, accum);
          }
        }
        if (elect_one()) mma_commit(&empty[stage]);
        if (++stage == S) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
      if (elect_one()) mma_commit(&tfull[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    // Every MMA this warp issued has finished before TMEM is released.
    if (elect_one()) mma_commit(drain);
    drain_wait(drain, 0, p.timeout_ns);
  } else if (warp >= 4) {
    // ---------------- epilogue ----------------
    const int ew = warp - 4;             // TMEM lanes 32*ew .. 32*ew+31
    const int row = ew * 32 + lane;
    const uint32_t s_out = smem_u32(sStore) + ew * 2 * kStoreBufBytes;
    uint32_t n_staged = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < p.total_tiles; t += gridDim.x) {
      int tm, tn;
      tile_coords(t, p, tm, tn);
      if (!wait_bar(&tfull[acc], acc_phase, g, 4, t)) break;
      tc_fence_after();
      const int m = tm * kBM + row;
      const bool m_ok = m < p.M;
      const float bias_m =
          (p.bias && p.bias_on_m && m_ok) ? load_as_f32(p.bias, p.bias_kind, m) : 0.f;
      const uint32_t t_row = tmem_base + ((uint32_t)(ew * 32) << 16) + acc * BN;
      drain_acc<OUT, AB, BN / 32>(p, &tmD, t_row, m, tm * kBM + ew * 32, tn * BN, bias_m, s_out,
                              n_staged, [&] {
                                tc_fence_before();
                                bar_arrive(&tempty[acc]);  // accumulator fully read
                              });
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    if (p.stage_out && lane == 0) bulk_wait_group<0>();  // stores done before the CTA exits
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

// ----------------------------------------------------------------------------------------
// CTA-pair variant: a cluster of two CTAs on two SMs computes one 256 x 256 tile with
// tcgen05.mma.cta_group::2 (M = 256, N = 256). CTA r stages rows [128r, 128r+128) of the
// A tile and columns [128r, 128r+128) of the B tile, so each SM streams half of B (32 KB of
// operands per 64-deep k-block instead of 48 KB, and the shared-memory read per MMA drops by
// a third); the even CTA issues the MMAs, both CTAs' TMA loads complete on its barrier, and
// its commits arrive on both CTAs' barriers. Each CTA's epilogue drains its own TMEM rows.
// ----------------------------------------------------------------------------------------
// The pair's tile is 256 × BNP: BNP = 256, or 224 for 32-bit outputs (8192 = 36.6 × 224: 37
// column tiles, so 1024, 2048 or 4096 rows of an 8192-wide output make whole waves of 74
// pairs). CTA r stages B rows [BNP/2·r, BNP/2·(r+1)) of the tile.
constexpr int kPairStages = 6;
constexpr int kPairHalfBytes = 128 * kRowBytes;             // 16 KB: 128 rows x 128 B
constexpr int kPairStageBytes = 2 * kPairHalfBytes;         // A half + B half (BNP = 256)
constexpr int kPairSmemBytes = kPairStages * kPairStageBytes + kStoreBytes + 256 + 1024;

template <int AB, int OUT, int BNP>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmD, const __grid_constant__ GemmParams p) {
  static_assert(BNP == 256 || (BNP == 224 && (OUT == OUT_F32 || OUT == OUT_I32)),
                "the 224-wide pair tile drains 7 chunks: 32-bit outputs only");
  constexpr int S = kPairStages;
  constexpr int kBHalfRows = BNP / 2;
  constexpr int kBHalfBytes = kBHalfRows * kRowBytes;       // 1 KB multiple: swizzle atoms
  constexpr int kStageBytes = kPairHalfBytes + kBHalfBytes;
  constexpr bool kInt = (AB == AB_S8 || AB == AB_U8);
  constexpr int kElemsPerRow = kInt ? 128 : 64;
  constexpr int kMmaK = kInt ? 32 : 16;
  constexpr int kMmasPerStage = kElemsPerRow / kMmaK;
  constexpr uint32_t kDescStep = (kMmaK * (kInt ? 1 : 2)) >> 4;
  constexpr uint32_t kIdesc =
      kInt ? make_idesc(2, AB == AB_S8 ? 1 : 0, AB == AB_S8 ? 1 : 0, 0, 0, 256, BNP)
           : make_idesc(1, AB == AB_BF16 ? 1 : 0, AB == AB_BF16 ? 1 : 0, 0, 0, 256, BNP);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_1024(smem_raw);
  uint8_t* sA = smem;                        // [S][128 rows][128 B]
  uint8_t* sB = smem + S * kPairHalfBytes;   // [S][BNP/2 rows][128 B]
  uint8_t* sStore = smem + S * kPairStageBytes;    // [4 epilogue warps][2][32×32 elements]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sStore + kStoreBytes);
  uint64_t* full = bars;            // [S]  leader: both CTAs' TMA bytes
  uint64_t* empty = bars + S;       // [S]  both: MMA done with the stage
  uint64_t* tfull = bars + 2 * S;   // [2]  both: accumulator ready
  uint64_t* tempty = tfull + 2;     // [2]  leader: 8 epilogue warps released it
  uint64_t* drain = tempty + 2;     // [1]  leader
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster_id = blockIdx.x >> 1;
  const int nclusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      bar_init(&full[s], 1);
      bar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      bar_init(&tfull[b], 1);
      bar_init(&tempty[b], 8);
    }
    bar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 2) {
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncwarp();        // barrier.cluster is .aligned: whole warps
  cluster_sync_all();  // barriers of both CTAs initialised before any remote signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const WaitGuard g{p.status, abort_flag, p.timeout_ns};
  // Programmatic stream serialization, as in the one-CTA kernel: global memory only after
  // the previous kernel of the stream has completed; the next may be scheduled now (it gets
  // SMs as this grid's CTAs exit).
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    int stage = 0;
    uint32_t phase = 0;
    uint32_t filled_mask = 0;
    uint32_t last_phase[kPairStages] = {0};
    bool ok = true;
    const uint64_t pol_a = p.l2_mode == 2 ? policy_evict_normal() : policy_for(p.l2_mode, true);
    const uint64_t pol_b = p.l2_mode == 2 ? policy_evict_normal() : policy_for(p.l2_mode, false);
    for (int t = cluster_id; t < p.total_tiles && ok; t += nclusters) {
      int tm, tn;
      tile_coords(t, p, tm, tn);
      for (int kb = 0; kb < p.num_kb; ++kb) {
        if (!wait_bar(&empty[stage], phase ^ 1, g, 31, t)) { ok = false; break; }
        const uint32_t full_leader = mapa_shared(smem_u32(&full[stage]), 0);
        if (leader) bar_arrive_expect_tx(&full[stage], 2 * kStageBytes);
        uint8_t* a_dst = sA + stage * kPairHalfBytes;
        uint8_t* b_dst = sB + stage * kBHalfBytes;
        const int a_row = tm * 256 + 128 * (int)rank;
        const int b_row = tn * BNP + kBHalfRows * (int)rank;
        if (!p.a_mn) {
          tma_load_2d_pair(a_dst, &tmA, kb * kElemsPerRow, a_row, full_leader, pol_a);
        } else {
          tma_load_2d_pair(a_dst, &tmA, a_row, kb * 64, full_leader, pol_a);
          tma_load_2d_pair(a_dst + kMnChunkBytes, &tmA, a_row + 64, kb * 64, full_leader, pol_a);
        }
        if (!p.b_mn) {
          tma_load_2d_pair(b_dst, &tmB, kb * kElemsPerRow, b_row, full_leader, pol_b);
        } else {
          tma_load_2d_pair(b_dst, &tmB, b_row, kb * 64, full_leader, pol_b);
          tma_load_2d_pair(b_dst + kMnChunkBytes, &tmB, b_row + 64, kb * 64, full_leader, pol_b);
        }
        filled_mask |= 1u << stage;
        last_phase[stage] = phase;
        if (++stage == S) { stage = 0; phase ^= 1; }
      }
    }
    if (!ok && leader) {
      for (int s = 0; s < S; ++s)
        if (filled_mask & (1u << s)) drain_wait(&full[s], last_phase[s], p.timeout_ns);
    }
  } else if (warp == 1 && leader) {
    // ---------------- MMA issuer (even CTA of the pair; one elected lane issues) --------
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    const uint32_t a_base = smem_u32(sA);
    const uint32_t b_base = smem_u32(sB);
    const uint32_t idesc = kIdesc | ((uint32_t)p.a_mn << 15) | ((uint32_t)p.b_mn << 16);
    const uint32_t a_step = p.a_mn ? (16 * 128) >> 4 : kDescStep;
    const uint32_t b_step = p.b_mn ? (16 * 128) >> 4 : kDescStep;
    for (int t = cluster_id; t < p.total_tiles && ok; t += nclusters) {
      if (!wait_bar_warp(&tempty[acc], acc_phase ^ 1, g, 32, t)) { ok = false; break; }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * BNP;
      for (int kb = 0; kb < p.num_kb; ++kb) {
        if (!wait_bar_warp(&full[stage], phase, g, 33, t)) { ok = false; break; }
        tc_fence_after();
        const uint64_t adesc = stage_desc(a_base + stage * kPairHalfBytes, p.a_mn);
        const uint64_t bdesc = stage_desc(b_base + stage * kBHalfBytes, p.b_mn);
#pragma unroll
        for (int k = 0; k < kMmasPerStage; ++k) {
          const uint32_t accum = (kb > 0 || k > 0) ? 1u : 0u;
          if (elect_one()) {
            if constexpr (kInt)
              mma_i8_ss_pair(d_tmem, adesc + k * kDescStep, bdesc + k * kDescStep, kIdesc, accum);
            else
              mma_f16_ss_pair(d_tmem, adesc + k * a_step, bdesc + k * b_step, idesc, accum);
          }
        }
        const uint32_t e = smem_u32(&empty[stage]);
        if (elect_one()) {
          mma_commit_pair(mapa_shared(e, 0));
          mma_commit_pair(mapa_shared(e, 1));
        }
        if (++stage == S) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
      const uint32_t f = smem_u32(&tfull[acc]);
      if (elect_one()) {
        mma_commit_pair(mapa_shared(f, 0));
        mma_commit_pair(mapa_shared(f, 1));
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    if (elect_one()) mma_commit_pair(mapa_shared(smem_u32(drain), 0));
    drain_wait(drain, 0, p.timeout_ns);
  } else if (warp >= 4) {
    // ---------------- epilogue (both CTAs, own TMEM rows) ----------------
    const int ew = warp - 4;
    const int row = ew * 32 + lane;
    const uint32_t s_out = smem_u32(sStore) + ew * 2 * kStoreBufBytes;
    uint32_t n_staged = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = cluster_id; t < p.total_tiles; t += nclusters) {
      int tm, tn;
      tile_coords(t, p, tm, tn);
      if (!wait_bar(&tfull[acc], acc_phase, g, 34, t)) break;
      tc_fence_after();
      const int m0 = tm * 256 + 128 * (int)rank;
      const int m = m0 + row;
      const bool m_ok = m < p.M;
      const float bias_m =
          (p.bias && p.bias_on_m && m_ok) ? load_as_f32(p.bias, p.bias_kind, m) : 0.f;
      const uint32_t t_row = tmem_base + ((uint32_t)(ew * 32) << 16) + acc * BNP;
      drain_acc<OUT, AB, BNP / 32>(p, &tmD, t_row, m, m0 + ew * 32, tn * BNP, bias_m, s_out,
                                   n_staged, [&] {
        tc_fence_before();
        __syncwarp();
        // TMEM read (tcgen05.wait::ld) and fenced: a CTA-scope release suffices, and skips
        // the cluster-scope release of the staging writes (small-K GEMM: +30 %).
        if (lane == 0) bar_arrive_cluster_cta(mapa_shared(smem_u32(&tempty[acc]), 0));
      });
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    if (p.stage_out && lane == 0) bulk_wait_group<0>();  // stores done before the CTA exits
  }

  tc_fence_before();
  __syncwarp();
  cluster_sync_all();  // the pair's MMAs are done with both CTAs' shared memory and TMEM
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 512);
  }
}

// ----------------------------------------------------------------------------------------
// Tall CTA-pair variant: the pair computes a 512 × 256 tile as two 256-row blocks, each one
// cta_group::2 MMA chain (M = 256, N = 256) into its own TMEM accumulator (columns 0-255 and
// 256-511 of both CTAs): per 64-deep k-block a CTA stages two 128-row halves of A (one per
// row block) and one 128-row half of B, so each B half feeds twice the MMAs of the square
// pair kernel and the operand traffic from L2 per FLOP is 3/4 of it (48 KB per CTA for two
// 256×256×64 products instead of 32 KB for one). TMEM then holds one tile, not two: the
// epilogue drains block 0, then block 1, and the MMA warp starts the next tile's block-0
// products as soon as block 0 is drained, running up to the ring's depth ahead of block 1
// (whose products wait for block 1's drain) and catching block 1 up once it is free.
// ----------------------------------------------------------------------------------------
constexpr int kTallStages = 4;
constexpr int kTallStageBytes = 3 * kPairHalfBytes;         // A half 0, A half 1, B half
constexpr int kTallSmemBytes = kTallStages * kTallStageBytes + kStoreBytes + 256 + 1024;
static_assert(kTallSmemBytes <= 232448, "tall pair stages exceed the shared-memory budget");

template <int AB, int OUT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tall_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmD, const __grid_constant__ GemmParams p) {
  constexpr int S = kTallStages;
  constexpr bool kInt = (AB == AB_S8 || AB == AB_U8);
  constexpr int kElemsPerRow = kInt ? 128 : 64;
  constexpr int kMmaK = kInt ? 32 : 16;
  constexpr int kMmasPerStage = kElemsPerRow / kMmaK;
  constexpr uint32_t kDescStep = (kMmaK * (kInt ? 1 : 2)) >> 4;
  constexpr uint32_t kIdesc =
      kInt ? make_idesc(2, AB == AB_S8 ? 1 : 0, AB == AB_S8 ? 1 : 0, 0, 0, 256, 256)
           : make_idesc(1, AB == AB_BF16 ? 1 : 0, AB == AB_BF16 ? 1 : 0, 0, 0, 256, 256);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_1024(smem_raw);
  uint8_t* sA = smem;                              // [S][2 halves][128 rows][128 B]
  uint8_t* sB = smem + S * 2 * kPairHalfBytes;     // [S][128 rows][128 B]
  uint8_t* sStore = smem + S * kTallStageBytes;    // [4 epilogue warps][2][32×32 elements]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sStore + kStoreBytes);
  uint64_t* full = bars;            // [S]  leader: both CTAs' TMA bytes
  uint64_t* empty = bars + S;       // [S]  both: both row blocks' MMAs done with the stage
  uint64_t* tfull = bars + 2 * S;   // [2]  both: row block b's accumulator ready
  uint64_t* tempty = tfull + 2;     // [2]  leader: 8 epilogue warps drained row block b
  uint64_t* drain = tempty + 2;     // [1]  leader
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster_id = blockIdx.x >> 1;
  const int nclusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      bar_init(&full[s], 1);
      bar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      bar_init(&tfull[b], 1);
      bar_init(&tempty[b], 8);
    }
    bar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 2) {
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncwarp();        // barrier.cluster is .aligned: whole warps
  cluster_sync_all();  // barriers of both CTAs initialised before any remote signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const WaitGuard g{p.status, abort_flag, p.timeout_ns};
  // Programmatic stream serialization, as in the one-CTA kernel: global memory only after
  // the previous kernel of the stream has completed; the next may be scheduled now (it gets
  // SMs as this grid's CTAs exit).
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    int stage = 0;
    uint32_t phase = 0;
    uint32_t filled_mask = 0;
    uint32_t last_phase[kTallStages] = {0};
    bool ok = true;
    const uint64_t pol_a = p.l2_mode == 2 ? policy_evict_normal() : policy_for(p.l2_mode, true);
    const uint64_t pol_b = p.l2_mode == 2 ? policy_evict_normal() : policy_for(p.l2_mode, false);
    for (int t = cluster_id; t < p.total_tiles && ok; t += nclusters) {
      int tm, tn;
      tile_coords(t, p, tm, tn);
      for (int kb = 0; kb < p.num_kb; ++kb) {
        if (!wait_bar(&empty[stage], phase ^ 1, g, 41, t)) { ok = false; break; }
        const uint32_t full_leader = mapa_shared(smem_u32(&full[stage]), 0);
        if (leader) bar_arrive_expect_tx(&full[stage], 2 * kTallStageBytes);
        uint8_t* b_dst = sB + stage * kPairHalfBytes;
        const int b_row = tn * 256 + 128 * (int)rank;
        for (int h = 0; h < 2; ++h) {
          uint8_t* a_dst = sA + (stage * 2 + h) * kPairHalfBytes;
          const int a_row = tm * 512 + 256 * h + 128 * (int)rank;
          if (!p.a_mn) {
            tma_load_2d_pair(a_dst, &tmA, kb * kElemsPerRow, a_row, full_leader, pol_a);
          } else {
            tma_load_2d_pair(a_dst, &tmA, a_row, kb * 64, full_leader, pol_a);
            tma_load_2d_pair(a_dst + kMnChunkBytes, &tmA, a_row + 64, kb * 64, full_leader, pol_a);
          }
        }
        if (!p.b_mn) {
          tma_load_2d_pair(b_dst, &tmB, kb * kElemsPerRow, b_row, full_leader, pol_b);
        } else {
          tma_load_2d_pair(b_dst, &tmB, b_row, kb * 64, full_leader, pol_b);
          tma_load_2d_pair(b_dst + kMnChunkBytes, &tmB, b_row + 64, kb * 64, full_leader, pol_b);
        }
        filled_mask |= 1u << stage;
        last_phase[stage] = phase;
        if (++stage == S) { stage = 0; phase ^= 1; }
      }
    }
    if (!ok && leader) {
      for (int s = 0; s < S; ++s)
        if (filled_mask & (1u << s)) drain_wait(&full[s], last_phase[s], p.timeout_ns);
    }
  } else if (warp == 1 && leader) {
    // ---------------- MMA issuer (even CTA of the pair; one elected lane issues) --------
    // Two cursors walk the same ring: row block 0 (s0) leads, row block 1 (s1) follows and
    // releases each stage to the producer once both blocks have consumed it.
    int s0 = 0, s1 = 0;
    uint32_t ph0 = 0, ph1 = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    const uint32_t a_base = smem_u32(sA);
    const uint32_t b_base = smem_u32(sB);
    const uint32_t idesc = kIdesc | ((uint32_t)p.a_mn << 15) | ((uint32_t)p.b_mn << 16);
    const uint32_t a_step = p.a_mn ? (16 * 128) >> 4 : kDescStep;
    const uint32_t b_step = p.b_mn ? (16 * 128) >> 4 : kDescStep;
    auto issue = [&](int blk, int stage, bool first) {
      const uint64_t adesc = stage_desc(a_base + (stage * 2 + blk) * kPairHalfBytes, p.a_mn);
      const uint64_t bdesc = stage_desc(b_base + stage * kPairHalfBytes, p.b_mn);
      const uint32_t d_tmem = tmem_base + 256 * blk;
#pragma unroll
      for (int k = 0; k < kMmasPerStage; ++k) {
        const uint32_t accum = (!first || k > 0) ? 1u : 0u;
        if (elect_one()) {
          if constexpr (kInt)
            mma_i8_ss_pair(d_tmem, adesc + k * kDescStep, bdesc + k * kDescStep, kIdesc, accum);
          else
            mma_f16_ss_pair(d_tmem, adesc + k * a_step, bdesc + k * b_step, idesc, accum);
        }
      }
    };
    auto commit_both = [&](uint64_t* bar) {
      const uint32_t a = smem_u32(bar);
      if (elect_one()) {
        mma_commit_pair(mapa_shared(a, 0));
        mma_commit_pair(mapa_shared(a, 1));
      }
    };
    for (int t = cluster_id; t < p.total_tiles && ok; t += nclusters) {
      if (!wait_bar_warp(&tempty[0], acc_phase ^ 1, g, 42, t)) { ok = false; break; }
      tc_fence_after();
      bool free1 = false;
      int kb1 = 0;
      // row block 1's products for k-blocks kb1..upto (their stages are full already)
      auto catch_up = [&](int upto) {
        for (; kb1 <= upto; ++kb1) {
          issue(1, s1, kb1 == 0);
          commit_both(&empty[s1]);
          if (++s1 == S) { s1 = 0; ph1 ^= 1; }
        }
      };
      for (int kb0 = 0; kb0 < p.num_kb; ++kb0) {
        if (!wait_bar_warp(&full[s0], ph0, g, 43, t)) { ok = false; break; }
        tc_fence_after();
        issue(0, s0, kb0 == 0);
        if (++s0 == S) { s0 = 0; ph0 ^= 1; }
        if (!free1) {
          free1 = __all_sync(0xffffffffu, bar_test_wait(smem_u32(&tempty[1]), acc_phase ^ 1));
          if (!free1 && kb0 + 1 - kb1 >= S) {   // every stage is held: block 1 must move
            if (!wait_bar_warp(&tempty[1], acc_phase ^ 1, g, 44, t)) { ok = false; break; }
            free1 = true;
          }
          if (free1) tc_fence_after();
        }
        if (free1) catch_up(kb0);
      }
      if (!ok) break;
      commit_both(&tfull[0]);
      if (!free1) {
        if (!wait_bar_warp(&tempty[1], acc_phase ^ 1, g, 44, t)) { ok = false; break; }
        tc_fence_after();
      }
      catch_up(p.num_kb - 1);
      commit_both(&tfull[1]);
      acc_phase ^= 1;
    }
    if (elect_one()) mma_commit_pair(mapa_shared(smem_u32(drain), 0));
    drain_wait(drain, 0, p.timeout_ns);
  } else if (warp >= 4) {
    // ---------------- epilogue (both CTAs, own TMEM rows; block 0, then block 1) -------
    const int ew = warp - 4;
    const int row = ew * 32 + lane;
    const uint32_t s_out = smem_u32(sStore) + ew * 2 * kStoreBufBytes;
    uint32_t n_staged = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int t = cluster_id; t < p.total_tiles && ok; t += nclusters) {
      int tm, tn;
      tile_coords(t, p, tm, tn);
      for (int blk = 0; blk < 2; ++blk) {
        if (!wait_bar(&tfull[blk], acc_phase, g, 45, t)) { ok = false; break; }
        tc_fence_after();
        const int m0 = tm * 512 + 256 * blk + 128 * (int)rank;
        const int m = m0 + row;
        const bool m_ok = m < p.M;
        const float bias_m =
            (p.bias && p.bias_on_m && m_ok) ? load_as_f32(p.bias, p.bias_kind, m) : 0.f;
        const uint32_t t_row = tmem_base + ((uint32_t)(ew * 32) << 16) + 256 * blk;
        drain_acc<OUT, AB, 8>(p, &tmD, t_row, m, m0 + ew * 32, tn * 256, bias_m, s_out,
                              n_staged, [&] {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) bar_arrive_cluster_cta(mapa_shared(smem_u32(&tempty[blk]), 0));
        });
      }
      acc_phase ^= 1;
    }
    if (p.stage_out && lane == 0) bulk_wait_group<0>();  // stores done before the CTA exits
  }

  tc_fence_before();
  __syncwarp();
  cluster_sync_all();  // the pair's MMAs are done with both CTAs' shared memory and TMEM
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 512);
  }
}

// ----------------------------------------------------------------------------------------
// Host side
// ----------------------------------------------------------------------------------------
namespace {

int ab_kind_of(int dt) {
  switch (dt) {
    case LVB_F16: return AB_F16;
    case LVB_BF16: return AB_BF16;
    case LVB_I8: return AB_S8;
    case LVB_U8: return AB_U8;
  }
  return -1;
}
int out_kind_of(int dt) {
  switch (dt) {
    case LVB_F32: return OUT_F32;
    case LVB_F16: return OUT_F16;
    case LVB_BF16: return OUT_BF16;
    case LVB_I32:
    case LVB_U32: return OUT_I32;
  }
  return -1;
}

template <int AB, int OUT, int BN>
int launch_t(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& td,
             const GemmParams& p, int ctas,
             cudaStream_t stream, DeviceState* dev) {
  using Cfg = GemmCfg<BN>;
  auto kern = gemm_tc_kernel<AB, OUT, BN>;
  // The attribute is per function and per device: set once per device (two threads setting
  // it at once set the same value).
  static std::atomic<bool> attr_set[kMaxDevices];
  const int dv = dev->device >= 0 && dev->device < kMaxDevices ? dev->device : 0;
  cudaError_t e;
  if (!attr_set[dv].load(std::memory_order_acquire)) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
    if (e != cudaSuccess) return fail_cuda(e, "lvb_gemm", "cudaFuncSetAttribute");
    attr_set[dv].store(true, std::memory_order_release);
  }
  // Programmatic stream serialization: a small GEMM's launch latency and setup (barriers,
  // TMEM allocation, descriptor prefetch) overlap the previous kernel of the stream; the
  // kernel waits for that kernel before its first global memory access.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, ta, tb, td, p);
  if (e != cudaSuccess) return fail_cuda(e, "lvb_gemm", "kernel launch");
  return LVB_OK;
}

// Persistent pair kernel: one cluster of 2 per SM pair, capped by how many clusters of this
// kernel can be resident at once (GPC boundaries can leave an SM without a partner).
template <int AB, int OUT, int BNP>
int launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& td,
                const GemmParams& p, int clusters,
                cudaStream_t stream, DeviceState* dev) {
  auto kern = gemm_tc2_kernel<AB, OUT, BNP>;
  static std::atomic<bool> attr_set[kMaxDevices];
  const int dva = dev->device >= 0 && dev->device < kMaxDevices ? dev->device : 0;
  cudaError_t e;
  if (!attr_set[dva].load(std::memory_order_acquire)) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kPairSmemBytes);
    if (e != cudaSuccess) return fail_cuda(e, "lvb_gemm", "cudaFuncSetAttribute");
    attr_set[dva].store(true, std::memory_order_release);
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kPairSmemBytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  static std::mutex mu;
  static int resident[kMaxDevices] = {0};
  {
    std::lock_guard<std::mutex> lk(mu);
    if (resident[dva] == 0) {
      int n = 0;
      cfg.gridDim = dim3(2 * std::max(1, dev->sm_count / 2));
      if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0)
        n = std::max(1, dev->sm_count / 2);
      cudaGetLastError();
      resident[dva] = n;
    }
    clusters = std::min(clusters, resident[dva]);
  }
  cfg.gridDim = dim3(2 * std::max(1, clusters));
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.numAttrs = 2;
  e = cudaLaunchKernelEx(&cfg, kern, ta, tb, td, p);
  if (e != cudaSuccess) return fail_cuda(e, "lvb_gemm", "cluster kernel launch");
  return LVB_OK;
}

// The tall pair kernel (512 × 256 tiles), launched like launch_pair.
template <int AB, int OUT>
int launch_tall(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& td,
                const GemmParams& p, int clusters, cudaStream_t stream, DeviceState* dev) {
  auto kern = gemm_tall_kernel<AB, OUT>;
  static std::atomic<bool> attr_set[kMaxDevices];
  const int dva = dev->device >= 0 && dev->device < kMaxDevices ? dev->device : 0;
  cudaError_t e;
  if (!attr_set[dva].load(std::memory_order_acquire)) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kTallSmemBytes);
    if (e != cudaSuccess) return fail_cuda(e, "lvb_gemm", "cudaFuncSetAttribute");
    attr_set[dva].store(true, std::memory_order_release);
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kTallSmemBytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  static std::mutex mu;
  static int resident[kMaxDevices] = {0};
  {
    std::lock_guard<std::mutex> lk(mu);
    if (resident[dva] == 0) {
      int n = 0;
      cfg.gridDim = dim3(2 * std::max(1, dev->sm_count / 2));
      if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0)
        n = std::max(1, dev->sm_count / 2);
      cudaGetLastError();
      resident[dva] = n;
    }
    clusters = std::min(clusters, resident[dva]);
  }
  cfg.gridDim = dim3(2 * std::max(1, clusters));
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.numAttrs = 2;
  e = cudaLaunchKernelEx(&cfg, kern, ta, tb, td, p);
  if (e != cudaSuccess) return fail_cuda(e, "lvb_gemm", "cluster kernel launch");
  return LVB_OK;
}

template <int AB, int OUT>
int launch_bn(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& td,
              const GemmParams& p, int ctas, cudaStream_t s, DeviceState* dev) {
  if (bn == 1024) return launch_tall<AB, OUT>(ta, tb, td, p, ctas / 2, s, dev);
  if (bn == 512) return launch_pair<AB, OUT, 256>(ta, tb, td, p, ctas / 2, s, dev);
  if (bn == 448) {   // CTA pairs with 256 x 224 tiles (32-bit outputs, B read K-major)
    if constexpr (OUT == OUT_F32 || OUT == OUT_I32) {
      if (p.b_mn) return fail(LVB_ERR_UNSUPPORTED, "lvb_gemm", "224-wide pair tile with MN-major B");
      return launch_pair<AB, OUT, 224>(ta, tb, td, p, ctas / 2, s, dev);
    }
    return fail(LVB_ERR_UNSUPPORTED, "lvb_gemm", "224-wide pair tile with a 16-bit output");
  }
  switch (bn) {
    case 256: return launch_t<AB, OUT, 256>(ta, tb, td, p, ctas, s, dev);
    case 128: return launch_t<AB, OUT, 128>(ta, tb, td, p, ctas, s, dev);
    case 64: return launch_t<AB, OUT, 64>(ta, tb, td, p, ctas, s, dev);
  }
  return fail(LVB_ERR_UNSUPPORTED, "lvb_gemm", "tile width not built");
}

}  // namespace

int gemm_smem_bytes(int bn) {
  switch (bn) {
    case 1024: return kTallSmemBytes;
    case 512:
    case 448: return kPairSmemBytes;
    case 256: return GemmCfg<256>::kSmemBytes;
    case 128: return GemmCfg<128>::kSmemBytes;
    case 64: return GemmCfg<64>::kSmemBytes;
  }
  return 0;
}
int gemm_stages(int bn) {
  switch (bn) {
    case 1024: return kTallStages;
    case 512:
    case 448: return kPairStages;
    case 256: return GemmCfg<256>::kStages;
    case 128: return GemmCfg<128>::kStages;
    case 64: return GemmCfg<64>::kStages;
  }
  return 0;
}

// K == 0: C = 0 (the empty sum), written through the same clamped addressing.
__global__ void gemm_zero_kernel(uint8_t* C, long long rows, long long cols, long long ld,
                                 int esize) {
  const long long total = rows * cols;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i % rows, c = i / rows;
    uint8_t* p = C + (c * ld + r) * esize;
    for (int b = 0; b < esize; ++b) p[b] = 0;
  }
}

int gemm_zero_fill(const lvb_gemm_desc* d, void* C, cudaStream_t stream) {
  // Lane-contiguous dimension first: column-major C has M contiguous, row-major N.
  const long long rows = d->c_rowmajor ? d->N : d->M;
  const long long cols = d->c_rowmajor ? d->M : d->N;
  const int es = dtype_size(d->c_type);
  const long long total = rows * cols;
  const int blocks = (int)std::min<long long>((total + 255) / 256, 4096);
  gemm_zero_kernel<<<blocks, 256, 0, stream>>>(reinterpret_cast<uint8_t*>(C), rows, cols, d->ldc,
                                               es);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LVB_OK : fail_cuda(e, "lvb_gemm", "zero-fill launch");
}

// Copies `rows` rows of `cols` elements (row stride `ld` elements, any alignment) into a
// dense buffer with row stride `dld` (a 16-byte multiple), zero-filling columns cols..dld-1,
// so a tensor map can describe it. Used when a caller's operand has a leading dimension or
// base address TMA cannot address; it is one extra pass over that operand.
template <typename T>
__global__ void repack_kernel(const T* __restrict__ src, long long rows, long long cols,
                              long long ld, T* __restrict__ dst, long long dld) {
  const long long total = rows * dld;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / dld, c = i - r * dld;
    dst[i] = c < cols ? src[r * ld + c] : T(0);
  }
}

// The same for an operand stored MN-contiguous: element (r, c) of the K-major result (r < rows
// along M or N, c < cols along K) sits at src[c*ld + r]. 32×32 tiles through shared memory,
// so both the read (along r) and the write (along c) are coalesced.
template <typename T>
__global__ void transpose_repack_kernel(const T* __restrict__ src, long long rows, long long cols,
                                        long long ld, T* __restrict__ dst, long long dld) {
  __shared__ T tile[32][33];
  const long long tiles_r = (rows + 31) / 32, tiles_c = (dld + 31) / 32;
  for (long long t = blockIdx.x; t < tiles_r * tiles_c; t += gridDim.x) {
    const long long r0 = (t % tiles_r) * 32, c0 = (t / tiles_r) * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
      const long long r = r0 + threadIdx.x, c = c0 + i;
      tile[i][threadIdx.x] = (r < rows && c < cols) ? src[c * ld + r] : T(0);
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
      const long long r = r0 + i, c = c0 + threadIdx.x;
      if (r < rows && c < dld) dst[r * dld + c] = tile[threadIdx.x][i];
    }
    __syncthreads();
  }
}

// Copy an operand of `rows` (M or N) × `cols` (K) into a dense K-major buffer with row
// stride `dld`; `mn_major` when the source is stored MN-contiguous (then it is transposed).
static int repack(const void* src, int esize, long long rows, long long cols, long long ld,
                  bool mn_major, void* dst, long long dld, cudaStream_t s) {
  if (mn_major) {
    const long long tiles = ((rows + 31) / 32) * ((dld + 31) / 32);
    const int blocks = (int)std::min<long long>(tiles, 8192);
    const dim3 tb(32, 8);
    if (esize == 1)
      transpose_repack_kernel<uint8_t><<<blocks, tb, 0, s>>>((const uint8_t*)src, rows, cols, ld,
                                                             (uint8_t*)dst, dld);
    else
      transpose_repack_kernel<uint16_t><<<blocks, tb, 0, s>>>((const uint16_t*)src, rows, cols,
                                                              ld, (uint16_t*)dst, dld);
  } else {
    const long long total = rows * dld;
    const int blocks = (int)std::min<long long>((total + 255) / 256, 8192);
    if (esize == 1)
      repack_kernel<uint8_t><<<blocks, 256, 0, s>>>((const uint8_t*)src, rows, cols, ld,
                                                     (uint8_t*)dst, dld);
    else
      repack_kernel<uint16_t><<<blocks, 256, 0, s>>>((const uint16_t*)src, rows, cols, ld,
                                                      (uint16_t*)dst, dld);
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LVB_OK : fail_cuda(e, "lvb_gemm", "repack launch");
}

// K == 0 with an epilogue: the accumulator is its initial value bias + R, then the
// activation, converted and stored (kernel space, like the GEMM's own epilogue).
template <int OUT>
__global__ void gemm_epilogue_only_kernel(const __grid_constant__ GemmParams p) {
  const long long total = (long long)p.M * p.N;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int m = (int)(i % p.M), n = (int)(i / p.M);
    const float bias_m = (p.bias && p.bias_on_m) ? load_as_f32(p.bias, p.bias_kind, m) : 0.f;
    store_out<OUT>(p.D, (long long)n * p.ldd + m, __float_as_uint(epi_value(p, 0.f, m, n, bias_m)));
  }
}

int gemm_launch_aligned(const lvb_gemm_desc* d, const lvb_gemm_plan& plan, const void* A,
                        const void* B, void* C, const lvb_epilogue* epi, cudaStream_t stream,
                        DeviceState* dev);

int gemm_launch(const lvb_gemm_desc* d, const lvb_gemm_plan& plan, const void* A, const void* B,
                void* C, const lvb_epilogue* epi, cudaStream_t stream, DeviceState* dev) {
  if (!plan.repack_a && !plan.repack_b)
    return gemm_launch_aligned(d, plan, A, B, C, epi, stream, dev);
  // Stream-ordered workspace for the repacked operand(s); freed on the same stream.
  const int es = dtype_size(d->a_type);
  const long long kp = (d->K + 15) / 16 * 16;  // 16 elements: a 16-byte multiple for 1 and 2 bytes
  const size_t bytes_a = plan.repack_a ? (size_t)d->M * kp * es : 0;
  const size_t bytes_b = plan.repack_b ? (size_t)d->N * kp * es : 0;
  void* ws = nullptr;
  cudaError_t e = workspace_alloc(dev, &ws, bytes_a + bytes_b, stream);
  if (e != cudaSuccess) return fail_cuda(e, "lvb_gemm", "workspace cudaMallocAsync");
  lvb_gemm_desc d2 = *d;
  lvb_gemm_plan plan2 = plan;
  const void* a = A;
  const void* b = B;
  int st = LVB_OK;
  if (plan.repack_a) {
    st = repack(A, es, d->M, d->K, d->lda, !d->a_rowmajor, ws, kp, stream);
    a = ws;
    d2.lda = kp;
    d2.a_rowmajor = 1;
    plan2.a_mnmajor = 0;
  }
  if (st == LVB_OK && plan.repack_b) {
    void* wb = (uint8_t*)ws + bytes_a;
    st = repack(B, es, d->N, d->K, d->ldb, d->b_rowmajor != 0, wb, kp, stream);
    b = wb;
    d2.ldb = kp;
    d2.b_rowmajor = 0;
    plan2.b_mnmajor = 0;
  }
  if (st == LVB_OK) st = gemm_launch_aligned(&d2, plan2, a, b, C, epi, stream, dev);
  e = cudaFreeAsync(ws, stream);
  if (st == LVB_OK && e != cudaSuccess) return fail_cuda(e, "lvb_gemm", "workspace cudaFreeAsync");
  return st;
}

// ----------------------------------------------------------------------------------------
// GEMM without allocation (lvb_gemm_noalloc)
//
// Some hosts may not allocate device memory at the moment they run a GEMM: a runtime that
// owns every byte of device memory through its own pool and forbids allocations behind its
// back, or a serving loop that must not allocate after warm-up. For them the scratch this
// GEMM needs lives in one file-scope device array instead: the device status word at its
// head, and the workspace that operands TMA cannot address (base or leading dimension not a
// 16-byte multiple) are repacked into. Every GPU that loads the library keeps this array until the process exits.
// ----------------------------------------------------------------------------------------
constexpr size_t kNoAllocHeadBytes = 256;                   // DevStatus, padded
constexpr size_t kNoAllocWorkspaceBytes = 16ull << 20;      // repack workspace: 16 MiB
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocHeadBytes + kNoAllocWorkspaceBytes];

// Identity of the calling thread's current CUDA context (cuCtxGetId through the runtime's
// driver entry point; 0 when unavailable). A device reset destroys the primary context and
// the next one has a new id, with the module — and the array — loaded afresh.
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);
static unsigned long long current_context_id() {
  static std::once_flag once;
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess && q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess && q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
    cudaGetLastError();
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current && get_id && get_current(&ctx) == CUDA_SUCCESS && ctx &&
      get_id(ctx, &id) == CUDA_SUCCESS)
    return id;
  return 0;
}

// Device address of g_noalloc_scratch, looked up once per device (and again if the device's
// context was replaced, e.g. after cudaDeviceReset) with that device current: host code may
// not use the symbol itself as a device pointer. The lookup loads this file's module when
// CUDA loads modules lazily, which is when the array itself is placed on the device.
struct NoallocScratch {
  void* addr = nullptr;
  unsigned long long ctx = 0;
};
static std::mutex g_noalloc_mu;
static NoallocScratch g_noalloc[128];

static int noalloc_scratch(int device, void** out, const char* op) {
  if (device < 0 || device >= 128) return fail(LVB_ERR_UNSUPPORTED, op, "device ordinal above 127");
  // No context may be current on this thread yet (id 0): then the lookup runs, which makes
  // the device's primary context current, and its id is recorded after it.
  const unsigned long long ctx = current_context_id();
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  NoallocScratch& slot = g_noalloc[device];
  if (!slot.addr || ctx == 0 || slot.ctx != ctx) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return fail_cuda(e, op, "cudaGetSymbolAddress(scratch)");
    slot.addr = p;
    slot.ctx = current_context_id();
  }
  *out = slot.addr;
  return LVB_OK;
}

// The status word of lvb_gemm_noalloc on the current device (for its reader and self-test).
int noalloc_status_word(DevStatus** out, const char* op) {
  int device = -1;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess)
    return fail(LVB_ERR_NO_DEVICE, op, std::string("no CUDA device: ") + cudaGetErrorString(e));
  void* scratch = nullptr;
  int st = noalloc_scratch(device, &scratch, op);
  if (st) return st;
  *out = reinterpret_cast<DevStatus*>(scratch);
  return LVB_OK;
}

}  // namespace lvb

extern "C" int lvb_gemm_noalloc(const lvb_gemm_desc* d, const void* A, const void* B, void* C,
                                void* stream) {
  using namespace lvb;
  const char* op = "lvb_gemm_noalloc";
  int st = lvb_gemm_check(d);
  if (st) return st;
  if (d->M == 0 || d->N == 0) return LVB_OK;
  if (!C) return fail(LVB_ERR_INVALID_ARG, op, "C is NULL");
  if (d->K > 0 && (!A || !B)) return fail(LVB_ERR_INVALID_ARG, op, "A or B is NULL");
  const int es = dtype_size(d->a_type);
  if (((uintptr_t)A) % es || ((uintptr_t)B) % es || ((uintptr_t)C) % dtype_size(d->c_type))
    return fail(LVB_ERR_INVALID_ARG, op, "pointer not aligned to its element size");
  int device = -1, major = 0, minor = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess)
    return fail(LVB_ERR_NO_DEVICE, op, std::string("no CUDA device: ") + cudaGetErrorString(e));
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (major != 10 || minor != 0)
    return fail(LVB_ERR_NO_DEVICE, op, "device is not sm_100", "run on a B200");
  void* scratch = nullptr;
  st = noalloc_scratch(device, &scratch, op);
  if (st) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);

  if (d->K > 0 && gemv_applies(d)) {
    // A matrix-vector product: the streaming kernel reads any alignment and layout in place
    // and runs without its k split (whose partial sums would need a workspace), so nothing
    // is copied or allocated. It has no waits, so no status word to clear.
    DeviceState local;
    local.device = device;
    local.sm_count = sms;
    local.status = reinterpret_cast<DevStatus*>(scratch);
    return gemv_launch(d, nullptr, A, B, C, s, &local, /*allow_workspace=*/false);
  }

  lvb_gemm_plan plan;
  st = gemm_plan_c(d, sms,
                   (uintptr_t)C % 16 == 0 && (d->ldc * dtype_size(d->c_type)) % 16 == 0, &plan);
  if (st) return st;
  if (((uintptr_t)A) % 16) plan.repack_a = 1;
  if (((uintptr_t)B) % 16) plan.repack_b = 1;
  const long long kp = (d->K + 15) / 16 * 16;
  const size_t bytes_a = plan.repack_a ? (size_t)d->M * kp * es : 0;
  const size_t bytes_b = plan.repack_b ? (size_t)d->N * kp * es : 0;
  if (d->K > 0 && bytes_a + bytes_b > kNoAllocWorkspaceBytes) {
    // 8-bit operands stored MN-contiguous (A column-major, B row-major) are copied K-major
    // at any alignment, so alignment alone cannot avoid the workspace for them.
    const bool mn8 = es == 1 && ((plan.repack_a && !d->a_rowmajor) || (plan.repack_b && d->b_rowmajor));
    char buf[240];
    std::snprintf(buf, sizeof buf,
                  "operands to repack need %zu bytes, above the %zu-byte static workspace%s",
                  bytes_a + bytes_b, (size_t)kNoAllocWorkspaceBytes,
                  mn8 ? " (an 8-bit operand stored MN-contiguous is always copied K-major)" : "");
    return fail(LVB_ERR_UNSUPPORTED, op, buf,
                mn8 ? "store 8-bit A row-major and B column-major (K-contiguous), or use lvb_gemm"
                    : "pass 16-byte aligned operands with 16-byte multiple leading dimensions, or use lvb_gemm");
  }

  // The status word must start at zero for this call; the array keeps the last call's bytes.
  DevStatus* status = reinterpret_cast<DevStatus*>(scratch);
  e = cudaMemsetAsync(status, 0, sizeof(DevStatus), s);
  if (e != cudaSuccess) return fail_cuda(e, op, "clearing the status word");
  if (d->K == 0) return gemm_zero_fill(d, C, s);

  DeviceState local;  // no allocation: the status word is the scratch head
  local.device = device;
  local.sm_count = sms;
  local.status = status;
  lvb_gemm_desc d2 = *d;
  const void* a = A;
  const void* b = B;
  uint8_t* ws = reinterpret_cast<uint8_t*>(scratch) + kNoAllocHeadBytes;
  if (plan.repack_a) {
    st = repack(A, es, d->M, d->K, d->lda, !d->a_rowmajor, ws, kp, s);
    if (st) return st;
    a = ws;
    d2.lda = kp;
    d2.a_rowmajor = 1;
    plan.a_mnmajor = 0;
  }
  if (plan.repack_b) {
    st = repack(B, es, d->N, d->K, d->ldb, d->b_rowmajor != 0, ws + bytes_a, kp, s);
    if (st) return st;
    b = ws + bytes_a;
    d2.ldb = kp;
    d2.b_rowmajor = 0;
    plan.b_mnmajor = 0;
  }
  plan.repack_a = plan.repack_b = 0;
  return gemm_launch_aligned(&d2, plan, a, b, C, nullptr, s, &local);
}

extern "C" int lvb_gemm_noalloc_status(void* stream, int32_t* code, int32_t* where,
                                       int32_t* block) {
  using namespace lvb;
  const char* op = "lvb_gemm_noalloc_status";
  DevStatus* word = nullptr;
  int st = noalloc_status_word(&word, op);
  if (st) return st;
  cudaError_t e = cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail_cuda(e, op, "cudaStreamSynchronize");
  DevStatus h;
  e = cudaMemcpy(&h, word, sizeof h, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return fail_cuda(e, op, "reading the status word");
  if (h.code != 0) {
    e = cudaMemset(word, 0, sizeof(DevStatus));
    if (e != cudaSuccess) return fail_cuda(e, op, "clearing the status word");
  }
  if (code) *code = h.code;
  if (where) *where = h.where;
  if (block) *block = h.block;
  return LVB_OK;
}

namespace lvb {

// Epilogue fields of the kernel parameters from the caller's description (kernel space:
// with swap_ab the caller's rows are the kernel's n).
static void set_epilogue(GemmParams& p, const lvb_epilogue* e, bool swap_ab) {
  p.epi = 0;
  p.act = LVB_ACT_NONE;
  p.bias = p.res = p.mul = p.ext = nullptr;
  p.bias_kind = p.res_kind = p.mul_kind = p.ext_kind = LVB_F32;
  p.bias_on_m = 0;
  p.ldr = p.ldm = p.lde = 0;
  p.prog_swap = swap_ab ? 1 : 0;
  p.prog.n = 0;
  p.kx = 0;
  p.cu_mode = p.cv_mode = 0;
  p.cu_f = p.cv_f = 0.f;
  p.cu_i = p.cv_i = 0;
  p.cu_ptr = p.cv_ptr = nullptr;
  p.cu_ld = p.cv_ld = 0;
  p.cu_mn = p.cv_mn = 0;
  if (!e) return;
  p.act = e->activation;
  p.bias = e->bias;
  p.bias_kind = e->bias_type;
  p.bias_on_m = (e->bias_axis == LVB_BIAS_PER_ROW) != swap_ab;
  p.res = e->residual;
  p.res_kind = e->residual_type;
  p.ldr = e->ldr;
  p.mul = e->mul;
  p.mul_kind = e->mul_type;
  p.ldm = e->ldm;
  if (e->program && e->program->n > 0) {
    p.prog.n = e->program->n;
    std::memcpy(p.prog.code, e->program->code, sizeof p.prog.code);
    p.ext = e->extra;
    p.ext_kind = e->extra_type;
    p.lde = e->lde;
  }
  p.epi = (p.act != LVB_ACT_NONE || p.bias || p.res || p.mul || p.prog.n) ? 1 : 0;
}

// The clamp term of the padded k extent (kernel space: kernel A is the caller's B when the
// product runs as Cᵀ = BᵀAᵀ). `ka`/`kb` are the kernel operands as the kernel reads them.
static void set_clamp(GemmParams& p, const lvb_epilogue* e, const lvb_gemm_desc* d, bool swap_ab,
                      const void* ka, long long lda_k, int ka_mn, const void* kb, long long ldb_k,
                      int kb_mn) {
  if (!e || e->k_pad <= d->K) return;
  const int mode_a = swap_ab ? e->b_clamp : e->a_clamp;
  const int mode_b = swap_ab ? e->a_clamp : e->b_clamp;
  const double val_a = swap_ab ? e->b_clamp_value : e->a_clamp_value;
  const double val_b = swap_ab ? e->a_clamp_value : e->b_clamp_value;
  const bool integer = d->a_type == LVB_I8 || d->a_type == LVB_U8;
  // the clamp constant as the operand's type reads it (tensor_clampbits): RNE to 16 bits
  auto as_operand = [&](double v) -> float {
    if (d->a_type == LVB_F16) return __half2float(__float2half_rn((float)v));
    return __bfloat162float(__float2bfloat16_rn((float)v));
  };
  // a reader of zero (undefined or a zero constant) makes the whole term zero
  auto zero = [&](int mode, double v) {
    return mode == LVB_CLAMP_UNDEFINED || (mode == LVB_CLAMP_CONSTANT &&
                                           (integer ? (long long)v == 0 : as_operand(v) == 0.f));
  };
  if (zero(mode_a, val_a) || zero(mode_b, val_b)) return;
  p.kx = (int)(e->k_pad - d->K);
  p.cu_mode = mode_a == LVB_CLAMP_TO_EDGE ? 2 : 1;
  p.cv_mode = mode_b == LVB_CLAMP_TO_EDGE ? 2 : 1;
  if (integer) {
    p.cu_i = (int)val_a;
    p.cv_i = (int)val_b;
  } else {
    p.cu_f = as_operand(val_a);
    p.cv_f = as_operand(val_b);
  }
  p.cu_ptr = ka;
  p.cu_ld = lda_k;
  p.cu_mn = ka_mn;
  p.cv_ptr = kb;
  p.cv_ld = ldb_k;
  p.cv_mn = kb_mn;
  p.epi = 1;
}

int gemm_epilogue_only(const lvb_gemm_desc* d, const lvb_epilogue* e, void* C,
                       cudaStream_t stream) {
  GemmParams p = {};
  const bool swap = d->c_rowmajor != 0;
  p.M = (int)(swap ? d->N : d->M);
  p.N = (int)(swap ? d->M : d->N);
  p.D = C;
  p.ldd = d->ldc;
  p.K = 0;
  set_epilogue(p, e, swap);
  set_clamp(p, e, d, swap, nullptr, 0, 0, nullptr, 0, 0);   // K == 0: constants only
  const long long total = (long long)p.M * p.N;
  const int blocks = (int)std::min<long long>((total + 255) / 256, 4096);
  switch (out_kind_of(d->c_type)) {
    case OUT_F32: gemm_epilogue_only_kernel<OUT_F32><<<blocks, 256, 0, stream>>>(p); break;
    case OUT_F16: gemm_epilogue_only_kernel<OUT_F16><<<blocks, 256, 0, stream>>>(p); break;
    case OUT_BF16: gemm_epilogue_only_kernel<OUT_BF16><<<blocks, 256, 0, stream>>>(p); break;
    default: return fail(LVB_ERR_UNSUPPORTED, "lvb_gemm_ex", "epilogue on an integer output");
  }
  cudaError_t err = cudaGetLastError();
  return err == cudaSuccess ? LVB_OK : fail_cuda(err, "lvb_gemm_ex", "epilogue launch");
}

// The tensor maps of one call: operands K-major (rows of K elements, boxes of 128 K-bytes ×
// tile rows) or MN-major (rows of MN elements, one per k, boxes of 64 MN elements × 64 k);
// the CTA pair stages half of the 256-column B tile per CTA. Kernel-space D is n-contiguous
// when the plan oriented the product that way (C can take TMA stores): its interior boxes
// (32 m × 64 n of 16-bit or 32 m × 32 n of 32-bit elements: rows of 128 bytes) then go out
// through TMA tensor stores with the 128B row swizzle the epilogue writes.
static int encode_maps(const lvb_gemm_desc* d, const lvb_gemm_plan& plan, const void* kA,
                       const void* kB, int64_t kM, int64_t kN, int64_t ldka, int64_t ldkb,
                       int ka_mn, int kb_mn, void* C, int d_nmajor, CUtensorMap* ta,
                       CUtensorMap* tb, CUtensorMap* td, int* stage_out) {
  const int esize = dtype_size(d->a_type);
  const uint32_t box_k = 128 / esize;
  int st = ka_mn ? make_tmap_2d(ta, kA, esize, (uint64_t)kM, (uint64_t)d->K, (uint64_t)ldka, 64,
                                64, "lvb_gemm")
                 : make_tmap_2d(ta, kA, esize, (uint64_t)d->K, (uint64_t)kM, (uint64_t)ldka,
                                box_k, kBM, "lvb_gemm");
  if (st) return st;
  st = kb_mn ? make_tmap_2d(tb, kB, esize, (uint64_t)kN, (uint64_t)d->K, (uint64_t)ldkb, 64, 64,
                            "lvb_gemm")
             : make_tmap_2d(tb, kB, esize, (uint64_t)d->K, (uint64_t)kN, (uint64_t)ldkb, box_k,
                            plan.cta_pair ? (uint32_t)plan.tile_n / 2 : (uint32_t)plan.tile_n,
                            "lvb_gemm");
  if (st) return st;
  const int osize = dtype_size(d->c_type);
  std::memset(td, 0, sizeof *td);
  *stage_out = 0;
  if (d_nmajor) {
    if (make_tmap_2d_sw(td, C, osize, (uint64_t)kN, (uint64_t)kM, (uint64_t)d->ldc,
                        osize == 2 ? 64 : 32, 32, 128, "lvb_gemm") == LVB_OK)
      *stage_out = 1;
    else
      clear_error();   // direct stores in the same orientation: correct, slower
  }
  return LVB_OK;
}

// A few recent calls' tensor maps per host thread (no lock: thread-local), compared byte for
// byte on everything the maps are encoded from.
struct MapKey {
  int device;
  int swap, pair, tile_n, a_mn, b_mn;
  lvb_gemm_desc d;
  const void* A;
  const void* B;
  void* C;
};
struct MapVal {
  CUtensorMap ta, tb, td;
  int stage_out;
};
constexpr int kMapCacheSize = 8;
struct MapCache {
  MapKey key[kMapCacheSize];
  MapVal val[kMapCacheSize];
  int used = 0, next = 0;
};
static thread_local MapCache t_maps;

static const MapVal* map_cache_find(const MapKey& k) {
  for (int i = 0; i < t_maps.used; ++i)
    if (std::memcmp(&t_maps.key[i], &k, sizeof k) == 0) return &t_maps.val[i];
  return nullptr;
}

static void map_cache_insert(const MapKey& k, const CUtensorMap& ta, const CUtensorMap& tb,
                             const CUtensorMap& td, int stage_out) {
  const int i = t_maps.next;
  t_maps.key[i] = k;
  t_maps.val[i].ta = ta;
  t_maps.val[i].tb = tb;
  t_maps.val[i].td = td;
  t_maps.val[i].stage_out = stage_out;
  t_maps.next = (i + 1) % kMapCacheSize;
  if (t_maps.used < kMapCacheSize) ++t_maps.used;
}

int gemm_launch_aligned(const lvb_gemm_desc* d, const lvb_gemm_plan& plan, const void* A,
                        const void* B, void* C, const lvb_epilogue* epi, cudaStream_t stream,
                        DeviceState* dev) {
  const int esize = dtype_size(d->a_type);
  // Kernel space: rows of "A" are the lane (contiguous-store) dimension.
  const void* kA = plan.swap_ab ? B : A;
  const void* kB = plan.swap_ab ? A : B;
  const int64_t kM = plan.swap_ab ? d->N : d->M;
  const int64_t kN = plan.swap_ab ? d->M : d->N;
  const int64_t ldka = plan.swap_ab ? d->ldb : d->lda;
  const int64_t ldkb = plan.swap_ab ? d->lda : d->ldb;
  // Operands the tensor core reads MN-major (16-bit only; the planner repacks 8-bit ones).
  const int ka_mn = plan.swap_ab ? plan.b_mnmajor : plan.a_mnmajor;
  const int kb_mn = plan.swap_ab ? plan.a_mnmajor : plan.b_mnmajor;
  const uint32_t box_k = 128 / esize;

  const int d_nmajor = (plan.swap_ab != 0) != (d->c_rowmajor != 0);
  CUtensorMap ta, tb, td;
  int stage_out = 0;
  // The three tensor maps depend only on the descriptor, the plan's orientation and tiles and
  // the three pointers: a call repeating a recent one on this thread reuses them (encoding
  // them is most of the host time of a small GEMM).
  MapKey key;
  std::memset(&key, 0, sizeof key);
  key.device = dev->device;
  key.d = *d;
  key.A = A;
  key.B = B;
  key.C = C;
  key.swap = plan.swap_ab;
  key.pair = plan.cta_pair;
  key.tile_n = plan.tile_n;
  key.a_mn = ka_mn;
  key.b_mn = kb_mn;
  if (const MapVal* hit = map_cache_find(key)) {
    ta = hit->ta;
    tb = hit->tb;
    td = hit->td;
    stage_out = hit->stage_out;
  } else {
    const int st = encode_maps(d, plan, kA, kB, kM, kN, ldka, ldkb, ka_mn, kb_mn, C, d_nmajor,
                               &ta, &tb, &td, &stage_out);
    if (st) return st;
    map_cache_insert(key, ta, tb, td, stage_out);
  }

  GemmParams p;
  p.a_mn = ka_mn;
  p.b_mn = kb_mn;
  p.d_nmajor = d_nmajor;
  p.stage_out = stage_out;
  set_epilogue(p, epi, plan.swap_ab != 0);
  set_clamp(p, epi, d, plan.swap_ab != 0, kA, ldka, ka_mn, kB, ldkb, kb_mn);
  p.M = (int)kM;
  p.N = (int)kN;
  p.K = (int)d->K;
  p.tiles_m = (int)((kM + plan.tile_m - 1) / plan.tile_m);
  p.tiles_n = (int)((kN + plan.tile_n - 1) / plan.tile_n);
  p.num_kb = (int)((d->K + box_k - 1) / box_k);
  p.total_tiles = p.tiles_m * p.tiles_n;
  // Raster group (row-tiles per group) and L2 policy; LVB_GEMM_GROUP / LVB_GEMM_L2 override
  // them for tuning.
  static const int env_group = [] {
    const char* s = std::getenv("LVB_GEMM_GROUP");
    return s ? std::atoi(s) : 0;
  }();
  static const int env_l2 = [] {
    const char* s = std::getenv("LVB_GEMM_L2");
    return s ? std::atoi(s) : -1;
  }();
  p.group_m = env_group > 0 ? env_group : (plan.cta_pair ? 8 : 16);
  p.l2_mode = (env_l2 >= 0 && env_l2 <= 2) ? env_l2 : 0;
  p.D = C;
  p.ldd = d->ldc;
  p.status = dev->status;
  p.timeout_ns = wait_timeout_ns();

  const int ab = ab_kind_of(d->a_type);
  const int out = out_kind_of(d->c_type);
  // 1024: the tall CTA-pair kernel (512 × 256 tiles); 512 / 448: the CTA-pair kernel with
  // 256 × 256 / 256 × 224 tiles
  const int bn = plan.cta_pair ? (plan.tile_m == 512 ? 1024 : 2 * plan.tile_n) : plan.tile_n;
  const int ctas = plan.ctas;
  if (ab == AB_F16) {
    if (out == OUT_F32) return launch_bn<AB_F16, OUT_F32>(bn, ta, tb, td, p, ctas, stream, dev);
    if (out == OUT_F16) return launch_bn<AB_F16, OUT_F16>(bn, ta, tb, td, p, ctas, stream, dev);
    if (out == OUT_BF16) return launch_bn<AB_F16, OUT_BF16>(bn, ta, tb, td, p, ctas, stream, dev);
  } else if (ab == AB_BF16) {
    if (out == OUT_F32) return launch_bn<AB_BF16, OUT_F32>(bn, ta, tb, td, p, ctas, stream, dev);
    if (out == OUT_F16) return launch_bn<AB_BF16, OUT_F16>(bn, ta, tb, td, p, ctas, stream, dev);
    if (out == OUT_BF16) return launch_bn<AB_BF16, OUT_BF16>(bn, ta, tb, td, p, ctas, stream, dev);
  } else if (ab == AB_S8 && out == OUT_I32) {
    return launch_bn<AB_S8, OUT_I32>(bn, ta, tb, td, p, ctas, stream, dev);
  } else if (ab == AB_U8 && out == OUT_I32) {
    return launch_bn<AB_U8, OUT_I32>(bn, ta, tb, td, p, ctas, stream, dev);
  }
  return fail(LVB_ERR_UNSUPPORTED, "lvb_gemm", "dtype combination not built");
}

}  // namespace lvb
