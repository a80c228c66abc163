// lvb_internal.h — host-side plumbing shared by the translation units of liblvb.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "lvb.h"   // include/ is on the compiler's include path (build.py)
#include "sm100.cuh"

namespace lvb {

// Thread-local error message; returns `status` so call sites can `return fail(...)`.
int fail(int status, const std::string& op, const std::string& msg, const std::string& hint = "");
int fail_cuda(cudaError_t e, const std::string& op, const char* what);
void clear_error();

// Per-device state, created on first use with the device current.
struct DeviceState {
  int device = -1;
  int sm_count = 0;
  int cc_major = 0, cc_minor = 0;
  size_t smem_optin = 0;
  DevStatus* status = nullptr;   // device status word (cudaMalloc'd once per device)
  cudaMemPool_t pool = nullptr;  // stream-ordered pool for workspaces (keeps freed memory)
};
// Returns nullptr (and sets the error) when the current device is unusable.
DeviceState* current_device_state(const char* op);

uint64_t wait_timeout_ns();

// Stream-ordered workspace from the device's pool; release it with cudaFreeAsync on the
// same stream.
cudaError_t workspace_alloc(DeviceState* dev, void** ptr, size_t bytes, cudaStream_t stream);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled_fn();

// 2-D map over a K-contiguous (or generally inner-contiguous) matrix of `rows` rows of
// `inner` elements, leading dimension `ld` elements, elements of `esize` bytes, box
// `box_inner` × `box_rows`, 128-byte swizzle. Returns 0 or an lvb_status.
int make_tmap_2d(CUtensorMap* tm, const void* base, int esize, uint64_t inner, uint64_t rows,
                 uint64_t ld, uint32_t box_inner, uint32_t box_rows, const char* op);

// The same with a chosen swizzle (0, 32, 64 or 128 bytes; 0 = boxes stored row-major in
// shared memory), for TMA stores.
int make_tmap_2d_sw(CUtensorMap* tm, const void* base, int esize, uint64_t inner, uint64_t rows,
                    uint64_t ld, uint32_t box_inner, uint32_t box_rows, int swizzle_bytes,
                    const char* op);

// Rank-n tiled map (n <= 5), 128-byte swizzle. dims/box innermost first; strides[i] is the
// element stride of dimension i+1.
int make_tmap_nd(CUtensorMap* tm, const void* base, int esize, int rank, const uint64_t* dims,
                 const uint64_t* strides, const uint32_t* box, const char* op);

// 3-D map [outer][rows][inner] with element strides (ld_rows, ld_outer).
int make_tmap_3d(CUtensorMap* tm, const void* base, int esize, uint64_t inner, uint64_t rows,
                 uint64_t outer, uint64_t ld_rows, uint64_t ld_outer, uint32_t box_inner,
                 uint32_t box_rows, const char* op);

int dtype_size(int dt);
const char* dtype_name(int dt);

// ---- GEMM (gemm_sm100.cu) ----
// lvb_gemm_plan_for with C's TMA-store capability known (its base and leading dimension):
// it decides the orientation of the product in kernel space.
// allow_gemv = false plans the tensor-core kernel even for a matrix-vector shape (epilogues
// the streaming kernel does not carry).
int gemm_plan_c(const lvb_gemm_desc* d, int32_t sm_count, bool c_tma_ok, lvb_gemm_plan* out,
                bool allow_gemv = true);

// `epi` is NULL for a plain GEMM.
int gemm_launch(const lvb_gemm_desc* d, const lvb_gemm_plan& plan, const void* A,
                const void* B, void* C, const lvb_epilogue* epi, cudaStream_t stream,
                DeviceState* dev);
// K == 0 with an epilogue: C = act(bias + R).
int gemm_epilogue_only(const lvb_gemm_desc* d, const lvb_epilogue* e, void* C,
                       cudaStream_t stream);

// The status word at the head of lvb_gemm_noalloc's static scratch array, on the current
// device (looked up without allocating).
int noalloc_status_word(DevStatus** out, const char* op);
// Enqueue the bounded-wait self-test kernel against `status` (see selftest.cu).
int selftest_launch(DevStatus* status, int32_t timeout_ms, cudaStream_t stream, const char* op);

// ---- matrix-vector products (gemv_sm100.cu): lvb_gemm with N == 1 or M == 1 ----
struct GemvPlan {
  int32_t k_contiguous;     // the matrix runs along k (one warp per row) or along rows
  int32_t ksplit;           // k split across CTAs (partial sums in a workspace) when > 1
  int64_t kchunk;           // elements of k per split
  int32_t ctas;             // CTAs along the rows
  int64_t workspace_bytes;  // ksplit·rows·4 when ksplit > 1
};
bool gemv_applies(const lvb_gemm_desc* d);
int gemv_plan(const lvb_gemm_desc* d, int sm_count, GemvPlan* out);
// allow_workspace = false: never split k (no partial-sum workspace is allocated).
int gemv_launch(const lvb_gemm_desc* d, const lvb_epilogue* e, const void* A, const void* B,
                void* C, cudaStream_t stream, DeviceState* dev, bool allow_workspace = true);

// ---- attention (attn_sm100.cu) ----
int attn_launch(const lvb_attn_desc* d, const void* Q, const void* K, const void* V, void* O,
                float* lse, cudaStream_t stream, DeviceState* dev);
// Few query rows per KV head (group·seq_q <= 32, head_dim 128): the HBM-bound decoding kernel
// (attn_decode_sm100.cu), split over the key range.
bool attn_decode_applies(const lvb_attn_desc* d);
void attn_decode_plan(const lvb_attn_desc* d, int sm_count, int* nsplit, int* bps, int* ctas);
int attn_decode_launch(const lvb_attn_desc* d, const long long qs[3], const long long ks[3],
                       const long long vs[3], const long long os[3], const void* Q, const void* K,
                       const void* V, void* O, float* lse, cudaStream_t stream, DeviceState* dev);

}  // namespace lvb
