// abi.cu — the extern "C" surface of liblvb: argument validation, planning, capability
// answers, per-device state, tensor-map construction and the runtime helpers. Kernels live
// in gemm_sm100.cu and attn_sm100.cu.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>

#include "lvb_internal.h"

namespace lvb {

// ---------------------------------------------------------------------------------------
// Errors
// ---------------------------------------------------------------------------------------
static thread_local std::string g_last_error;

int fail(int status, const std::string& op, const std::string& msg, const std::string& hint) {
  g_last_error = op + ": " + msg;
  if (!hint.empty()) g_last_error += " (" + hint + ")";
  return status;
}
int fail_cuda(cudaError_t e, const std::string& op, const char* what) {
  return fail(LVB_ERR_CUDA, op, std::string(what) + " failed: " + cudaGetErrorString(e),
              "check the device and the pointers passed");
}
void clear_error() { g_last_error.clear(); }

int dtype_size(int dt) {
  switch (dt) {
    case LVB_F16:
    case LVB_BF16: return 2;
    case LVB_F32:
    case LVB_I32:
    case LVB_U32: return 4;
    case LVB_I8:
    case LVB_U8: return 1;
  }
  return 0;
}
const char* dtype_name(int dt) {
  switch (dt) {
    case LVB_F16: return "Float16";
    case LVB_BF16: return "BFloat16";
    case LVB_F32: return "Float32";
    case LVB_I8: return "Int8";
    case LVB_U8: return "UInt8";
    case LVB_I32: return "Int32";
    case LVB_U32: return "UInt32";
  }
  return "unknown";
}

// ---------------------------------------------------------------------------------------
// Wait limit
// ---------------------------------------------------------------------------------------
static std::mutex g_timeout_mu;
static int64_t g_timeout_ms = -1;

uint64_t wait_timeout_ns() {
  std::lock_guard<std::mutex> lk(g_timeout_mu);
  if (g_timeout_ms < 0) {
    g_timeout_ms = 2000;
    if (const char* s = std::getenv("LVB_WAIT_TIMEOUT_MS")) {
      long long v = std::atoll(s);
      if (v > 0) g_timeout_ms = v;
    }
  }
  return (uint64_t)g_timeout_ms * 1000000ull;
}

// ---------------------------------------------------------------------------------------
// Per-device state
// ---------------------------------------------------------------------------------------
static std::mutex g_dev_mu;
static std::map<int, DeviceState*> g_devices;

DeviceState* current_device_state(const char* op) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    fail(LVB_ERR_NO_DEVICE, op, std::string("no CUDA device: ") + cudaGetErrorString(e),
         "run on a machine with a B200");
    return nullptr;
  }
  // Device states live for the process: a thread remembers the last one it looked up.
  static thread_local int tl_dev = -1;
  static thread_local DeviceState* tl_state = nullptr;
  if (dev == tl_dev && tl_state) return tl_state;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  auto it = g_devices.find(dev);
  if (it != g_devices.end()) {
    tl_dev = dev;
    tl_state = it->second;
    return it->second;
  }
  DeviceState* st = new DeviceState();
  st->device = dev;
  cudaDeviceGetAttribute(&st->sm_count, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&st->cc_major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&st->cc_minor, cudaDevAttrComputeCapabilityMinor, dev);
  int optin = 0;
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  st->smem_optin = (size_t)optin;
  if (st->cc_major != 10 || st->cc_minor != 0) {
    char buf[128];
    std::snprintf(buf, sizeof buf, "device %d is sm_%d%d, this library is built for sm_100a", dev,
                  st->cc_major, st->cc_minor);
    delete st;
    fail(LVB_ERR_NO_DEVICE, op, buf, "run on a B200");
    return nullptr;
  }
  e = cudaMalloc(&st->status, sizeof(DevStatus));
  if (e == cudaSuccess) e = cudaMemset(st->status, 0, sizeof(DevStatus));
  if (e != cudaSuccess) {
    delete st;
    fail_cuda(e, op, "allocating the device status word");
    return nullptr;
  }
  // The library's own stream-ordered pool for workspaces. It keeps up to 512 MiB of freed
  // workspace instead of handing it back at every synchronisation (the default pool's
  // behaviour), so a workspace of the same size on the next call costs no mapping; the
  // process's default pool is left as it is.
  cudaMemPoolProps props = {};
  props.allocType = cudaMemAllocationTypePinned;
  props.location.type = cudaMemLocationTypeDevice;
  props.location.id = dev;
  if (cudaMemPoolCreate(&st->pool, &props) == cudaSuccess) {
    uint64_t keep = 512ull << 20;
    cudaMemPoolSetAttribute(st->pool, cudaMemPoolAttrReleaseThreshold, &keep);
  } else {
    cudaGetLastError();
    st->pool = nullptr;   // workspaces then come from the default pool
  }
  g_devices[dev] = st;
  return st;
}

cudaError_t workspace_alloc(DeviceState* dev, void** ptr, size_t bytes, cudaStream_t stream) {
  if (dev && dev->pool) return cudaMallocFromPoolAsync(ptr, bytes, dev->pool, stream);
  return cudaMallocAsync(ptr, bytes, stream);
}

// ---------------------------------------------------------------------------------------
// Tensor maps
// ---------------------------------------------------------------------------------------
EncodeTiledFn encode_tiled_fn() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

static CUtensorMapDataType tma_type(int esize) {
  return esize == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                    : (esize == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT32);
}

int make_tmap_2d(CUtensorMap* tm, const void* base, int esize, uint64_t inner, uint64_t rows,
                 uint64_t ld, uint32_t box_inner, uint32_t box_rows, const char* op) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return fail(LVB_ERR_CUDA, op, "cuTensorMapEncodeTiled unavailable", "driver too old");
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {ld * (uint64_t)esize};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(tm, tma_type(esize), 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[160];
    std::snprintf(buf, sizeof buf, "cuTensorMapEncodeTiled failed (%d) for %llu x %llu, ld %llu",
                  (int)r, (unsigned long long)rows, (unsigned long long)inner,
                  (unsigned long long)ld);
    return fail(LVB_ERR_UNSUPPORTED, op, buf, "pointers must be 16-byte aligned, ld*size a multiple of 16");
  }
  return LVB_OK;
}

int make_tmap_2d_sw(CUtensorMap* tm, const void* base, int esize, uint64_t inner, uint64_t rows,
                    uint64_t ld, uint32_t box_inner, uint32_t box_rows, int swizzle_bytes,
                    const char* op) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return fail(LVB_ERR_CUDA, op, "cuTensorMapEncodeTiled unavailable", "driver too old");
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {ld * (uint64_t)esize};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle sw = swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                : swizzle_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                                      : CU_TENSOR_MAP_SWIZZLE_NONE;
  CUresult r = enc(tm, tma_type(esize), 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(LVB_ERR_UNSUPPORTED, op, "cuTensorMapEncodeTiled failed for a store map");
  return LVB_OK;
}

int make_tmap_3d(CUtensorMap* tm, const void* base, int esize, uint64_t inner, uint64_t rows,
                 uint64_t outer, uint64_t ld_rows, uint64_t ld_outer, uint32_t box_inner,
                 uint32_t box_rows, const char* op) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return fail(LVB_ERR_CUDA, op, "cuTensorMapEncodeTiled unavailable", "driver too old");
  cuuint64_t dims[3] = {inner, rows, outer};
  cuuint64_t strides[2] = {ld_rows * (uint64_t)esize, ld_outer * (uint64_t)esize};
  cuuint32_t box[3] = {box_inner, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(tm, tma_type(esize), 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[160];
    std::snprintf(buf, sizeof buf, "cuTensorMapEncodeTiled(3d) failed (%d)", (int)r);
    return fail(LVB_ERR_UNSUPPORTED, op, buf, "pointers must be 16-byte aligned, strides*size multiples of 16");
  }
  return LVB_OK;
}

int make_tmap_nd(CUtensorMap* tm, const void* base, int esize, int rank, const uint64_t* dims,
                 const uint64_t* strides, const uint32_t* box, const char* op) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return fail(LVB_ERR_CUDA, op, "cuTensorMapEncodeTiled unavailable", "driver too old");
  if (rank < 1 || rank > 5) return fail(LVB_ERR_INVALID_ARG, op, "tensor map rank");
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i + 1 < rank) s[i] = strides[i] * (uint64_t)esize;
  }
  CUresult r = enc(tm, tma_type(esize), rank, const_cast<void*>(base), d, s, b, e,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[160];
    std::snprintf(buf, sizeof buf, "cuTensorMapEncodeTiled(rank %d) failed (%d)", rank, (int)r);
    return fail(LVB_ERR_UNSUPPORTED, op, buf,
                "pointers must be 16-byte aligned, strides*size multiples of 16");
  }
  return LVB_OK;
}

int gemm_smem_bytes(int bn);
int gemm_stages(int bn);
int gemm_zero_fill(const lvb_gemm_desc* d, void* C, cudaStream_t stream);

}  // namespace lvb

using namespace lvb;

// =========================================================================================
// extern "C"
// =========================================================================================
extern "C" {

int lvb_abi_version(void) { return LVB_ABI_VERSION; }

const char* lvb_last_error(void) { return g_last_error.c_str(); }

const char* lvb_status_string(int s) {
  switch (s) {
    case LVB_OK: return "LVB_OK";
    case LVB_ERR_INVALID_ARG: return "LVB_ERR_INVALID_ARG";
    case LVB_ERR_UNSUPPORTED: return "LVB_ERR_UNSUPPORTED";
    case LVB_ERR_CUDA: return "LVB_ERR_CUDA";
    case LVB_ERR_TIMEOUT: return "LVB_ERR_TIMEOUT";
    case LVB_ERR_NCCL: return "LVB_ERR_NCCL";
    case LVB_ERR_NO_DEVICE: return "LVB_ERR_NO_DEVICE";
  }
  return "LVB_ERR_UNKNOWN";
}

// ---------------------------------------------------------------------------------------
// Capabilities
// ---------------------------------------------------------------------------------------
// Subgroup-scope shapes a warp can issue on sm_100 (mma.sync class), and the
// workgroup-scope shapes the fused tcgen05 kernels tile with (one CTA, TMEM accumulator).
static const lvb_matrix_shape kShapes[] = {
    {LVB_F16, LVB_F32, 16, 16, 16, LVB_SUBGROUP_SCOPE},
    {LVB_F16, LVB_F32, 16, 8, 16, LVB_SUBGROUP_SCOPE},
    {LVB_F16, LVB_F16, 16, 16, 16, LVB_SUBGROUP_SCOPE},
    {LVB_F16, LVB_F16, 16, 8, 16, LVB_SUBGROUP_SCOPE},
    {LVB_BF16, LVB_F32, 16, 16, 16, LVB_SUBGROUP_SCOPE},
    {LVB_BF16, LVB_F32, 16, 8, 16, LVB_SUBGROUP_SCOPE},
    {LVB_I8, LVB_I32, 16, 16, 32, LVB_SUBGROUP_SCOPE},
    {LVB_I8, LVB_I32, 16, 8, 32, LVB_SUBGROUP_SCOPE},
    {LVB_U8, LVB_U32, 16, 16, 32, LVB_SUBGROUP_SCOPE},
    {LVB_U8, LVB_U32, 16, 8, 32, LVB_SUBGROUP_SCOPE},
    {LVB_F16, LVB_F32, 128, 256, 16, LVB_WORKGROUP_SCOPE},
    {LVB_F16, LVB_F32, 128, 128, 16, LVB_WORKGROUP_SCOPE},
    {LVB_F16, LVB_F32, 128, 64, 16, LVB_WORKGROUP_SCOPE},
    {LVB_BF16, LVB_F32, 128, 256, 16, LVB_WORKGROUP_SCOPE},
    {LVB_BF16, LVB_F32, 128, 128, 16, LVB_WORKGROUP_SCOPE},
    {LVB_BF16, LVB_F32, 128, 64, 16, LVB_WORKGROUP_SCOPE},
    {LVB_I8, LVB_I32, 128, 256, 32, LVB_WORKGROUP_SCOPE},
    {LVB_I8, LVB_I32, 128, 128, 32, LVB_WORKGROUP_SCOPE},
    {LVB_I8, LVB_I32, 128, 64, 32, LVB_WORKGROUP_SCOPE},
    {LVB_U8, LVB_U32, 128, 256, 32, LVB_WORKGROUP_SCOPE},
    {LVB_U8, LVB_U32, 128, 128, 32, LVB_WORKGROUP_SCOPE},
    {LVB_U8, LVB_U32, 128, 64, 32, LVB_WORKGROUP_SCOPE},
};
static const int kNumShapes = sizeof(kShapes) / sizeof(kShapes[0]);

int lvb_caps_sm100(lvb_device_caps* out) {
  if (!out) return fail(LVB_ERR_INVALID_ARG, "lvb_caps_sm100", "out is NULL");
  std::memset(out, 0, sizeof *out);
  out->coopmat = 1;
  out->tile = 16;
  out->subgroup = 32;
  out->coopmatsubgroup = 32;
  out->sharedbudget = 232448;  // 227 KiB opt-in per CTA
  out->workgrouplimit = 1024;
  out->cores = 148;
  out->warps = 64;
  // (invocations, M, N, K) — a workgroup-scope fp16 matrix is a CTA tile held in TMEM:
  // 128 lanes (one warpgroup reads them), N in steps of 16, K in steps of 16.
  const int rows[][4] = {{128, 128, 16, 16}, {256, 128, 16, 16}};
  out->n_wggran = 2;
  for (int i = 0; i < 2; ++i)
    for (int j = 0; j < 4; ++j) out->wggran[i][j] = rows[i][j];
  int n_sub = 0;
  for (int i = 0; i < kNumShapes; ++i) n_sub += kShapes[i].scope == LVB_SUBGROUP_SCOPE;
  out->n_shapes = n_sub;
  out->cc_major = 10;
  out->cc_minor = 0;
  return LVB_OK;
}

int lvb_caps(int device, lvb_device_caps* out) {
  if (!out) return fail(LVB_ERR_INVALID_ARG, "lvb_caps", "out is NULL");
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n)
    return fail(LVB_ERR_NO_DEVICE, "lvb_caps", "device not present", "check CUDA_VISIBLE_DEVICES");
  int major = 0, minor = 0, sms = 0, smem = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
  if (major != 10 || minor != 0)
    return fail(LVB_ERR_NO_DEVICE, "lvb_caps", "device is not sm_100", "run on a B200");
  lvb_caps_sm100(out);
  out->cores = sms;
  out->sharedbudget = smem;
  return LVB_OK;
}

int lvb_matrix_shapes(lvb_matrix_shape* out, int32_t capacity, int32_t* count) {
  if (!count) return fail(LVB_ERR_INVALID_ARG, "lvb_matrix_shapes", "count is NULL");
  if (capacity > 0 && !out) return fail(LVB_ERR_INVALID_ARG, "lvb_matrix_shapes", "out is NULL");
  *count = kNumShapes;
  for (int i = 0; i < kNumShapes && i < capacity; ++i) out[i] = kShapes[i];
  return LVB_OK;
}

int lvb_bestshape(int32_t ab, int32_t acc, int32_t scope, lvb_matrix_shape* out) {
  if (!out) return fail(LVB_ERR_INVALID_ARG, "lvb_bestshape", "out is NULL");
  const lvb_matrix_shape* best = nullptr;
  for (int i = 0; i < kNumShapes; ++i) {
    const lvb_matrix_shape& s = kShapes[i];
    if (s.ab != ab || s.acc != acc || s.scope != scope) continue;
    if (!best) { best = &s; continue; }
    // squarest, then largest (Lava's isbetter, src/vocabulary/matrix.jl:165-172)
    long sa = std::labs((long)s.M - s.N) + std::labs((long)s.N - s.K);
    long sb = std::labs((long)best->M - best->N) + std::labs((long)best->N - best->K);
    if (sa != sb) { if (sa < sb) best = &s; continue; }
    if ((long)s.M * s.N * s.K > (long)best->M * best->N * best->K) best = &s;
  }
  if (!best)
    return fail(LVB_ERR_UNSUPPORTED, "lvb_bestshape", "no shape for this type pair and scope");
  *out = *best;
  return LVB_OK;
}

// ---------------------------------------------------------------------------------------
// GEMM
// ---------------------------------------------------------------------------------------
static bool gemm_types_ok(int a, int b, int c) {
  if (a != b) return false;
  if (a == LVB_F16 || a == LVB_BF16) return c == LVB_F32 || c == LVB_F16 || c == LVB_BF16;
  if (a == LVB_I8) return c == LVB_I32;
  if (a == LVB_U8) return c == LVB_U32;
  return false;
}

int lvb_gemm_check(const lvb_gemm_desc* d) {
  const char* op = "lvb_gemm";
  if (!d) return fail(LVB_ERR_INVALID_ARG, op, "descriptor is NULL");
  if (d->M < 0 || d->N < 0 || d->K < 0)
    return fail(LVB_ERR_INVALID_ARG, op, "negative extent", "M, N, K must be >= 0");
  if (d->M > INT32_MAX || d->N > INT32_MAX || d->K > INT32_MAX)
    return fail(LVB_ERR_UNSUPPORTED, op, "extent above 2^31-1", "split the problem");
  if (!gemm_types_ok(d->a_type, d->b_type, d->c_type)) {
    std::string m = std::string("no kernel for ") + dtype_name(d->a_type) + " x " +
                    dtype_name(d->b_type) + " -> " + dtype_name(d->c_type);
    return fail(LVB_ERR_UNSUPPORTED, op, m,
                "supported: Float16/BFloat16 -> Float32/Float16/BFloat16, Int8 -> Int32, UInt8 -> UInt32");
  }
  // An empty operand (K == 0) has no layout to check: C is the empty sum.
  if (d->K > 0) {
    // Row-major: `stride` elements between rows; column-major: between columns
    // (src/device/coopmat_intrinsics.jl:57-75).
    if (d->a_rowmajor ? d->lda < d->K : d->lda < std::max<int64_t>(1, d->M))
      return fail(LVB_ERR_INVALID_ARG, op, d->a_rowmajor ? "lda < K" : "lda < M");
    if (d->b_rowmajor ? d->ldb < std::max<int64_t>(1, d->N) : d->ldb < d->K)
      return fail(LVB_ERR_INVALID_ARG, op, d->b_rowmajor ? "ldb < N" : "ldb < K");
  }
  const int64_t cmin = std::max<int64_t>(1, d->c_rowmajor ? d->N : d->M);
  if (d->ldc < cmin) return fail(LVB_ERR_INVALID_ARG, op, d->c_rowmajor ? "ldc < N" : "ldc < M");
  return LVB_OK;
}

static bool float_type(int t) { return t == LVB_F32 || t == LVB_F16 || t == LVB_BF16; }

// An M×N epilogue matrix in C's layout (residual, S, the program's extra operand).
static int check_cmatrix(const char* op, const lvb_gemm_desc* d, const void* ptr, int type,
                         int64_t ld, const char* what, const char* ld_name) {
  if (!float_type(type)) {
    return fail(LVB_ERR_UNSUPPORTED, op,
                std::string(what) + " type must be Float32, Float16 or BFloat16");
  }
  const int64_t rmin = std::max<int64_t>(1, d->c_rowmajor ? d->N : d->M);
  if (ld < rmin)
    return fail(LVB_ERR_INVALID_ARG, op, std::string(ld_name) + (d->c_rowmajor ? " < N" : " < M"));
  if ((uintptr_t)ptr % dtype_size(type))
    return fail(LVB_ERR_INVALID_ARG, op, std::string(what) + " not aligned to its element size");
  return LVB_OK;
}

int lvb_pe_program_check(const lvb_pe_program* prog) {
  const char* op = "lvb_pe_program";
  if (!prog) return fail(LVB_ERR_INVALID_ARG, op, "program is NULL");
  if (prog->n < 0 || prog->n > LVB_PE_MAX_INSTR)
    return fail(LVB_ERR_INVALID_ARG, op, "instruction count outside 0..32");
  for (int i = 0; i < prog->n; ++i) {
    const lvb_pe_instr& I = prog->code[i];
    char buf[96];
    if (I.op >= LVB_PE_NUM_OPS) {
      std::snprintf(buf, sizeof buf, "instruction %d: unknown opcode %d", i, (int)I.op);
      return fail(LVB_ERR_INVALID_ARG, op, buf);
    }
    if (I.dst >= LVB_PE_REGS || I.a >= LVB_PE_REGS || I.b >= LVB_PE_REGS) {
      std::snprintf(buf, sizeof buf, "instruction %d: register above r7", i);
      return fail(LVB_ERR_INVALID_ARG, op, buf);
    }
  }
  return LVB_OK;
}

int lvb_gemm_ex_check(const lvb_gemm_desc* d, const lvb_epilogue* e) {
  const char* op = "lvb_gemm_ex";
  int st = lvb_gemm_check(d);
  if (st || !e) return st;
  const bool prog = e->program && e->program->n > 0;
  const bool any = e->bias || e->residual || e->activation != LVB_ACT_NONE || e->mul || prog;
  if (e->activation < LVB_ACT_NONE || e->activation > LVB_ACT_SILU)
    return fail(LVB_ERR_INVALID_ARG, op, "unknown activation");
  if (any && !float_type(d->c_type))
    return fail(LVB_ERR_UNSUPPORTED, op, "epilogue on an integer output",
                "coopmat_add, coopmat_mul, the activations and per-element programs are "
                "floating-point; only the clamp modes apply to integer pairs");
  if (e->bias) {
    if (!float_type(e->bias_type))
      return fail(LVB_ERR_UNSUPPORTED, op, "bias type must be Float32, Float16 or BFloat16");
    if (e->bias_axis != LVB_BIAS_PER_ROW && e->bias_axis != LVB_BIAS_PER_COL)
      return fail(LVB_ERR_INVALID_ARG, op, "bias_axis must be per-row (0) or per-column (1)");
    if ((uintptr_t)e->bias % dtype_size(e->bias_type))
      return fail(LVB_ERR_INVALID_ARG, op, "bias not aligned to its element size");
  }
  if (e->residual && (st = check_cmatrix(op, d, e->residual, e->residual_type, e->ldr, "residual", "ldr")))
    return st;
  if (e->mul && (st = check_cmatrix(op, d, e->mul, e->mul_type, e->ldm, "mul (coopmat_mul operand)", "ldm")))
    return st;
  if (e->program && (st = lvb_pe_program_check(e->program))) return st;
  if (e->extra) {
    if (!prog)
      return fail(LVB_ERR_INVALID_ARG, op, "extra matrix without a per-element program");
    if ((st = check_cmatrix(op, d, e->extra, e->extra_type, e->lde, "extra (program operand)", "lde")))
      return st;
  }
  if (e->k_pad != 0 && e->k_pad != d->K) {
    if (e->k_pad < d->K)
      return fail(LVB_ERR_INVALID_ARG, op, "k_pad < K", "k_pad is the padded k extent, >= K (0: none)");
    if (e->k_pad > INT32_MAX) return fail(LVB_ERR_UNSUPPORTED, op, "k_pad above 2^31-1");
    const bool integer = d->a_type == LVB_I8 || d->a_type == LVB_U8;
    const int modes[2] = {e->a_clamp, e->b_clamp};
    const double vals[2] = {e->a_clamp_value, e->b_clamp_value};
    for (int i = 0; i < 2; ++i) {
      const char* who = i ? "b_clamp" : "a_clamp";
      if (modes[i] < LVB_CLAMP_UNDEFINED || modes[i] > LVB_CLAMP_TO_EDGE)
        return fail(LVB_ERR_INVALID_ARG, op, std::string(who) + ": unknown clamp mode");
      if (modes[i] == LVB_CLAMP_TO_EDGE && d->K == 0)
        return fail(LVB_ERR_INVALID_ARG, op, std::string(who) + ": TO_EDGE with K == 0",
                    "an empty operand has no edge element");
      if (modes[i] == LVB_CLAMP_CONSTANT && integer) {
        const double lo = d->a_type == LVB_I8 ? -128 : 0, hi = d->a_type == LVB_I8 ? 127 : 255;
        if (vals[i] != (double)(long long)vals[i] || vals[i] < lo || vals[i] > hi)
          return fail(LVB_ERR_INVALID_ARG, op,
                      std::string(who) + ": the clamp value of an 8-bit operand is an integer in its range");
      }
    }
    if (d->K == 0 && !float_type(d->c_type))
      return fail(LVB_ERR_UNSUPPORTED, op, "k_pad with K == 0 on an integer output");
  }
  return LVB_OK;
}

int lvb_gemm_plan_for(const lvb_gemm_desc* d, int32_t sm_count, lvb_gemm_plan* out) {
  const bool c_tma_ok = d && (d->ldc * dtype_size(d->c_type)) % 16 == 0;
  return gemm_plan_c(d, sm_count, c_tma_ok, out);
}

}  // extern "C"
namespace lvb {
// c_tma_ok: C's base (when known) and leading dimension allow TMA stores.
int gemm_plan_c(const lvb_gemm_desc* d, int32_t sm_count, bool c_tma_ok, lvb_gemm_plan* out,
                bool allow_gemv) {
  int st = lvb_gemm_check(d);
  if (st) return st;
  if (!out) return fail(LVB_ERR_INVALID_ARG, "lvb_gemm", "plan is NULL");
  if (sm_count <= 0) sm_count = 148;
  std::memset(out, 0, sizeof *out);
  if (d->M == 0 || d->N == 0) return LVB_OK;   // nothing to launch
  if (allow_gemv && gemv_applies(d)) {
    GemvPlan g;
    gemv_plan(d, sm_count, &g);
    out->gemv = 1;
    out->gemv_ksplit = g.ksplit;
    out->ctas = g.ctas;
    out->launches = g.ksplit > 1 ? 2 : 1;
    return LVB_OK;
  }
  // Orientation: the kernel stores its accumulator rows (m) from TMEM lanes. When C can take
  // TMA stores (leading dimension a 16-byte multiple), kernel-space n is C's contiguous
  // dimension, so each thread's 32 columns are one contiguous run staged as 16-byte vectors;
  // otherwise kernel-space m is, so a warp's direct stores of one column are contiguous.
  // LVB_GEMM_STORE=direct forces the second (tuning).
  static const bool env_direct = [] {
    const char* s = std::getenv("LVB_GEMM_STORE");
    return s && std::string(s) == "direct";
  }();
  const bool c_tma = c_tma_ok && !env_direct;
  out->swap_ab = (d->c_rowmajor != 0) != c_tma ? 1 : 0;
  const int64_t kM = out->swap_ab ? d->N : d->M;
  const int64_t kN = out->swap_ab ? d->M : d->N;
  const int64_t tiles_m = (kM + 127) / 128;
  // MN-contiguous operands (A column-major, B row-major) are read MN-major in place when they
  // are 16-bit; 8-bit ones are copied K-major first.
  const int es = dtype_size(d->a_type);
  const bool a_mn = !d->a_rowmajor, b_mn = d->b_rowmajor != 0;
  out->repack_a = (d->lda * es) % 16 != 0 || (a_mn && es == 1);
  out->repack_b = (d->ldb * es) % 16 != 0 || (b_mn && es == 1);
  out->a_mnmajor = a_mn && !out->repack_a;
  out->b_mnmajor = b_mn && !out->repack_b;
  const bool kb_mn = out->swap_ab ? out->a_mnmajor : out->b_mnmajor;
  const bool out32 = dtype_size(d->c_type) == 4;
  // Pick the tile width by estimated efficiency: wave quantisation times the intrinsic
  // efficiency of the narrower MMA (operand re-reads grow as BN shrinks).
  // Candidates 1024, 512 and 448 stand for the CTA-pair kernels with 512×256, 256×256 and
  // 256×224 tiles (one tile per two SMs; the 512-row tile shares each B stage between two
  // 256-row blocks, a quarter less operand traffic per FLOP; the 224-wide tile for 32-bit
  // outputs with B read K-major makes whole waves of 8192-wide outputs at 1024 or 2048 rows).
  // LVB_GEMM_TILE=1024|512|448|256|128|64 forces one (tuning).
  const int cands[6] = {1024, 512, 448, 256, 128, 64};
  // The tall pair tile's factor: C2 at 1,512 vs 1,425 TFLOP/s (20 launches) and 1,335 vs
  // 1,279 (400 launches, at the power cap) against the square pair tile.
  const double intrinsic[6] = {1.12, 1.08, 1.0, 1.0, 0.86, 0.62};
  static const int forced = [] {
    const char* s = std::getenv("LVB_GEMM_TILE");
    return s ? std::atoi(s) : 0;
  }();
  double best = -1;
  int bn = 256;
  for (int i = 0; i < 6; ++i) {
    if (forced && cands[i] != forced) continue;
    if (cands[i] == 448 && (!out32 || kb_mn)) continue;
    const bool pair = cands[i] >= 448;
    const bool tall = cands[i] == 1024;        // 512 × 256 tiles on a CTA pair
    const int64_t pw = tall ? 256 : cands[i] / 2;   // the pair's tile width
    const int64_t tm = tall ? (kM + 511) / 512 : pair ? (kM + 255) / 256 : tiles_m;
    const int64_t tn = pair ? (kN + pw - 1) / pw : (kN + cands[i] - 1) / cands[i];
    const int64_t slots = pair ? std::max(1, sm_count / 2) : sm_count;
    const int64_t tiles = tm * tn;
    const int64_t waves = (tiles + slots - 1) / slots;
    const double eff = waves ? intrinsic[i] * (double)tiles / (double)(waves * slots) : 0;
    if (eff > best + 1e-9) { best = eff; bn = cands[i]; }
  }
  const bool pair = bn >= 448;
  out->cta_pair = pair ? 1 : 0;
  out->tile_m = bn == 1024 ? 512 : pair ? 256 : 128;
  out->tile_n = bn == 1024 ? 256 : pair ? bn / 2 : bn;
  out->tile_k = 128 / dtype_size(d->a_type);
  out->stages = gemm_stages(bn);
  out->tiles = (int32_t)(((kM + out->tile_m - 1) / out->tile_m) *
                         ((kN + out->tile_n - 1) / out->tile_n));
  out->ctas = pair ? 2 * std::max(1, std::min<int32_t>(out->tiles, std::max(1, sm_count / 2)))
                   : std::max(1, std::min<int32_t>(out->tiles, sm_count));
  out->smem_bytes = gemm_smem_bytes(bn);
  out->tmem_cols = pair ? 512 : 2 * bn;
  out->instr_m = pair ? 256 : out->tile_m;
  out->instr_n = out->tile_n;
  out->instr_k = (d->a_type == LVB_I8 || d->a_type == LVB_U8) ? 32 : 16;
  out->launches = d->K == 0 ? 1 : 1 + out->repack_a + out->repack_b;
  return LVB_OK;
}
}  // namespace lvb
extern "C" {

static int gemm_enqueue(const char* op, const lvb_gemm_desc* d, const lvb_epilogue* e,
                        const void* A, const void* B, void* C, void* stream) {
  if (d->M == 0 || d->N == 0) return LVB_OK;
  if (!C) return fail(LVB_ERR_INVALID_ARG, op, "C is NULL");
  if (d->K > 0 && (!A || !B)) return fail(LVB_ERR_INVALID_ARG, op, "A or B is NULL");
  const int es = dtype_size(d->a_type);
  if (((uintptr_t)A) % es || ((uintptr_t)B) % es || ((uintptr_t)C) % dtype_size(d->c_type))
    return fail(LVB_ERR_INVALID_ARG, op, "pointer not aligned to its element size");
  DeviceState* dev = current_device_state(op);
  if (!dev) return LVB_ERR_NO_DEVICE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool prog = e && e->program && e->program->n > 0;
  const bool clamp = e && e->k_pad > d->K;
  const bool epi = e && (e->bias || e->residual || e->activation != LVB_ACT_NONE || e->mul ||
                         prog || clamp);
  if (d->K == 0) return epi ? gemm_epilogue_only(d, e, C, s) : gemm_zero_fill(d, C, s);
  // The matrix-vector kernel carries bias, residual and activation; coopmat_mul, programs and
  // clamped k tails run on the tensor-core kernel at any shape.
  if (gemv_applies(d) && !(e && (e->mul || prog || clamp)))
    return gemv_launch(d, epi ? e : nullptr, A, B, C, s, dev);
  lvb_gemm_plan plan;
  const bool c_tma_ok =
      (uintptr_t)C % 16 == 0 && (d->ldc * dtype_size(d->c_type)) % 16 == 0;
  // The plan depends only on the descriptor, the SM count and whether C takes TMA stores: a
  // call repeating the last one on this thread (a small GEMM in a loop, whose time is the
  // host's) reuses it. The key is compared byte for byte, so a miss is always safe.
  struct PlanMemo {
    lvb_gemm_desc d;
    int32_t sm_count;
    int32_t c_tma_ok;
    lvb_gemm_plan plan;
    bool valid;
  };
  static thread_local PlanMemo memo{};
  if (memo.valid && memo.sm_count == dev->sm_count && memo.c_tma_ok == (int32_t)c_tma_ok &&
      std::memcmp(&memo.d, d, sizeof *d) == 0) {
    plan = memo.plan;
  } else {
    int st = gemm_plan_c(d, dev->sm_count, c_tma_ok, &plan, /*allow_gemv=*/false);
    if (st) return st;
    memo.d = *d;
    memo.sm_count = dev->sm_count;
    memo.c_tma_ok = (int32_t)c_tma_ok;
    memo.plan = plan;
    memo.valid = true;
  }
  if (((uintptr_t)A) % 16) plan.repack_a = 1, plan.a_mnmajor = 0;
  if (((uintptr_t)B) % 16) plan.repack_b = 1, plan.b_mnmajor = 0;
  return gemm_launch(d, plan, A, B, C, epi ? e : nullptr, s, dev);
}

int lvb_gemm(const lvb_gemm_desc* d, const void* A, const void* B, void* C, void* stream) {
  // The check depends only on the descriptor: the last one that passed on this thread
  // passes again.
  static thread_local lvb_gemm_desc checked{};
  static thread_local bool checked_valid = false;
  if (!(d && checked_valid && std::memcmp(&checked, d, sizeof *d) == 0)) {
    const int st = lvb_gemm_check(d);
    if (st) return st;
    checked = *d;
    checked_valid = true;
  }
  return gemm_enqueue("lvb_gemm", d, nullptr, A, B, C, stream);
}

int lvb_gemm_ex(const lvb_gemm_desc* d, const lvb_epilogue* e, const void* A, const void* B,
                void* C, void* stream) {
  int st = lvb_gemm_ex_check(d, e);
  if (st) return st;
  return gemm_enqueue("lvb_gemm_ex", d, e, A, B, C, stream);
}

// ---------------------------------------------------------------------------------------
// Attention
// ---------------------------------------------------------------------------------------
int lvb_attention_check(const lvb_attn_desc* d) {
  const char* op = "lvb_attention_fwd";
  if (!d) return fail(LVB_ERR_INVALID_ARG, op, "descriptor is NULL");
  if (d->batch < 0 || d->heads_q < 0 || d->heads_kv < 0 || d->seq_q < 0 || d->seq_kv < 0 ||
      d->head_dim < 0)
    return fail(LVB_ERR_INVALID_ARG, op, "negative extent");
  if (d->dtype != LVB_F16 && d->dtype != LVB_BF16)
    return fail(LVB_ERR_UNSUPPORTED, op, std::string("no kernel for ") + dtype_name(d->dtype),
                "Float16 or BFloat16");
  if (d->heads_kv == 0 || (d->heads_q % d->heads_kv) != 0)
    return fail(LVB_ERR_INVALID_ARG, op, "heads_q must be a positive multiple of heads_kv");
  if (d->head_dim != 128 && d->head_dim != 64)
    return fail(LVB_ERR_UNSUPPORTED, op, "head_dim must be 64 or 128");
  if (!(d->scale > 0.0f) || d->scale != d->scale)
    return fail(LVB_ERR_INVALID_ARG, op, "scale must be a positive finite number");
  if (d->seq_q > INT32_MAX || d->seq_kv > INT32_MAX || d->batch * d->heads_q > INT32_MAX)
    return fail(LVB_ERR_UNSUPPORTED, op, "extent above 2^31-1");
  const int64_t* strides[4] = {d->q_stride, d->k_stride, d->v_stride, d->o_stride};
  for (int t = 0; t < 4; ++t) {
    const int64_t* s = strides[t];
    if (s[0] == 0 && s[1] == 0 && s[2] == 0) continue;
    if (s[2] < d->head_dim) return fail(LVB_ERR_INVALID_ARG, op, "seq stride < head_dim");
    if ((s[0] * 2) % 16 || (s[1] * 2) % 16 || (s[2] * 2) % 16)
      return fail(LVB_ERR_UNSUPPORTED, op, "strides must be multiples of 16 bytes");
  }
  return LVB_OK;
}

int lvb_attention_plan_for(const lvb_attn_desc* d, int32_t sm_count, lvb_attn_plan* out) {
  int st = lvb_attention_check(d);
  if (st) return st;
  if (!out) return fail(LVB_ERR_INVALID_ARG, "lvb_attention_fwd", "plan is NULL");
  if (sm_count <= 0) sm_count = 148;
  std::memset(out, 0, sizeof *out);
  out->splits = 1;
  if (d->batch == 0 || d->heads_q == 0 || d->seq_q == 0) return LVB_OK;
  if (d->seq_kv == 0) {
    out->kernel = LVB_ATTN_EMPTY;
    out->launches = 1;
    return LVB_OK;
  }
  if (attn_decode_applies(d)) {
    int ns = 1, bps = 1, ctas = 1;
    attn_decode_plan(d, sm_count, &ns, &bps, &ctas);
    out->kernel = LVB_ATTN_DECODE;
    out->splits = ns;
    out->ctas = ctas;
    out->launches = ns > 1 ? 2 : 1;   // + the merge of the splits
    return LVB_OK;
  }
  out->kernel = LVB_ATTN_FLASH;
  const long long items = ((d->seq_q + 255) / 256) * d->batch * d->heads_q;
  out->ctas = (int32_t)std::min<long long>(items, sm_count);   // persistent
  out->launches = 1;
  return LVB_OK;
}

int lvb_attention_fwd(const lvb_attn_desc* d, const void* Q, const void* K, const void* V,
                      void* O, float* lse, void* stream) {
  const char* op = "lvb_attention_fwd";
  int st = lvb_attention_check(d);
  if (st) return st;
  if (d->batch == 0 || d->heads_q == 0 || d->seq_q == 0) return LVB_OK;
  if (!Q || !O || (d->seq_kv > 0 && (!K || !V)))
    return fail(LVB_ERR_INVALID_ARG, op, "Q, K, V or O is NULL");
  if (((uintptr_t)Q) % 16 || ((uintptr_t)K) % 16 || ((uintptr_t)V) % 16 || ((uintptr_t)O) % 16)
    return fail(LVB_ERR_UNSUPPORTED, op, "tensors must start on 16-byte boundaries");
  DeviceState* dev = current_device_state(op);
  if (!dev) return LVB_ERR_NO_DEVICE;
  return attn_launch(d, Q, K, V, O, lse, reinterpret_cast<cudaStream_t>(stream), dev);
}

// ---------------------------------------------------------------------------------------
// Sharding
// ---------------------------------------------------------------------------------------
int lvb_shard_range(int64_t total, int32_t world, int32_t rank, int64_t align, int64_t* begin,
                    int64_t* count) {
  const char* op = "lvb_shard_range";
  if (!begin || !count) return fail(LVB_ERR_INVALID_ARG, op, "begin or count is NULL");
  if (total < 0 || world <= 0 || rank < 0 || rank >= world || align <= 0)
    return fail(LVB_ERR_INVALID_ARG, op, "need total >= 0, 0 <= rank < world, align > 0");
  // Whole aligned chunks are dealt out as evenly as possible, lower ranks first; the ragged
  // tail chunk (total % align) goes to the rank that owns the last chunk.
  const int64_t chunks = (total + align - 1) / align;
  const int64_t base = chunks / world, extra = chunks % world;
  const int64_t c0 = rank * base + std::min<int64_t>(rank, extra);
  const int64_t nc = base + (rank < extra ? 1 : 0);
  int64_t b = std::min(total, c0 * align);
  int64_t e = std::min(total, (c0 + nc) * align);
  *begin = b;
  *count = e - b;
  return LVB_OK;
}

// ---------------------------------------------------------------------------------------
// Runtime helpers
// ---------------------------------------------------------------------------------------
int lvb_device_count(int32_t* n) {
  if (!n) return fail(LVB_ERR_INVALID_ARG, "lvb_device_count", "n is NULL");
  int c = 0;
  cudaError_t e = cudaGetDeviceCount(&c);
  if (e != cudaSuccess) { *n = 0; return LVB_OK; }
  *n = c;
  return LVB_OK;
}
int lvb_set_device(int device) {
  cudaError_t e = cudaSetDevice(device);
  return e == cudaSuccess ? LVB_OK : fail_cuda(e, "lvb_set_device", "cudaSetDevice");
}
int lvb_malloc(void** ptr, size_t bytes) {
  if (!ptr) return fail(LVB_ERR_INVALID_ARG, "lvb_malloc", "ptr is NULL");
  cudaError_t e = cudaMalloc(ptr, bytes);
  return e == cudaSuccess ? LVB_OK : fail_cuda(e, "lvb_malloc", "cudaMalloc");
}
int lvb_free(void* ptr) {
  cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? LVB_OK : fail_cuda(e, "lvb_free", "cudaFree");
}
int lvb_memcpy_htod(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes && (!dst || !src)) return fail(LVB_ERR_INVALID_ARG, "lvb_memcpy_htod", "NULL pointer");
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, (cudaStream_t)stream);
  return e == cudaSuccess ? LVB_OK : fail_cuda(e, "lvb_memcpy_htod", "cudaMemcpyAsync");
}
int lvb_memcpy_dtoh(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes && (!dst || !src)) return fail(LVB_ERR_INVALID_ARG, "lvb_memcpy_dtoh", "NULL pointer");
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, (cudaStream_t)stream);
  return e == cudaSuccess ? LVB_OK : fail_cuda(e, "lvb_memcpy_dtoh", "cudaMemcpyAsync");
}
int lvb_stream_create(void** stream) {
  if (!stream) return fail(LVB_ERR_INVALID_ARG, "lvb_stream_create", "stream is NULL");
  cudaError_t e = cudaStreamCreateWithFlags((cudaStream_t*)stream, cudaStreamNonBlocking);
  return e == cudaSuccess ? LVB_OK : fail_cuda(e, "lvb_stream_create", "cudaStreamCreate");
}
int lvb_stream_destroy(void* stream) {
  cudaError_t e = cudaStreamDestroy((cudaStream_t)stream);
  return e == cudaSuccess ? LVB_OK : fail_cuda(e, "lvb_stream_destroy", "cudaStreamDestroy");
}
int lvb_stream_synchronize(void* stream) {
  cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
  return e == cudaSuccess ? LVB_OK : fail_cuda(e, "lvb_stream_synchronize", "cudaStreamSynchronize");
}
int lvb_device_status(void* stream, int32_t* code, int32_t* where, int32_t* block) {
  const char* op = "lvb_device_status";
  DeviceState* dev = current_device_state(op);
  if (!dev) return LVB_ERR_NO_DEVICE;
  cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) return fail_cuda(e, op, "cudaStreamSynchronize");
  DevStatus h;
  e = cudaMemcpy(&h, dev->status, sizeof h, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return fail_cuda(e, op, "reading the status word");
  if (h.code != 0) {
    e = cudaMemset(dev->status, 0, sizeof(DevStatus));
    if (e != cudaSuccess) return fail_cuda(e, op, "clearing the status word");
  }
  if (code) *code = h.code;
  if (where) *where = h.where;
  if (block) *block = h.block;
  return LVB_OK;
}
int lvb_set_wait_timeout_ms(int64_t ms) {
  if (ms <= 0) return fail(LVB_ERR_INVALID_ARG, "lvb_set_wait_timeout_ms", "ms must be > 0");
  wait_timeout_ns();  // settle the env default first
  std::lock_guard<std::mutex> lk(g_timeout_mu);
  g_timeout_ms = ms;
  return LVB_OK;
}

}  // extern "C"
