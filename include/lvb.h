/*
 * lvb.h — C ABI of liblvb, the B200 (sm_100a) backend for the cooperative-matrix GEMM and
 * flash-attention path of Lava.jl.
 *
 * Lava.jl is a compiler: a kernel author writes a GEMM or attention kernel against its
 * device vocabulary (CoopMatrix / AcceleratedMatrix / WorkgroupMatrix, coopmat_load,
 * muladd, convert, copyto!, coopmat_reduce, coopmat_perelement, tensor_load with clamp),
 * Lava lowers it to SPIR-V and a Vulkan runtime dispatches it. This library replaces that
 * execution path for the two ops that vocabulary exists to serve: every entry point below
 * is what a host package binds with `ccall` in place of compiling and dispatching a
 * coopmat kernel. The reference interface each one stands in for is cited beside it
 * (paths relative to the Lava.jl source tree).
 *
 * Conventions
 *  - Plain pointers and sizes; device pointers are CUDA device addresses, `stream` is a
 *    cudaStream_t / CUstream (NULL = the legacy default stream).
 *  - Every entry point returns an lvb_status. On failure lvb_last_error() returns a
 *    thread-local message of the form "<operation>: <message> (<suggestion>)", the triad
 *    of Lava's LavaError (src/runtime/errors.jl:4-24).
 *  - Work is enqueued on the caller's stream and returns without synchronising. A device
 *    side failure (a bounded wait that expired) is recorded in a per-device status word
 *    that lvb_device_status() reads, like Lava's exception flag word that the host checks
 *    at the next synchronisation (src/compiler/entry_wrapper.jl:9-11,199-216).
 *  - The GEMM kernels are launched with programmatic stream serialization: they may be
 *    scheduled while the stream's previous kernel ends but touch global memory only after
 *    it has completed (griddepcontrol.wait), and they let the next kernel be scheduled
 *    early. A caller's kernel launched after a GEMM with that same attribute must wait
 *    (griddepcontrol.wait) before reading the GEMM's output; other kernels see plain stream
 *    order.
 *  - The library never frees caller memory and holds no pointer past a call.
 */
#ifndef LVB_H
#define LVB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LVB_ABI_VERSION 5

typedef enum lvb_status {
  LVB_OK = 0,
  LVB_ERR_INVALID_ARG = 1, /* a null pointer, a negative size, a leading dimension too small */
  LVB_ERR_UNSUPPORTED = 2, /* a legal request this build does not implement (dtype pair, layout, alignment) */
  LVB_ERR_CUDA = 3,        /* a CUDA runtime/driver call failed */
  LVB_ERR_TIMEOUT = 4,     /* a kernel's bounded wait expired (read through lvb_device_status) */
  LVB_ERR_NCCL = 5,        /* NCCL missing or a collective failed */
  LVB_ERR_NO_DEVICE = 6    /* no sm_100 device visible */
} lvb_status;

/* Component types. Lava's coopmat component types are Float16, Float32, Int8, UInt8,
 * Int32, UInt32 (src/device/coopmat_intrinsics.jl:16-19); BFloat16 is added for B200. */
typedef enum lvb_dtype {
  LVB_F16 = 0,
  LVB_BF16 = 1,
  LVB_F32 = 2,
  LVB_I8 = 3,
  LVB_U8 = 4,
  LVB_I32 = 5,
  LVB_U32 = 6
} lvb_dtype;

/* Matrix scopes (src/vocabulary/matrix.jl:60-66). */
typedef enum lvb_scope { LVB_SUBGROUP_SCOPE = 0, LVB_WORKGROUP_SCOPE = 1 } lvb_scope;

/* ---------------------------------------------------------------------------------------
 * Capabilities — the answer a backend gives to Lava.caps(backend) (src/vocabulary/caps.jl:
 * 54-65, 120) and to matrix_shapes / supports / bestshape (caps.jl:158-169,
 * src/vocabulary/matrix.jl:88-172).
 * ------------------------------------------------------------------------------------- */
typedef struct lvb_matrix_shape {
  int32_t ab;    /* lvb_dtype of A and B */
  int32_t acc;   /* lvb_dtype of the accumulator */
  int32_t M, N, K;
  int32_t scope; /* lvb_scope */
} lvb_matrix_shape;

typedef struct lvb_device_caps {
  int32_t coopmat;          /* matrix multiply-add usable at all */
  int32_t tile;             /* square fp16->fp32 instruction extent */
  int32_t subgroup;         /* lanes per subgroup (warp) */
  int32_t coopmatsubgroup;  /* subgroup width a matrix kernel gets */
  int64_t sharedbudget;     /* bytes of workgroup-shared memory per workgroup */
  int32_t workgrouplimit;   /* threads per workgroup */
  int32_t cores;            /* SMs */
  int32_t warps;            /* max resident subgroups per SM */
  int32_t n_wggran;         /* rows used in wggran */
  int32_t wggran[8][4];     /* (invocations, M, N, K) workgroup-scope granularity rows */
  int32_t n_shapes;         /* number of subgroup-scope shapes lvb_matrix_shapes reports */
  int32_t cc_major, cc_minor;
} lvb_device_caps;

/* Static caps of a B200 (sm_100a) — host only, needs no GPU. Used by lvb_caps and by tests
 * that check a tiling decision on a machine without the device (caps.jl:84-108). */
int lvb_caps_sm100(lvb_device_caps* out);
/* Caps of CUDA device `device`: the sm_100a table with the live SM count / shared budget.
 * Returns LVB_ERR_NO_DEVICE when the device is absent or not sm_100. */
int lvb_caps(int device, lvb_device_caps* out);
/* The subgroup-scope shape table (matrix_shapes, caps.jl:158-159). Writes up to
 * `capacity` entries and the total count to *count. Host only. */
int lvb_matrix_shapes(lvb_matrix_shape* out, int32_t capacity, int32_t* count);
/* bestshape (matrix.jl:155-172): squarest, then largest, among shapes with ab/acc/scope.
 * Returns LVB_ERR_UNSUPPORTED when the table has none (Lava's `nothing`). Host only. */
int lvb_bestshape(int32_t ab, int32_t acc, int32_t scope, lvb_matrix_shape* out);

/* ---------------------------------------------------------------------------------------
 * GEMM: C = A·B with accumulation in C's element type, as coopmat_muladd does
 * (src/vocabulary/coopmat.jl:190-203; src/device/coopmat_intrinsics.jl:303-320), loads and
 * stores with Lava's addressing — `stride` elements between rows (row-major, Val(true)) or
 * columns (column-major) (coopmat.jl:124-161; coopmat_intrinsics.jl:57-75,179-218) — and
 * the fp32 -> fp16/bf16 conversion of `convert` (round to nearest even; coopmat.jl:178-182)
 * fused into the store. Ragged edges follow TENSOR_CLAMP_CONSTANT with value 0
 * (src/vocabulary/tensor.jl:46-51): the tile is computed over zero-filled operands and the
 * store is clamped to the matrix. Replaces compiling and dispatching a coopmat GEMM kernel
 * (the loop of test/glsl/coopmat2_gemm_regs.comp:53-83).
 * ------------------------------------------------------------------------------------- */
typedef struct lvb_gemm_desc {
  int32_t a_type, b_type, c_type; /* lvb_dtype */
  int32_t a_rowmajor;             /* A (M×K): 1 row-major (lda >= K), 0 column-major (lda >= M) */
  int32_t b_rowmajor;             /* B (K×N): 0 column-major (ldb >= K), 1 row-major (ldb >= N) */
  int32_t c_rowmajor;             /* 0: C (M×N) column-major (ldc >= M); 1: row-major (ldc >= N) */
  int64_t M, N, K;
  int64_t lda, ldb, ldc;          /* elements */
} lvb_gemm_desc;

/* The tiling the library will use for a descriptor (host only, no GPU). */
typedef struct lvb_gemm_plan {
  int32_t swap_ab;      /* 1: computed as Cᵀ = Bᵀ·Aᵀ so the store is lane-contiguous */
  int32_t tile_m, tile_n, tile_k;
  int32_t stages;
  int32_t tiles;        /* output tiles */
  int32_t ctas;         /* persistent CTAs launched (<= SM count) */
  int32_t smem_bytes;   /* dynamic shared memory per CTA */
  int32_t tmem_cols;    /* TMEM columns allocated per CTA */
  int32_t instr_m, instr_n, instr_k; /* tcgen05.mma shape */
  int32_t repack_a, repack_b;        /* operand copied K-major into an aligned stream-ordered
                                        workspace first (leading dimension or base not 16-byte
                                        aligned, or an 8-bit operand stored MN-contiguous) */
  int32_t cta_pair;                  /* 1: tiles on CTA pairs (tcgen05 cta_group::2): 256x256,
                                        256x224 (32-bit outputs), or 512x256 (tile_m 512: two
                                        256-row blocks sharing each B stage) */
  int32_t a_mnmajor, b_mnmajor;      /* operand read by the tensor core MN-major, in place (A
                                        column-major / B row-major, 16-bit types) */
  int32_t gemv;                      /* 1: N == 1 or M == 1 — a matrix-vector product, streamed
                                        by the HBM-bound kernel (dot4x8 for 8-bit types), not
                                        the tensor core; the tile fields above are then 0 */
  int32_t gemv_ksplit;               /* k split across CTAs for it (partial sums in a
                                        stream-ordered workspace, added in a fixed order) */
  int32_t launches;                  /* kernel launches per call, operand copies and the
                                        split sums included (0 for an empty C) */
} lvb_gemm_plan;

/* Validate a descriptor (host only). */
int lvb_gemm_check(const lvb_gemm_desc* d);
/* Validate and plan for `sm_count` SMs (host only). */
int lvb_gemm_plan_for(const lvb_gemm_desc* d, int32_t sm_count, lvb_gemm_plan* out);
/* Enqueue C = A·B on `stream` (on the current CUDA device). Supported pairs:
 *   F16×F16 -> F32|F16|BF16,  BF16×BF16 -> F32|F16|BF16,  I8×I8 -> I32,  U8×U8 -> U32.
 * Every layout of A, B and C, any leading dimension >= the extent. A K-contiguous operand
 * (A row-major, B column-major) is read K-major; an MN-contiguous one — Lava's transposing
 * tensor view, permutation (1,0) (src/device/tensor_intrinsics.jl:212-320) — is read
 * MN-major in place when its type is 16-bit. An operand whose base or leading dimension is
 * not a 16-byte multiple, or an 8-bit operand stored MN-contiguous, is first copied K-major
 * on the device into a stream-ordered workspace (allocated on `stream` from the library's
 * per-device memory pool, which keeps up to 512 MiB of freed workspace for the next call,
 * and freed on `stream`). With N == 1 or M == 1 the product is a matrix-vector product and runs on the
 * HBM-bound kernel instead (any layout; 8-bit operands through dot4x8, Lava's
 * src/vocabulary/vocabulary.jl:18-35); when its rows alone cannot fill the GPU, k is split
 * across CTAs with partial sums in a stream-ordered workspace. */
int lvb_gemm(const lvb_gemm_desc* d, const void* A, const void* B, void* C, void* stream);

/* Fused epilogue: C = f(act((A·B + bias + R) ⊙ S)), computed in fp32 and converted once to
 * C's type, with A·B taken over the padded k extent when k_pad > K (the clamp modes).
 * The accumulator starting from bias + residual is Lava's coopmat_add accumulator
 * initialisation — the bias loaded at stride 0 so every column (or row) reads the same
 * vector, the residual at its own leading dimension (src/device/coopmat_intrinsics.jl:
 * 435-447; src/compiler/spirv/coopmat.jl:873-878) — and `act` the per-element function a
 * GEMM applies to its accumulator with coopmat_perelement / getcomp+setcomp (coopmat_
 * intrinsics.jl:322-331,551-593) before convert and copyto! (src/vocabulary/coopmat.jl:
 * 166-176); S the coopmat_mul operand and f the caller's per-element program. Bias, residual,
 * S, activation and program need a floating-point output (coopmat_add and coopmat_mul are
 * OpFAdd / OpFMul); the clamp modes apply to every pair, integer ones exactly. */
typedef enum lvb_activation {
  LVB_ACT_NONE = 0,
  LVB_ACT_RELU = 1,       /* x < 0 ? 0 : x */
  LVB_ACT_GELU_TANH = 2,  /* 0.5x(1 + tanh(sqrt(2/pi)(x + 0.044715x^3))) */
  LVB_ACT_GELU_ERF = 3,   /* 0.5x(1 + erf(x/sqrt(2))) */
  LVB_ACT_SILU = 4        /* x / (1 + exp(-x)) */
} lvb_activation;

typedef enum lvb_bias_axis {
  LVB_BIAS_PER_ROW = 0,   /* bias[i] added to row i: M elements (column-major stride-0 load) */
  LVB_BIAS_PER_COL = 1    /* bias[j] added to column j: N elements (row-major stride-0 load) */
} lvb_bias_axis;

/* Tensor clamp modes of the operands' loads (src/vocabulary/tensor.jl:46-51). */
typedef enum lvb_clamp {
  LVB_CLAMP_UNDEFINED = 0, /* a read past the extent is undefined; this library reads 0 */
  LVB_CLAMP_CONSTANT = 1,  /* reads the clamp value, rounded to the operand's type
                              (tensor_clampbits, tensor.jl:83-85) */
  LVB_CLAMP_TO_EDGE = 2    /* reads the nearest element inside the operand */
} lvb_clamp;

/* A caller-supplied per-element function, Lava's coopmat_perelement(f, m, extras...)
 * (src/device/coopmat_intrinsics.jl:520-678): f(row0, col0, elem, extra) evaluated for every
 * element of the result, with 0-based row and column of C (coopmat_intrinsics.jl:551-593),
 * the element, and the element at the same position of an optional second matrix (the
 * matrix-operand form). Written as a straight-line program over 8 registers of 32 bits; at
 * its start r0 = the element (float), r1 = row (int32), r2 = col (int32), r3 = the extra
 * matrix's element (float, 0 without one), r4..r7 = 0; its result is r0 (float). Float
 * operations round as IEEE fp32 (exp/log/tanh/erf within a few ulp of the correctly rounded
 * value); integer operations wrap as int32. */
#define LVB_PE_MAX_INSTR 32
#define LVB_PE_REGS 8
typedef enum lvb_pe_op {
  LVB_PE_CONST = 0,   /* r[dst] = the fp32 value with bits imm */
  LVB_PE_ICONST = 1,  /* r[dst] = (int32)imm */
  LVB_PE_MOV = 2,     /* r[dst] = r[a] */
  LVB_PE_FADD = 3,    /* r[dst] = r[a] + r[b] (fp32) */
  LVB_PE_FSUB = 4,
  LVB_PE_FMUL = 5,
  LVB_PE_FDIV = 6,
  LVB_PE_FMIN = 7,    /* fminf / fmaxf: a NaN operand yields the other */
  LVB_PE_FMAX = 8,
  LVB_PE_FFMA = 9,    /* r[dst] = fma(r[a], r[b], r[dst]) */
  LVB_PE_FNEG = 10,   /* r[dst] = f(r[a]) for the unary functions below */
  LVB_PE_FABS = 11,
  LVB_PE_FEXP = 12,
  LVB_PE_FEXP2 = 13,
  LVB_PE_FLOG = 14,
  LVB_PE_FTANH = 15,
  LVB_PE_FSQRT = 16,
  LVB_PE_FRSQRT = 17,
  LVB_PE_FFLOOR = 18,
  LVB_PE_FERF = 19,
  LVB_PE_I2F = 20,    /* r[dst] = (float)(int32)r[a] (RNE) */
  LVB_PE_IADD = 21,   /* r[dst] = r[a] + r[b] (int32, wrapping) */
  LVB_PE_ISUB = 22,
  LVB_PE_IMUL = 23,
  LVB_PE_IMIN = 24,
  LVB_PE_IMAX = 25,
  LVB_PE_FLT = 26,    /* r[dst] = (r[a] < r[b]) ? 1 : 0 (int32 result; fp32 comparison) */
  LVB_PE_FLE = 27,
  LVB_PE_FEQ = 28,
  LVB_PE_ILT = 29,    /* the same with int32 operands */
  LVB_PE_ILE = 30,
  LVB_PE_IEQ = 31,
  LVB_PE_SELECT = 32, /* r[dst] = r[a] != 0 ? r[b] : r[dst] (bitwise test of the word) */
  LVB_PE_NUM_OPS = 33
} lvb_pe_op;

typedef struct lvb_pe_instr {
  uint8_t op;         /* lvb_pe_op */
  uint8_t dst, a, b;  /* registers 0..7 (unused operands 0) */
  uint32_t imm;       /* LVB_PE_CONST: fp32 bits; LVB_PE_ICONST: int32 */
} lvb_pe_instr;

typedef struct lvb_pe_program {
  int32_t n;          /* instructions used, 0..LVB_PE_MAX_INSTR */
  lvb_pe_instr code[LVB_PE_MAX_INSTR];
} lvb_pe_program;

typedef struct lvb_epilogue {
  const void* bias;       /* NULL: none. Contiguous vector of bias_type */
  const void* residual;   /* NULL: none. M×N in C's layout, leading dimension ldr; may be C
                             itself (same pointer, ldr == ldc, same type), no other overlap */
  int64_t ldr;
  int32_t bias_type;      /* LVB_F32 | LVB_F16 | LVB_BF16 */
  int32_t bias_axis;      /* lvb_bias_axis */
  int32_t residual_type;  /* LVB_F32 | LVB_F16 | LVB_BF16 */
  int32_t activation;     /* lvb_activation */
  /* coopmat_mul (src/device/coopmat_intrinsics.jl:402-464): the accumulator multiplied
   * element-wise by S, M×N in C's layout with leading dimension ldm (NULL: none). */
  const void* mul;
  int64_t ldm;
  int32_t mul_type;       /* LVB_F32 | LVB_F16 | LVB_BF16 */
  int32_t extra_type;     /* LVB_F32 | LVB_F16 | LVB_BF16 */
  /* the matrix operand of the per-element program (r3), M×N in C's layout (NULL: none) */
  const void* extra;
  int64_t lde;
  const lvb_pe_program* program;  /* NULL: none. Read during the call only. */
  /* Clamped operand loads over a padded k extent: the product runs over k_pad >= K columns
   * of A and rows of B, and the reads past K take each operand's clamp mode — what a Lava
   * kernel computes when its k loop steps a tile that does not divide K through tensor
   * layouts with these clamps (tensor_intrinsics.jl:139-148). k_pad 0 (or K): no padding,
   * clamps unused. Rows past M and columns past N are never stored, so only the k tail of
   * each operand is read through its clamp. */
  int64_t k_pad;
  int32_t a_clamp;        /* lvb_clamp of A's reads past column K-1 */
  int32_t b_clamp;        /* lvb_clamp of B's reads past row K-1 */
  double a_clamp_value;   /* LVB_CLAMP_CONSTANT: the value (integer types: an integer in range) */
  double b_clamp_value;
} lvb_epilogue;

/* Validate a per-element program: instruction count, opcodes, registers (host only). */
int lvb_pe_program_check(const lvb_pe_program* program);
/* Validate a descriptor with its epilogue (host only; `e` may be NULL). */
int lvb_gemm_ex_check(const lvb_gemm_desc* d, const lvb_epilogue* e);
/* lvb_gemm with the fused epilogue `e` (NULL: exactly lvb_gemm). With K == 0 the result is
 * act(bias + R). */
int lvb_gemm_ex(const lvb_gemm_desc* d, const lvb_epilogue* e, const void* A, const void* B,
                void* C, void* stream);

/* lvb_gemm for callers that must not allocate device memory while they run a GEMM (a host
 * runtime that owns all device memory through its own pool, a serving loop that forbids
 * allocation after warm-up). No counterpart in the
 * reference: Lava has no host GEMM entry point at all; this is a second form of lvb_gemm.
 * Same arguments, semantics and results as lvb_gemm; it calls no cudaMalloc, cudaFree,
 * cudaMallocAsync or other device allocator. Its scratch — the device status word and the
 * workspace for operands that must be copied first — is one static device array of
 * 16 MiB + 256 bytes that every GPU loading the library keeps until the process exits.
 * Operands needing more than 16 MiB of copies are refused with LVB_ERR_UNSUPPORTED. An operand
 * is copied when its base or leading dimension is not a 16-byte multiple, and an 8-bit operand
 * stored MN-contiguous (Int8/UInt8 A column-major or B row-major) is copied K-major at any
 * alignment; other operands need no copy, at any size. The first call on a device looks up
 * the array's device address (cudaGetSymbolAddress) with that device current, which also
 * loads this part of the library onto the device when CUDA loads modules lazily (the array
 * is placed on the device then); make that first call before any stream capture. The address
 * is looked up again when the device's context has been replaced (cudaDeviceReset). All
 * calls share the one array and it keeps the last call's contents (the status word is cleared
 * at the start of each call): calls that can overlap on the GPU (different streams, or
 * different host threads) race on it and must be ordered by the caller. A wait that runs out
 * is recorded in that shared word, which lvb_gemm_noalloc_status reads (not the word
 * lvb_device_status reads). */
int lvb_gemm_noalloc(const lvb_gemm_desc* d, const void* A, const void* B, void* C,
                     void* stream);
/* Synchronise `stream`, then read and clear lvb_gemm_noalloc's status word on the current
 * device: *code is LVB_OK or LVB_ERR_TIMEOUT (a bounded wait inside the last noalloc call ran
 * out and C is incomplete), *where the wait site, *block the first CTA that gave up. Allocates
 * nothing. No counterpart in the reference (see lvb_gemm_noalloc). */
int lvb_gemm_noalloc_status(void* stream, int32_t* code, int32_t* where, int32_t* block);
/* Failure-path self-test of that word: lvb_selftest_wait_timeout recording into
 * lvb_gemm_noalloc's status word instead of lvb_device_status's. Allocates nothing. */
int lvb_gemm_noalloc_selftest_wait_timeout(int32_t timeout_ms, void* stream);

/* ---------------------------------------------------------------------------------------
 * Flash-attention forward: O = softmax(scale·Q·Kᵀ + mask)·V per (batch, query head), fp32
 * online softmax, P converted to the input type for the second product — the key-block
 * loop a Lava flash kernel writes with coopmat_muladd, coopmat_reduce(max/+, Row),
 * coopmat_perelement(exp) and coopmat_convert (src/device/coopmat_intrinsics.jl:520-755;
 * src/compiler/spirv/coopmat.jl:783-822,887-991). GQA: query head h reads KV head
 * h / (heads_q / heads_kv). Causal: query i sees keys j <= i + (seq_kv - seq_q).
 * Tensors are [batch][head][seq][head_dim] with head_dim contiguous — Lava's (E, L, H, B)
 * column-major arrays (src/device/sharedmemory.jl:73-76).
 * ------------------------------------------------------------------------------------- */
typedef struct lvb_attn_desc {
  int32_t dtype;      /* LVB_F16 or LVB_BF16 for Q, K, V and O */
  int32_t causal;
  int64_t batch, heads_q, heads_kv, seq_q, seq_kv, head_dim;
  float scale;        /* usually 1/sqrt(head_dim) */
  int32_t reserved;
  /* element strides of batch, head and seq; 0 for all three of a tensor = packed */
  int64_t q_stride[3], k_stride[3], v_stride[3], o_stride[3];
} lvb_attn_desc;

int lvb_attention_check(const lvb_attn_desc* d);

/* Which kernel lvb_attention_fwd runs for a descriptor (host only, no GPU). */
typedef enum lvb_attn_kernel {
  LVB_ATTN_FLASH = 0,   /* persistent CTAs, two 128-row query tiles per work item, keys
                           streamed in 128-key blocks */
  LVB_ATTN_DECODE = 1,  /* few query rows per KV head (group·seq_q <= 32, head_dim 128): the
                           KV cache streamed once, split over the keys, the splits merged
                           by a second kernel */
  LVB_ATTN_EMPTY = 2    /* seq_kv == 0: O = 0, lse = -inf */
} lvb_attn_kernel;

typedef struct lvb_attn_plan {
  int32_t kernel;     /* lvb_attn_kernel */
  int32_t splits;     /* key-range splits per (batch, KV head) (LVB_ATTN_DECODE), else 1 */
  int32_t ctas;       /* CTAs of the main kernel */
  int32_t launches;   /* kernel launches per call (0 when there is no output) */
} lvb_attn_plan;

int lvb_attention_plan_for(const lvb_attn_desc* d, int32_t sm_count, lvb_attn_plan* out);
/* Enqueue the forward pass. `lse` (nullable) receives the fp32 natural-log row
 * log-sum-exp of scale·QKᵀ, laid out [batch][heads_q][seq_q]. */
int lvb_attention_fwd(const lvb_attn_desc* d, const void* Q, const void* K, const void* V,
                      void* O, float* lse, void* stream);

/* ---------------------------------------------------------------------------------------
 * Sharding across the GPUs of one box. Lava has no multi-device code; the units of this
 * path are independent (GEMM output rows, attention (batch, kv-head) groups), so each rank
 * computes a contiguous range and no collective is needed on the data path. Host only.
 * ------------------------------------------------------------------------------------- */
/* Contiguous share of `total` units for `rank` of `world`: *begin, *count. Shares are made
 * of whole chunks of `align` units (the chunk counts of two ranks differ by at most one,
 * lower ranks take the extra ones); the ragged last chunk (total % align) falls in the last
 * non-empty share. */
int lvb_shard_range(int64_t total, int32_t world, int32_t rank, int64_t align, int64_t* begin,
                    int64_t* count);

/* Optional all-gather of the shards over NVLink/NVSwitch, for hosts without their own
 * collective library (Python hosts can use torch.distributed instead). One communicator per
 * process and GPU, NCCL underneath; NCCL (libnccl.so.2) is opened at first use, and its
 * absence is LVB_ERR_NCCL, not a load failure of this library. Lava has no counterpart: its
 * runtime is single-device. */
#define LVB_COMM_ID_BYTES 128
typedef struct lvb_comm_id {
  char bytes[LVB_COMM_ID_BYTES];
} lvb_comm_id;
typedef struct lvb_comm lvb_comm;
/* A new communicator id. Made once (by rank 0); the host hands the bytes to every rank. */
int lvb_comm_unique_id(lvb_comm_id* id);
/* Join communicator `id` as `rank` of `nranks` on the current device; every rank must call
 * it (it returns once all have joined). */
int lvb_comm_init(lvb_comm** comm, const lvb_comm_id* id, int32_t nranks, int32_t rank);
int lvb_comm_destroy(lvb_comm* comm);
int lvb_comm_size(const lvb_comm* comm, int32_t* nranks, int32_t* rank);
/* Enqueue on `stream`: recv[r·bytes .. (r+1)·bytes) = rank r's send[0 .. bytes) for every
 * rank r (rank order, equal sizes: pad a short last shard). `send` may be recv's own slot
 * (recv + rank·bytes). Every rank calls it with the same `bytes`, in the same order as its
 * other collectives. For row shards of a row-major output (lvb_shard_range with the GEMM's
 * 128-row alignment) the gathered bytes are the whole output. */
int lvb_allgather(lvb_comm* comm, const void* send, void* recv, size_t bytes, void* stream);

/* ---------------------------------------------------------------------------------------
 * Runtime helpers for host packages that own device buffers (Lava leaves these to its
 * runtime; LavaDeviceArray is a non-owning (ptr, dims) value, src/device/devicearray.jl:
 * 25-38).
 * ------------------------------------------------------------------------------------- */
int lvb_abi_version(void);
const char* lvb_last_error(void);
const char* lvb_status_string(int status);
int lvb_device_count(int32_t* n);
int lvb_set_device(int device);
int lvb_malloc(void** ptr, size_t bytes);
int lvb_free(void* ptr);
int lvb_memcpy_htod(void* dst, const void* src, size_t bytes, void* stream);
int lvb_memcpy_dtoh(void* dst, const void* src, size_t bytes, void* stream);
int lvb_stream_create(void** stream);
int lvb_stream_destroy(void* stream);
int lvb_stream_synchronize(void* stream);
/* Synchronise `stream`, then read and clear the current device's status word. *code is
 * LVB_OK or LVB_ERR_TIMEOUT; *where is the wait site, *block the first CTA that gave up. */
int lvb_device_status(void* stream, int32_t* code, int32_t* where, int32_t* block);
/* Wall-clock limit of every in-kernel wait, in milliseconds (default 2000; also read from
 * the environment variable LVB_WAIT_TIMEOUT_MS at first use). */
int lvb_set_wait_timeout_ms(int64_t ms);
/* Failure-path self-test: enqueue one CTA whose bounded mbarrier wait (the kind every kernel
 * uses) can never be satisfied and runs out after `timeout_ms` (1..2000). Afterwards
 * lvb_device_status reports LVB_ERR_TIMEOUT at wait site 99, and the context stays usable.
 * The reference's counterpart is the exception-flag path a throwing Lava kernel takes
 * (src/compiler/entry_wrapper.jl:199-216). */
int lvb_selftest_wait_timeout(int32_t timeout_ms, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* LVB_H */
