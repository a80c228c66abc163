// attn_decode_sm100.cu — attention forward for few query rows per KV head (decoding: seq_q of
// 1 to a few, GQA groups of up to 32 query heads), B200 (sm_100a).
//
// Same semantics as the flash kernel (O = softmax(scale·QKᵀ + mask)·V, fp32 online softmax,
// P rounded to the input type for the second product; src/device/coopmat_intrinsics.jl:
// 520-755), but the work has the opposite shape: a KV head is read by only group·seq_q query
// rows, so the kernel streams the KV cache once from HBM and is bound by its bandwidth. The
// products are turned around so the key block fills the tensor core's 128 rows:
//   Sᵀ (128 keys × NR rows) = K_j (128 × D) · Qᵀ,   Oᵀ (D × NR) += V_jᵀ · P_jᵀ
// with NR = 16 or 32 ≥ group·seq_q (the rows of one KV head's query heads and positions).
//   * work item = (batch, KV head, key range); a key range of a long cache is split so that
//     every SM streams; partial (O, max, sum) of the splits are merged by a second kernel
//     (flash-decoding); a single split writes O directly;
//   * persistent CTAs, 192 threads: warps 0-3 softmax and epilogue (thread = key of the block
//     for Sᵀ, = head-dim element for Oᵀ), warp 4 TMA (Q of the item, then K_j, V_j through a
//     6-slot ring, running ahead across items), warp 5 MMA (QK_j into one of two Sᵀ
//     buffers, then PV_{j-1}, so the next scores are ready while the softmax works);
//   * row max over the block's keys: warp shuffles, then the four warps through shared
//     memory; lazy rescale of Oᵀ (only when a row's max grows by more than 2^8);
//   * Pᵀ goes to shared memory (K-major, 128-byte swizzle) as the B operand of the second
//     product; Vᵀ is read MN-major straight from the V block.
#include <algorithm>
#include <cmath>
#include <cstdlib>

#include "lvb_internal.h"

namespace lvb {

namespace {

constexpr int kDecThreads = 192;
constexpr int kDecTmaWarp = 4;
constexpr int kDecMmaWarp = 5;
constexpr int kDecRing = 6;
constexpr int kDecD = 128;
constexpr int kDecChunk = 128 * 128;          // one 64-dim chunk of a 128-key block
constexpr int kDecBlockBytes = 128 * kDecD * 2;

struct DecParams {
  int B, Hq, Hkv, Sq, Skv, group, nrows, causal;
  int nsplit, bps, items;   // key blocks per split, work items = B·Hkv·nsplit
  float scale_log2;
  void* O;
  long long o_sb, o_sh, o_ss;
  float* lse;
  float* part;              // [items][NR][D] unnormalised O (nsplit > 1)
  float* part_ml;           // [items][NR][2] (max in log2 units, sum)
  DevStatus* status;
  unsigned long long timeout_ns;
};

template <int NR>
struct DecCfg {
  static constexpr int kQBytes = 2 * NR * 128;        // two 64-dim chunks of NR rows
  static constexpr int kPBytes = 2 * NR * 128;        // two 64-key chunks of NR rows
  static constexpr int kTmemCols = NR == 16 ? 64 : 128;
  static constexpr int kSmem = kDecRing * kDecBlockBytes + 2 * kQBytes + 2 * kPBytes + 2 * 4 * NR * 4 +
                               512 + 1024;
};

template <bool BF16>
__device__ __forceinline__ uint16_t to_bits16(float v) {
  if constexpr (BF16) return __bfloat16_as_ushort(__float2bfloat16_rn(v));
  else return __half_as_ushort(__float2half_rn(v));
}

__device__ __forceinline__ void dec_drain(uint64_t* bar, uint32_t parity, uint64_t timeout_ns) {
  const uint32_t a = smem_u32(bar);
  const uint64_t t0 = global_ns();
  while (!bar_try_wait(a, parity)) {
    if (global_ns() - t0 > timeout_ns) return;
  }
}

template <int NR>
__device__ __forceinline__ void tmem_ld_nr(uint32_t taddr, uint32_t (&r)[NR]) {
  if constexpr (NR == 1) tmem_ld1(taddr, r);
  else if constexpr (NR == 4) tmem_ld4(taddr, r);
  else if constexpr (NR == 8) tmem_ld8(taddr, r);
  else if constexpr (NR == 16) tmem_ld16(taddr, r);
  else tmem_ld32(taddr, r);
}

template <int NR>
__device__ __forceinline__ void tmem_st_nr(uint32_t taddr, uint32_t (&r)[NR]) {
  if constexpr (NR == 1) tmem_st1(taddr, r);
  else if constexpr (NR == 4) tmem_st4(taddr, r);
  else if constexpr (NR == 8) tmem_st8(taddr, r);
  else if constexpr (NR == 16) tmem_st16(taddr, r);
  else tmem_st32(taddr, r);
}

__device__ __forceinline__ void item_coords(int item, const DecParams& p, int& b, int& hk,
                                            int& kb0, int& kb1) {
  const int bh = item / p.nsplit;
  const int split = item - bh * p.nsplit;
  b = bh / p.Hkv;
  hk = bh - b * p.Hkv;
  const int nkb = (p.Skv + 127) / 128;
  kb0 = split * p.bps;
  kb1 = min(nkb, kb0 + p.bps);
}

// NR: the N of the products (16 or 32, the tensor core's minimum is 16 for 128 rows); RR <= NR:
// the rows the softmax works on (1, 4, 8, 16 or 32, the smallest that holds the query rows:
// the other columns of Sᵀ, Pᵀ and Oᵀ are computed but never read).
template <int NR, int RR, bool BF16>
__global__ void __launch_bounds__(kDecThreads, 1)
    attn_decode_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const DecParams p) {
  using Cfg = DecCfg<NR>;
  constexpr int R = kDecRing;
  constexpr uint32_t kFmt = BF16 ? 1 : 0;
  constexpr uint32_t kIdescQK = make_idesc(1, kFmt, kFmt, 0, 0, 128, NR);
  constexpr uint32_t kIdescPV = make_idesc(1, kFmt, kFmt, 1, 0, 128, NR);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_1024(smem_raw);
  uint8_t* sRing = smem;                                  // [R][2 chunks][128 keys][128 B]
  uint8_t* sQ = sRing + R * kDecBlockBytes;               // [2 bufs][2 chunks][NR rows][128 B]
  uint8_t* sP = sQ + 2 * Cfg::kQBytes;                    // [2 bufs][2 chunks][NR rows][128 B]
  float* sRed = reinterpret_cast<float*>(sP + 2 * Cfg::kPBytes);   // [2][4 warps][NR]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sRed + 2 * 4 * NR);
  uint64_t* kv_full = bars;              // [R]
  uint64_t* kv_empty = kv_full + R;      // [R]
  uint64_t* q_full = kv_empty + R;       // [2] Q buffers: item it uses buffer it & 1, so the
  uint64_t* q_empty = q_full + 2;        // [2] next item's Q loads while this one runs
  uint64_t* s_full = q_empty + 2;        // [2]
  uint64_t* s_empty = s_full + 2;        // [2] (128 arrivals)
  uint64_t* p_full = s_empty + 2;        // [2] (128 arrivals)
  uint64_t* p_empty = p_full + 2;        // [2] PV of that buffer done
  uint64_t* o_full = p_empty + 2;        // last PV of an item done
  uint64_t* o_empty = o_full + 1;        // epilogue read Oᵀ (128 arrivals)
  uint64_t* drain = o_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < R; ++s) {
      bar_init(&kv_full[s], 1);
      bar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      bar_init(&q_full[i], 1);
      bar_init(&q_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      bar_init(&s_full[i], 1);
      bar_init(&s_empty[i], 128);
      bar_init(&p_full[i], 128);
      bar_init(&p_empty[i], 1);
    }
    bar_init(o_full, 1);
    bar_init(o_empty, 128);
    bar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kDecMmaWarp) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem;                 // Sᵀ buffers: columns [0, NR) and [NR, 2NR)
  const uint32_t tO = tmem + 2 * NR;        // Oᵀ: columns [2NR, 3NR)
  const WaitGuard g{p.status, abort_flag, p.timeout_ns};

  if (warp == kDecTmaWarp) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      int n = 0;        // ring items issued (K_j and V_j are one item each)
      int it = 0;       // items of this CTA
      int q_loads = 0;  // Q tiles issued
      bool ok = true;
      for (int item = blockIdx.x; item < p.items && ok; item += gridDim.x, ++it) {
        int b, hk, kb0, kb1;
        item_coords(item, p, b, hk, kb0, kb1);
        // Q of the item once the previous item's last QK has read the old one.
        const int qb = it & 1;
        if (!wait_bar(&q_empty[qb], (uint32_t)((it >> 1) & 1) ^ 1, g, 51, item)) {
          ok = false;
          break;
        }
        bar_arrive_expect_tx(&q_full[qb], 2 * p.nrows * 128);   // the box holds the real rows
        for (int c = 0; c < 2; ++c)
          tma_load_4d(sQ + qb * Cfg::kQBytes + c * NR * 128, &tmQ, c * 64, 0, hk * p.group, b,
                      &q_full[qb]);
        ++q_loads;
        for (int kb = kb0; kb < kb1 && ok; ++kb) {
          for (int v = 0; v < 2; ++v, ++n) {
            const int slot = n % R;
            if (!wait_bar(&kv_empty[slot], (uint32_t)((n / R) & 1) ^ 1, g, 52, n)) {
              ok = false;
              break;
            }
            bar_arrive_expect_tx(&kv_full[slot], kDecBlockBytes);
            const CUtensorMap* tm = v ? &tmV : &tmK;
            for (int c = 0; c < 2; ++c)
              tma_load_4d(sRing + slot * kDecBlockBytes + c * kDecChunk, tm, c * 64, kb * 128,
                          hk, b, &kv_full[slot]);
          }
        }
      }
      if (!ok) {
        // Let the copies this thread started land before the CTA's shared memory goes away.
        for (int i = max(0, n - R); i < n; ++i)
          dec_drain(&kv_full[i % R], (uint32_t)((i / R) & 1), p.timeout_ns);
        for (int i = max(0, q_loads - 2); i < q_loads; ++i)
          dec_drain(&q_full[i & 1], (uint32_t)((i >> 1) & 1), p.timeout_ns);
      }
    }
  } else if (warp == kDecMmaWarp) {
    // ---------------- MMA issuer: the warp waits, one elected lane issues ----------------
    // Iteration j issues QK_j (into Sᵀ buffer g & 1, g = the block's index over this CTA's
    // items) and then PV_{j-1}, so block j's scores are computed while the softmax of block
    // j-1 runs. Ring item 2j is K_j, 2j+1 is V_j.
    const uint32_t r_base = smem_u32(sRing);
    const uint32_t q_base = smem_u32(sQ);
    const uint32_t p_base = smem_u32(sP);
    int n_ring = 0;   // ring items consumed before this item
    int gb = 0;       // blocks before this item
    int it = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < p.items && ok; item += gridDim.x, ++it) {
      int b, hk, kb0, kb1;
      item_coords(item, p, b, hk, kb0, kb1);
      const int nb = kb1 - kb0;   // >= 1: the planner makes no empty split
      const int qb = it & 1;
      if (!wait_bar_warp(&q_full[qb], (uint32_t)((it >> 1) & 1), g, 53, item)) { ok = false; break; }
      for (int j = 0; j <= nb && ok; ++j) {
        if (j < nb) {
          const int gj = gb + j;
          const int nk = n_ring + 2 * j;
          const int sk = nk % R;
          if (!wait_bar_warp(&kv_full[sk], (uint32_t)((nk / R) & 1), g, 54, nk)) { ok = false; break; }
          if (!wait_bar_warp(&s_empty[gj & 1], (uint32_t)((gj >> 1) & 1) ^ 1, g, 55, gj)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t o = (kk >> 2) * kDecChunk + (kk & 3) * 32;
            const uint64_t ad = sdesc_sw128(r_base + sk * kDecBlockBytes + o, 16, 1024);
            const uint64_t bd = sdesc_sw128(q_base + qb * Cfg::kQBytes + (kk >> 2) * NR * 128 +
                                                (kk & 3) * 32, 16, 1024);
            if (elect_one()) mma_f16_ss(tS + NR * (gj & 1), ad, bd, kIdescQK, kk > 0 ? 1u : 0u);
          }
          if (elect_one()) {
            mma_commit(&s_full[gj & 1]);
            mma_commit(&kv_empty[sk]);                   // K_j read
            if (j == nb - 1) mma_commit(&q_empty[qb]);   // the item's Q read for the last time
          }
        }
        if (j > 0) {
          const int gp = gb + j - 1;
          const int nv = n_ring + 2 * (j - 1) + 1;
          const int sv = nv % R;
          const int pb = gp & 1;
          if (!wait_bar_warp(&kv_full[sv], (uint32_t)((nv / R) & 1), g, 56, nv)) { ok = false; break; }
          if (!wait_bar_warp(&p_full[pb], (uint32_t)((gp >> 1) & 1), g, 57, gp)) { ok = false; break; }
          if (j == 1 && it > 0) {
            // Oᵀ of the previous item read by its epilogue before the first PV overwrites it.
            if (!wait_bar_warp(o_empty, (uint32_t)((it - 1) & 1), g, 58, item)) { ok = false; break; }
          }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {   // 16 keys per MMA
            const uint64_t ad = sdesc_sw128(r_base + sv * kDecBlockBytes + kk * 16 * 128, kDecChunk, 1024);
            const uint64_t bd = sdesc_sw128(p_base + pb * Cfg::kPBytes + (kk >> 2) * NR * 128 + (kk & 3) * 32, 16, 1024);
            if (elect_one()) mma_f16_ss(tO, ad, bd, kIdescPV, (j == 1 && kk == 0) ? 0u : 1u);
          }
          if (elect_one()) {
            mma_commit(&p_empty[pb]);
            mma_commit(&kv_empty[sv]);                   // V_{j-1} read
            if (j == nb) mma_commit(o_full);
          }
        }
      }
      n_ring += 2 * nb;
      gb += nb;
    }
    if (elect_one()) mma_commit(drain);
    dec_drain(drain, 0, p.timeout_ns);
  } else {
    // ---------------- softmax and epilogue: warps 0-3 ----------------
    // All four warps run every block and meet at named barrier 1 in the same order, also
    // after a wait gave up (then without waiting, on stale data), so none is left behind.
    const int t = (int)(warp * 32 + lane);              // key within the block / Oᵀ lane (d)
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const float NEG_INF = -INFINITY;
    const float sl = p.scale_log2;
    bool ok = true;
    int gb = 0;
    int it = 0;
    // Row r = (query head within the group) · seq_q + position; its last visible key.
    int last_key[RR];
#pragma unroll
    for (int r = 0; r < RR; ++r) {
      const int sq = r % max(p.Sq, 1);
      last_key[r] = r < p.nrows ? (p.causal ? sq + p.Skv - p.Sq : p.Skv - 1) : -1;
    }
    for (int item = blockIdx.x; item < p.items; item += gridDim.x, ++it) {
      int b, hk, kb0, kb1;
      item_coords(item, p, b, hk, kb0, kb1);
      const int nb = kb1 - kb0;
      float m_ref[RR], l_part[RR];
#pragma unroll
      for (int r = 0; r < RR; ++r) {
        m_ref[r] = NEG_INF;
        l_part[r] = 0.f;
      }
      for (int j = 0; j < nb; ++j, ++gb) {
        const int key = (kb0 + j) * 128 + t;
        if (!wait_bar(&s_full[gb & 1], (uint32_t)((gb >> 1) & 1), g, 61, gb)) ok = false;
        tc_fence_after();
        uint32_t sv[RR];
        tmem_ld_nr<RR>(tS + lane_off + NR * (gb & 1), sv);
        tmem_wait_ld();
        tc_fence_before();
        bar_arrive(&s_empty[gb & 1]);
        float x[RR];
#pragma unroll
        for (int r = 0; r < RR; ++r)
          x[r] = key <= last_key[r] ? __uint_as_float(sv[r]) * sl : NEG_INF;
        // Block max per row: within the warp, then across the four warps.
        float* red = sRed + (gb & 1) * 4 * NR;
#pragma unroll
        for (int r = 0; r < RR; ++r) {
          float v = x[r];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
          if (lane == 0) red[warp * NR + r] = v;
        }
        named_barrier_sync(1, 128);
        bool resc = false;
        float alpha[RR];
#pragma unroll
        for (int r = 0; r < RR; ++r) {
          const float bm = fmaxf(fmaxf(red[r], red[NR + r]), fmaxf(red[2 * NR + r], red[3 * NR + r]));
          alpha[r] = 1.f;
          if (bm > m_ref[r] + 8.f) {        // also the first block that sees a key (m_ref = -inf)
            if (m_ref[r] != NEG_INF) {
              alpha[r] = fast_exp2(m_ref[r] - bm);
              resc = true;
            }
            m_ref[r] = bm;
          }
        }
        if (resc && j > 0) {
          // Oᵀ holds PV up to block j-1: let it finish, then rescale its columns.
          if (!wait_bar(&p_empty[(gb - 1) & 1], (uint32_t)(((gb - 1) >> 1) & 1), g, 62, gb)) ok = false;
          tc_fence_after();
          uint32_t o[RR];
          tmem_ld_nr<RR>(tO + lane_off, o);
          tmem_wait_ld();
#pragma unroll
          for (int r = 0; r < RR; ++r) o[r] = __float_as_uint(__uint_as_float(o[r]) * alpha[r]);
          tmem_st_nr<RR>(tO + lane_off, o);
          tmem_wait_st();
        }
        // Pᵀ of this block into buffer gb & 1 once the PV of block gb - 2 has read it.
        if (!wait_bar(&p_empty[gb & 1], (uint32_t)((gb >> 1) & 1) ^ 1, g, 63, gb)) ok = false;
        uint8_t* pb = sP + (gb & 1) * Cfg::kPBytes + (t >> 6) * NR * 128;
        const int kin = t & 63;            // key within the 64-key chunk
#pragma unroll
        for (int r = 0; r < RR; ++r) {
          const float pr = (m_ref[r] == NEG_INF) ? 0.f : fast_exp2(x[r] - m_ref[r]);
          l_part[r] = l_part[r] * alpha[r] + pr;
          // K-major, 128-byte swizzle: 16-byte unit (kin / 8) of row r moves to (kin / 8) ^ (r % 8).
          const int unit = (kin >> 3) ^ (r & 7);
          *reinterpret_cast<uint16_t*>(pb + r * 128 + unit * 16 + (kin & 7) * 2) = to_bits16<BF16>(pr);
        }
        fence_proxy_async_smem();
        tc_fence_before();
        bar_arrive(&p_full[gb & 1]);
      }

      // ---------------- epilogue of the item ----------------
      if (nb > 0 && !wait_bar(o_full, (uint32_t)(it & 1), g, 64, item)) ok = false;
      tc_fence_after();
      uint32_t o[RR];
      if (nb > 0) {
        tmem_ld_nr<RR>(tO + lane_off, o);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int r = 0; r < RR; ++r) o[r] = 0u;
      }
      tc_fence_before();
      bar_arrive(o_empty);
      // Row sums over the 128 keys of every block: each thread holds its keys' share.
      float* red = sRed;      // both halves are free: the last block's barrier has passed
      named_barrier_sync(1, 128);
#pragma unroll
      for (int r = 0; r < RR; ++r) {
        float v = l_part[r];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        if (lane == 0) red[warp * NR + r] = v;
      }
      named_barrier_sync(1, 128);
#pragma unroll
      for (int r = 0; r < RR; ++r) {
        // after a wait gave up the values are stale: keep the barriers, store nothing
        if (r >= p.nrows || !ok) continue;
        const float l = (red[r] + red[NR + r]) + (red[2 * NR + r] + red[3 * NR + r]);
        const int hq = hk * p.group + r / p.Sq;
        const int sq = r % p.Sq;
        const float ov = __uint_as_float(o[r]);
        if (p.nsplit == 1) {
          const float inv = l > 0.f ? 1.f / l : 0.f;
          uint16_t* dst = reinterpret_cast<uint16_t*>(p.O) + (long long)b * p.o_sb +
                          (long long)hq * p.o_sh + (long long)sq * p.o_ss;
          dst[t] = to_bits16<BF16>(ov * inv);
          if (p.lse && t == 0)
            p.lse[((long long)b * p.Hq + hq) * p.Sq + sq] =
                l > 0.f ? (m_ref[r] + __log2f(l)) * 0.69314718055994530942f : NEG_INF;
        } else {
          p.part[((long long)item * NR + r) * kDecD + t] = ov;
          if (t == 0) {
            p.part_ml[((long long)item * NR + r) * 2 + 0] = m_ref[r];
            p.part_ml[((long long)item * NR + r) * 2 + 1] = l;
          }
        }
      }
      // The sums' slots are rewritten by the next item's first block only after barrier 1.
      named_barrier_sync(1, 128);
    }
  }

  tc_fence_before();
  __syncthreads();
  // This CTA has stored all it will: the merge kernel may be scheduled (it still waits for
  // the whole grid's results before reading them).
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (warp == kDecMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

constexpr int kMaxSplits = 1024;

// Merge the splits of one (batch, KV head) row: O = Σ 2^(m_s - m) O_s / Σ 2^(m_s - m) l_s,
// m = max m_s. One CTA per (batch·KV head, row), thread = head-dim element: the splits'
// (max, sum) pairs are read one per thread and reduced through shared memory, then every
// thread streams its column of the partial outputs with independent loads. Launched as a
// programmatic dependent of the decode kernel: it is scheduled while the decode kernel ends
// and waits (griddepcontrol.wait) for its results before reading them.
template <int NR, bool BF16>
__global__ void __launch_bounds__(kDecD) attn_decode_combine_kernel(const DecParams p) {
  __shared__ float w[kMaxSplits];
  __shared__ float red[kDecD / 32];
  __shared__ float bcast;
  const int bh = blockIdx.x;           // batch·Hkv + KV head
  const int r = blockIdx.y;            // row within the group
  const int t = threadIdx.x;           // head-dim element
  const int lane = t & 31, wp = t >> 5;
  const int b = bh / p.Hkv, hk = bh - b * p.Hkv;
  const long long item0 = (long long)bh * p.nsplit;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // the splits' maxima, one per thread (strided), reduced to m
  float mloc = -INFINITY;
  for (int s = t; s < p.nsplit; s += kDecD) {
    const float ms = p.part_ml[((item0 + s) * NR + r) * 2];
    w[s] = ms;
    mloc = fmaxf(mloc, ms);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, o));
  if (lane == 0) red[wp] = mloc;
  __syncthreads();
  if (t == 0) {
    float m = red[0];
    for (int i = 1; i < kDecD / 32; ++i) m = fmaxf(m, red[i]);
    bcast = m;
  }
  __syncthreads();
  const float m = bcast;
  // weights 2^(m_s - m) in shared memory, and the weighted sum of the splits' row sums
  float dloc = 0.f;
  for (int s = t; s < p.nsplit; s += kDecD) {
    const float ms = w[s];
    const float ws = (m == -INFINITY || ms == -INFINITY) ? 0.f : fast_exp2(ms - m);
    w[s] = ws;
    dloc += ws * p.part_ml[((item0 + s) * NR + r) * 2 + 1];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) dloc += __shfl_xor_sync(0xffffffffu, dloc, o);
  __syncthreads();   // every w[s] written; red reused
  if (lane == 0) red[wp] = dloc;
  __syncthreads();
  float den = 0.f;
#pragma unroll
  for (int i = 0; i < kDecD / 32; ++i) den += red[i];
  // the weighted partial outputs, in split order
  float num = 0.f;
  const float* col = p.part + (item0 * NR + r) * kDecD + t;
  const long long stride = (long long)NR * kDecD;
  int s = 0;
  for (; s + 4 <= p.nsplit; s += 4) {
    const float v0 = col[(s + 0) * stride], v1 = col[(s + 1) * stride];
    const float v2 = col[(s + 2) * stride], v3 = col[(s + 3) * stride];
    num += w[s] * v0;
    num += w[s + 1] * v1;
    num += w[s + 2] * v2;
    num += w[s + 3] * v3;
  }
  for (; s < p.nsplit; ++s) num += w[s] * col[s * stride];
  const int hq = hk * p.group + r / p.Sq;
  const int sq = r % p.Sq;
  uint16_t* dst = reinterpret_cast<uint16_t*>(p.O) + (long long)b * p.o_sb +
                  (long long)hq * p.o_sh + (long long)sq * p.o_ss;
  dst[t] = to_bits16<BF16>(den > 0.f ? num / den : 0.f);
  if (p.lse && t == 0)
    p.lse[((long long)b * p.Hq + hq) * p.Sq + sq] =
        den > 0.f ? (m + __log2f(den)) * 0.69314718055994530942f : -INFINITY;
}

template <int NR, int RR, bool BF16>
int launch_decode(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                  const DecParams& p, int ctas, cudaStream_t stream) {
  auto kern = attn_decode_kernel<NR, RR, BF16>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       DecCfg<NR>::kSmem);
  if (e != cudaSuccess) return fail_cuda(e, "lvb_attention_fwd", "cudaFuncSetAttribute (decode)");
  kern<<<ctas, kDecThreads, DecCfg<NR>::kSmem, stream>>>(tq, tk, tv, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail_cuda(e, "lvb_attention_fwd", "decode launch");
  if (p.nsplit > 1) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.B * p.Hkv, p.nrows);
    cfg.blockDim = dim3(kDecD);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, attn_decode_combine_kernel<NR, BF16>, p);
    if (e != cudaSuccess) return fail_cuda(e, "lvb_attention_fwd", "decode merge launch");
  }
  return LVB_OK;
}

}  // namespace

bool attn_decode_applies(const lvb_attn_desc* d) {
  return d->head_dim == kDecD && d->seq_kv > 0 && d->seq_q >= 1 &&
         (d->heads_q / d->heads_kv) * d->seq_q <= 32;
}

void attn_decode_plan(const lvb_attn_desc* d, int sm_count, int* nsplit, int* bps, int* ctas) {
  const long long bh = d->batch * d->heads_kv;
  const int nkb = (int)((d->seq_kv + 127) / 128);
  const int sms = std::max(1, sm_count);
  // Split the key blocks of each (batch, KV head) so that the work items spread evenly over
  // the persistent CTAs (one per SM): among 2-8 items per SM, the split count whose last
  // round of items is fullest; at least two key blocks per item.
  long long best_ns = 1;
  double best_eff = -1.0;
  const long long lo = std::max<long long>(1, (2LL * sms + bh - 1) / bh);
  const long long hi = std::max<long long>(lo, (8LL * sms + bh - 1) / bh);
  for (long long ns = lo; ns <= hi; ++ns) {
    const int b = (int)((nkb + ns - 1) / ns);
    if (ns > 1 && b < 2) break;
    const long long real_ns = (nkb + b - 1) / b;
    const long long items = bh * real_ns;
    const long long c = std::min<long long>(items, sms);
    const long long rounds = (items + c - 1) / c;
    const double eff = (double)items / (double)(rounds * c);
    if (eff > best_eff + 1e-9) { best_eff = eff; best_ns = real_ns; }
  }
  // LVB_DECODE_SPLITS=n forces the split count (tuning).
  static const int forced = [] {
    const char* e = std::getenv("LVB_DECODE_SPLITS");
    return e ? std::atoi(e) : 0;
  }();
  if (forced > 0) best_ns = std::min<long long>(forced, nkb);
  best_ns = std::min<long long>(best_ns, kMaxSplits);
  const int b = (int)((nkb + best_ns - 1) / best_ns);
  *nsplit = (int)((nkb + b - 1) / b);
  *bps = b;
  *ctas = (int)std::min<long long>(bh * *nsplit, (long long)sms);
}

int attn_decode_launch(const lvb_attn_desc* d, const long long qs[3], const long long ks[3],
                       const long long vs[3], const long long os[3], const void* Q, const void* K,
                       const void* V, void* O, float* lse, cudaStream_t stream, DeviceState* dev) {
  const char* op = "lvb_attention_fwd";
  const int group = (int)(d->heads_q / d->heads_kv);
  const int nrows = group * (int)d->seq_q;
  CUtensorMap tq, tk, tv;
  {
    const uint64_t dims[4] = {(uint64_t)d->head_dim, (uint64_t)d->seq_q, (uint64_t)d->heads_q,
                              (uint64_t)d->batch};
    const uint64_t str[3] = {(uint64_t)qs[2], (uint64_t)qs[1], (uint64_t)qs[0]};
    const uint32_t box[4] = {64, (uint32_t)d->seq_q, (uint32_t)group, 1};
    int st = make_tmap_nd(&tq, Q, 2, 4, dims, str, box, op);
    if (st) return st;
  }
  {
    const uint64_t dims[4] = {(uint64_t)d->head_dim, (uint64_t)d->seq_kv, (uint64_t)d->heads_kv,
                              (uint64_t)d->batch};
    const uint64_t strk[3] = {(uint64_t)ks[2], (uint64_t)ks[1], (uint64_t)ks[0]};
    const uint64_t strv[3] = {(uint64_t)vs[2], (uint64_t)vs[1], (uint64_t)vs[0]};
    const uint32_t box[4] = {64, 128, 1, 1};
    int st = make_tmap_nd(&tk, K, 2, 4, dims, strk, box, op);
    if (st) return st;
    st = make_tmap_nd(&tv, V, 2, 4, dims, strv, box, op);
    if (st) return st;
  }
  DecParams p = {};
  p.B = (int)d->batch;
  p.Hq = (int)d->heads_q;
  p.Hkv = (int)d->heads_kv;
  p.Sq = (int)d->seq_q;
  p.Skv = (int)d->seq_kv;
  p.group = group;
  p.nrows = nrows;
  p.causal = d->causal ? 1 : 0;
  int ctas;
  attn_decode_plan(d, dev->sm_count, &p.nsplit, &p.bps, &ctas);
  p.items = p.B * p.Hkv * p.nsplit;
  p.scale_log2 = d->scale * 1.4426950408889634f;
  p.O = O;
  p.o_sb = os[0];
  p.o_sh = os[1];
  p.o_ss = os[2];
  p.lse = lse;
  p.status = dev->status;
  p.timeout_ns = wait_timeout_ns();
  const int NR = nrows <= 16 ? 16 : 32;
  void* ws = nullptr;
  if (p.nsplit > 1) {
    const size_t bytes = (size_t)p.items * NR * (kDecD + 2) * sizeof(float);
    cudaError_t e = workspace_alloc(dev, &ws, bytes, stream);
    if (e != cudaSuccess) return fail_cuda(e, op, "decode workspace allocation");
    p.part = reinterpret_cast<float*>(ws);
    p.part_ml = p.part + (size_t)p.items * NR * kDecD;
  }
  const bool bf16 = d->dtype == LVB_BF16;
  int st;
  if (nrows == 1)
    st = bf16 ? launch_decode<16, 1, true>(tq, tk, tv, p, ctas, stream)
              : launch_decode<16, 1, false>(tq, tk, tv, p, ctas, stream);
  else if (nrows <= 4)
    st = bf16 ? launch_decode<16, 4, true>(tq, tk, tv, p, ctas, stream)
              : launch_decode<16, 4, false>(tq, tk, tv, p, ctas, stream);
  else if (nrows <= 8)
    st = bf16 ? launch_decode<16, 8, true>(tq, tk, tv, p, ctas, stream)
              : launch_decode<16, 8, false>(tq, tk, tv, p, ctas, stream);
  else if (NR == 16)
    st = bf16 ? launch_decode<16, 16, true>(tq, tk, tv, p, ctas, stream)
              : launch_decode<16, 16, false>(tq, tk, tv, p, ctas, stream);
  else
    st = bf16 ? launch_decode<32, 32, true>(tq, tk, tv, p, ctas, stream)
              : launch_decode<32, 32, false>(tq, tk, tv, p, ctas, stream);
  if (ws) {
    cudaError_t e = cudaFreeAsync(ws, stream);
    if (st == LVB_OK && e != cudaSuccess) return fail_cuda(e, op, "decode workspace free");
  }
  return st;
}

}  // namespace lvb
