// attn_sm100.cu — causal / GQA flash-attention forward for B200 (sm_100a).
//
// What it computes is the key-block loop a Lava flash kernel writes with the coopmat
// vocabulary: S = Q·Kᵀ (coopmat_muladd, K read through a transposing view), row max
// (coopmat_reduce(max, Row), result smeared along the row), P = exp(S - m)
// (coopmat_perelement), row sum (coopmat_reduce(+, Row)), P converted fp32 -> fp16/bf16 and
// from accumulator to MatrixA use (coopmat_convert), O = P·V + rescaled O
// (src/device/coopmat_intrinsics.jl:520-755; src/compiler/spirv/coopmat.jl:783-822,887-991),
// then O / l stored through a clamped layout.
//
// How, per CTA = two 128-row query tiles of one (batch, query head):
//   * TMEM: S | P_0 | P_1 | O_0 | O_1 = 128 + 64 + 64 + 128 + 128 = 512 columns. One S buffer
//     serves both tiles in turn: a softmax warpgroup copies its S into registers and frees
//     the buffer at once, so the other tile's Q·Kᵀ runs while this tile's softmax works. P_t
//     (16-bit pairs, 64 columns) has its own columns, and the P·V product takes P straight
//     from TMEM (tcgen05.mma with the A operand in TMEM), so P never touches shared memory;
//   * warp 10 lane 0 (TMA): both Q tiles once, then the K/V blocks through a 5-slot ring of
//     128-key blocks in the order the products release them, K_0, K_1, V_0, K_2, V_1, ...
//     (128B swizzle, zero fill past seq_kv);
//   * warps 0 and 1 (MMA issuers; each warp waits, an elected lane issues): warp 0 runs the
//     Q·Kᵀ products into the S buffer in the order S_0(0), S_1(0), S_0(1), S_1(1), ..., each
//     once the previous S has been copied out; warp 1 runs the P·V products, each once its
//     tile's P is stored. A softmax warpgroup stores P_t(j), copies S_t(j+1) out and only
//     then announces both, so the other tile's next Q·Kᵀ (which that softmax waits for)
//     goes to the tensor core first and this P·V (needed only at this tile's next P store)
//     after it. The two softmax warpgroups run side by side, half a block apart;
//   * warps 2-5 / 6-9 (softmax, one warpgroup per tile; each covers the four TMEM lane
//     quarters, warp % 4): thread = query row, the whole 128-key row sits in registers, so
//     max and sum need no shuffles; exp2 in the log2 domain with the scale folded in; the O
//     rescale is lazy (only when the running max grows by more than 2^8, which keeps every
//     p <= 256) and done in TMEM by the same warp after the tile's previous P·V has finished
//     (which also frees P_t);
//   * persistent: one CTA per SM takes (head, query-tile pair) items from a global counter,
//     head by head and the heaviest causal pair of a head first, so the items in flight
//     share a few heads' K/V blocks in L2; the TMA warp publishes the next item through a
//     shared-memory queue and loads its Q and first K/V blocks while the current item ends.
#include <algorithm>
#include <cmath>

#include "lvb_internal.h"

namespace lvb {

constexpr int kAttnThreads = 352;
// Warp roles: the two MMA issuers, the TMA producer; warps 2-9 are the softmax warpgroups.
constexpr int kQkWarp = 0, kPvWarp = 1, kTmaWarp = 10;
constexpr int kChunk = 128 * 128;       // bytes of one 128-row x 64-element swizzled chunk

struct AttnParams {
  int B, Hq, Hkv, Sq, Skv, group, num_pairs, causal;
  int total_items;             // num_pairs · B · Hq work items
  int tail_heads;              // the last heads' items are handed out heaviest first
  int* work_counter;           // zero at launch; items are taken from it in order
  float scale_log2;
  void* O;
  long long o_sb, o_sh, o_ss;  // element strides of batch, head, seq
  float* lse;
  DevStatus* status;
  unsigned long long timeout_ns;
};

template <int D>
struct AttnCfg {
  static constexpr int kTileBytes = 128 * D * 2;  // Q tile or K/V block
  static constexpr int kQBytes = 2 * kTileBytes;
  static constexpr int kRing = D == 128 ? 5 : 8;
  static constexpr int kSmem = kQBytes + kRing * kTileBytes + 512 + 1024;   // + barriers
};

__device__ __forceinline__ void drain_wait_a(uint64_t* bar, uint32_t parity, uint64_t timeout_ns) {
  const uint32_t a = smem_u32(bar);
  const uint64_t t0 = global_ns();
  while (!bar_try_wait(a, parity)) {
    if (global_ns() - t0 > timeout_ns) return;
  }
}

// Ring order of an item's K/V blocks: K_0, K_1, V_0, K_2, V_1, ..., K_{nb-1}, V_{nb-2},
// V_{nb-1} — the order in which the products release them (K_{j+1} with the second tile's
// Q·Kᵀ, V_j with its P·V, half a block later), so each load has about two blocks of slack.
__device__ __forceinline__ int ring_k(int j) { return j == 0 ? 0 : 2 * j - 1; }
__device__ __forceinline__ int ring_v(int j, int nb) { return j + 1 < nb ? 2 * j + 2 : 2 * j + 1; }

// An issuer's wait: a non-blocking test first (a completed phase is the common case and
// mbarrier.try_wait costs far more even then), the bounded suspending wait otherwise.
__device__ __forceinline__ bool issuer_wait(uint64_t* bar, uint32_t parity, const WaitGuard& g,
                                            int where, int detail) {
  bool ok = bar_test_wait(smem_u32(bar), parity);
  if (!__all_sync(0xffffffffu, ok)) ok = wait_bar_warp(bar, parity, g, where, detail);
  return ok;
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (BF16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

// Geometry of one work item = (batch·head, pair of 128-row query tiles). Items are numbered
// head by head, the heaviest causal pair of a head first, and handed out in that order, so
// the CTAs running at any moment work on a few heads and share their K/V blocks in L2. The
// items of the last `tail_heads` heads (about two waves of items) are numbered heaviest pair
// first across those heads instead: the last items taken are then the lightest, and the CTAs
// finish together (longest-first), while those heads' K/V still fit in L2.
struct AttnItem {
  int b, h, hk, q0, n_tile0, n_tile1, n_blocks;
};

__device__ __forceinline__ AttnItem attn_item(int item, const AttnParams& p) {
  AttnItem it;
  const int tail_start = p.total_items - p.tail_heads * p.num_pairs;
  int bh, pair;
  if (item >= tail_start) {
    const int j = item - tail_start;
    bh = p.B * p.Hq - p.tail_heads + j % p.tail_heads;
    pair = p.num_pairs - 1 - j / p.tail_heads;
  } else {
    bh = item / p.num_pairs;
    pair = p.num_pairs - 1 - (item - bh * p.num_pairs);
  }
  it.b = bh / p.Hq;
  it.h = bh - it.b * p.Hq;
  it.hk = it.h / p.group;
  it.q0 = pair * 256;
  const int off = p.Skv - p.Sq;  // query q sees keys <= q + off
  const int kv_blocks = (p.Skv + 127) / 128;
  // Key blocks per query tile: under the causal mask tile 0 stops one block earlier than
  // tile 1 whenever its last row's keys end before tile 1's; n_blocks = max over the tiles.
  it.n_tile0 = kv_blocks;
  it.n_tile1 = kv_blocks;
  if (p.causal) {
    const int last0 = min(it.q0 + 127, p.Sq - 1) + off;
    const int last1 = min(it.q0 + 255, p.Sq - 1) + off;
    it.n_tile0 = last0 < 0 ? 0 : min(kv_blocks, last0 / 128 + 1);
    it.n_tile1 = last1 < 0 ? 0 : min(kv_blocks, last1 / 128 + 1);
  }
  it.n_blocks = max(it.n_tile0, it.n_tile1);
  return it;
}

// 11 warps: three share a scheduler on three of the four sub-partitions (16,384 registers
// each), which caps a thread at 168 registers; the softmax threads keep a 128-key score row
// in registers within that. Two issuer warps instead of one: an issuing thread cannot run
// ahead of the tensor core by more than a few MMAs, and a wait costs a warp a few hundred
// cycles even when the barrier is already complete, so with one warp the tensor core idled
// through every wait; with two, one warp's products run while the other waits.
//
// Persistent: one CTA per SM takes items from a global counter until they run out. The TMA
// warp takes the next item as soon as it has issued the current one's loads and publishes it
// through a small shared-memory queue; so the next item's Q and first K/V blocks load while
// the current item's last blocks and its epilogue run, and its first products start as soon
// as the tensor core is free.
template <int D, bool BF16>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  using Cfg = AttnCfg<D>;
  constexpr int R = Cfg::kRing;
  constexpr int kDChunks = D / 64;
  constexpr int kSched = 4;
  constexpr uint32_t kFmt = BF16 ? 1 : 0;
  constexpr uint32_t kIdescQK = make_idesc(1, kFmt, kFmt, 0, 0, 128, 128);
  constexpr uint32_t kIdescPV = make_idesc(1, kFmt, kFmt, 0, 1, 128, D);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_1024(smem_raw);
  uint8_t* sQ = smem;                                   // [2][D/64 chunks][128 rows][128 B]
  uint8_t* sRing = sQ + Cfg::kQBytes;                   // [R][D/64 chunks][128 rows][128 B]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sRing + R * Cfg::kTileBytes);
  uint64_t* q_full = bars;
  uint64_t* q_empty = q_full + 1;          // the item's last QK read Q
  uint64_t* ring_full = q_empty + 1;       // [R]
  uint64_t* ring_empty = ring_full + R;    // [R]
  uint64_t* s_full = ring_empty + R;       // [2] QK_t done: the S buffer holds tile t's S
  uint64_t* s_free = s_full + 2;           // the S buffer's owner copied it out (4 warps)
  uint64_t* p_full = s_free + 1;           // [2] softmax_t wrote P_t (4 warps)
  uint64_t* pv_done = p_full + 2;          // [2] PV_t done
  uint64_t* sched_full = pv_done + 2;      // [kSched] item index published
  uint64_t* sched_empty = sched_full + kSched;   // [kSched] read by 2 MMA warps, 8 softmax warps
  uint64_t* drain = sched_empty + kSched;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* sched_item = reinterpret_cast<volatile int*>(tmem_slot + 2);   // [kSched]
  // qk_after[t]: Q·Kᵀ products issued right after a copy-out of tile t's S (the P·V warp
  // lets those go first).
  volatile int* qk_after = sched_item + kSched;                                 // [2]

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();

  if (threadIdx.x == 0) {
    bar_init(q_full, 1);
    bar_init(q_empty, 1);
    for (int s = 0; s < R; ++s) {
      bar_init(&ring_full[s], 1);
      bar_init(&ring_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      bar_init(&s_full[t], 1);
      bar_init(&p_full[t], 4);
      bar_init(&pv_done[t], 1);
    }
    bar_init(s_free, 4);
    for (int s = 0; s < kSched; ++s) {
      bar_init(&sched_full[s], 1);
      bar_init(&sched_empty[s], 10);
    }
    bar_init(drain, 2);
    *abort_flag = 0;
    qk_after[0] = 0;
    qk_after[1] = 0;
    fence_barrier_init();
  }
  if (warp == kQkWarp) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const WaitGuard g{p.status, abort_flag, p.timeout_ns};

  if (warp == kTmaWarp) {
    if (lane == 0) {
      // ---------------- scheduler + TMA producer ----------------
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      int rn = 0;      // ring items issued
      int qi = 0;      // Q tiles issued
      bool ok = true;
      for (int k = 0; ok; ++k) {
        const int slot = k % kSched;
        if (!wait_bar(&sched_empty[slot], (uint32_t)((k / kSched) & 1) ^ 1, g, 10, k)) {
          ok = false;
          break;
        }
        const int item = atomicAdd(p.work_counter, 1);
        sched_item[slot] = item;
        bar_arrive(&sched_full[slot]);            // release: the index is visible to waiters
        if (item >= p.total_items) break;         // the end marker is published too
        const AttnItem it = attn_item(item, p);
        if (it.n_blocks == 0) continue;
        // Q of this item once the previous item's last QK has read the old one.
        if (!wait_bar(q_empty, (uint32_t)(qi & 1) ^ 1, g, 11, item)) { ok = false; break; }
        bar_arrive_expect_tx(q_full, Cfg::kQBytes);
        for (int t = 0; t < 2; ++t)
          for (int c = 0; c < kDChunks; ++c)
            tma_load_4d(sQ + t * Cfg::kTileBytes + c * kChunk, &tmQ, c * 64, it.q0 + 128 * t,
                        it.h, it.b, q_full);
        ++qi;
        for (int i = 0; i < 2 * it.n_blocks; ++i, ++rn) {
          const int s = rn % R;
          if (!wait_bar(&ring_empty[s], (uint32_t)((rn / R) & 1) ^ 1, g, 12, rn)) {
            ok = false;
            break;
          }
          bar_arrive_expect_tx(&ring_full[s], Cfg::kTileBytes);
          // Item i of the ring order: K_0; odd i: K_{(i+1)/2}, or V_{nb-1} for the last;
          // even i > 0: V_{i/2 - 1}.
          bool is_k;
          int blk;
          if (i == 0) {
            is_k = true;
            blk = 0;
          } else if (i & 1) {
            blk = (i + 1) >> 1;
            is_k = blk < it.n_blocks;
            if (!is_k) blk = it.n_blocks - 1;
          } else {
            is_k = false;
            blk = (i >> 1) - 1;
          }
          const CUtensorMap* tm = is_k ? &tmK : &tmV;
          for (int c = 0; c < kDChunks; ++c)
            tma_load_4d(sRing + s * Cfg::kTileBytes + c * kChunk, tm, c * 64, blk * 128, it.hk,
                        it.b, &ring_full[s]);
        }
      }
      if (!ok) {
        // Let every copy this thread started land before the CTA's shared memory goes away.
        if (qi > 0) drain_wait_a(q_full, (uint32_t)((qi - 1) & 1), p.timeout_ns);
        for (int i = max(0, rn - R); i < rn; ++i)
          drain_wait_a(&ring_full[i % R], (uint32_t)((i / R) & 1), p.timeout_ns);
      }
    }
  } else if (warp == kQkWarp || warp == kPvWarp) {
    // ---------------- MMA issuers: one warp the Q·Kᵀ products, one the P·V products ----
    // The two touch disjoint TMEM columns (S at 0; P_t at 128 + 64t and O_t at 256 + 128t)
    // and disjoint ring slots (K / V blocks), so while one waits for its next operand the
    // other's products keep the tensor core busy (an issuing thread cannot run ahead of the
    // tensor core by much). In each warp the whole warp waits and one elected lane issues a
    // whole product and its commits, with the shared-memory descriptors precomputed and
    // advanced in their 16-byte address field.
    const bool qk_role = warp == kQkWarp;
    const uint32_t q_base = smem_u32(sQ);
    const uint32_t r_base = smem_u32(sRing);
    const uint64_t qd0 = sdesc_sw128(q_base, 16, 1024);
    const uint64_t kd0 = sdesc_sw128(r_base, 16, 1024);
    const uint64_t vd0 = sdesc_sw128(r_base, kChunk, 1024);
    constexpr uint32_t kTile16 = Cfg::kTileBytes >> 4;
    int rc = 0;               // ring items of the items before the current one
    int qi = 0;               // items with work before the current one
    int gt[2] = {0, 0};       // blocks of each tile before the current item
    int fills = 0;            // Q·Kᵀ products written to the S buffer so far
    int prev_tile = 0;        // tile of the last S written
    int after[2] = {0, 0};    // copy of qk_after (written by the Q·Kᵀ warp only)
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int sslot = k % kSched;
      if (!wait_bar_warp(&sched_full[sslot], (uint32_t)((k / kSched) & 1), g, 19, k)) break;
      const int item = sched_item[sslot];
      __syncwarp();
      if (elect_one()) bar_arrive(&sched_empty[sslot]);
      if (item >= p.total_items) break;
      const AttnItem it = attn_item(item, p);
      if (it.n_blocks == 0) continue;
      const int nt[2] = {it.n_tile0, it.n_tile1};
      const int nb = it.n_blocks;
      // Ring item i of this item (ring_k / ring_v); each warp waits for its items in
      // increasing order, once each (a slot is refilled only after its release).
      int ring_seen = -1;     // this warp's ring items of the item already waited for
      auto ring_wait = [&](int i, int where) -> bool {
        if (i <= ring_seen) return true;
        const int x = rc + i;
        if (!issuer_wait(&ring_full[x % R], (uint32_t)((x / R) & 1), g, where, i)) return false;
        ring_seen = i;
        return true;
      };
      auto release = [&](int i) {
        if (elect_one()) mma_commit(&ring_empty[(rc + i) % R]);
        __syncwarp();
      };
      if (qk_role) {
        if (!wait_bar_warp(q_full, (uint32_t)(qi & 1), g, 12, item)) break;
        const int n_qk = nt[0] + nt[1];
        int qk_done = 0;
        // Q·Kᵀ of tile t for key block j into the S buffer, once the previous S is copied
        // out; the commit on q_empty after the item's last one releases Q.
        auto fill = [&](int t, int j) -> bool {
          if (!ring_wait(ring_k(j), 13)) return false;
          if (fills > 0 && !issuer_wait(s_free, (uint32_t)((fills - 1) & 1), g, 17, j))
            return false;
          tc_fence_after();
          const bool last = ++qk_done == n_qk;
          if (elect_one()) {
            const uint64_t ad = qd0 + (uint64_t)(t * kTile16);
            const uint64_t bd = kd0 + (uint64_t)(((rc + ring_k(j)) % R) * kTile16);
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t o = ((kk >> 2) * kChunk + (kk & 3) * 32) >> 4;
              mma_f16_ss(tmem, ad + o, bd + o, kIdescQK, kk > 0 ? 1u : 0u);
            }
            mma_commit(&s_full[t]);
            if (last) mma_commit(q_empty);
          }
          __syncwarp();
          if (fills > 0) {
            ++after[prev_tile];
            if (lane == 0) qk_after[prev_tile] = after[prev_tile];
          }
          prev_tile = t;
          ++fills;
          return true;
        };
        // Fill order S_0(0), S_1(0), S_0(1), S_1(1), ...: each softmax warpgroup copies its
        // next S out when it has finished a block (the first at the item's start), so each
        // Q·Kᵀ runs while the other tile's softmax works.
        if (nt[0] > 0) ok = fill(0, 0);
        if (ok && nt[1] > 0) ok = fill(1, 0);
        if (ok && nt[0] > 1) ok = fill(0, 1);
        if (!ok) break;
        release(0);                                              // K_0
        for (int j = 0; j < nb && ok; ++j) {
          if (j + 1 < nt[1]) ok = fill(1, j + 1);
          if (ok && j + 2 < nt[0]) ok = fill(0, j + 2);
          if (!ok) break;
          if (j + 1 < nb) release(ring_k(j + 1));                // K_{j+1}: last use
        }
      } else {
        for (int j = 0; j < nb && ok; ++j) {
          if (!ring_wait(ring_v(j, nb), 14)) { ok = false; break; }
          for (int t = 0; t < 2; ++t) {
            if (j >= nt[t]) continue;
            if (!issuer_wait(&p_full[t], (uint32_t)((gt[t] + j) & 1), g, 15, j)) {
              ok = false;
              break;
            }
            // P_t(j) was announced together with the copy-out of S_t(j+1), which lets the
            // other tile's next Q·Kᵀ into the S buffer; that product is on the critical path
            // (the other softmax waits for it), this P·V is not (it is needed at this tile's
            // next P store), so let the Q·Kᵀ reach the tensor core first. A priority hint
            // only: after ~2 us the P·V goes anyway.
            if (j + 1 < nt[t] && !(t == 1 && j + 2 == nt[1] && nt[1] >= nt[0])) {
              const int target = gt[t] + j + 2;
              if (qk_after[t] < target) {
                const uint64_t t0 = global_ns();
                while (qk_after[t] < target && global_ns() - t0 < 2000) {
                }
              }
              __syncwarp();
            }
            tc_fence_after();
            if (elect_one()) {
              // V block: rows are keys (128 B = 64 head-dim elements each), chunks of 64
              // dims kChunk bytes apart: MN-major, SBO = 8 key rows, LBO = next 64-dim chunk.
              const uint64_t bd = vd0 + (uint64_t)(((rc + ring_v(j, nb)) % R) * kTile16);
              const uint32_t tp = tmem + 128 + 64 * t;
#pragma unroll
              for (int kk = 0; kk < 8; ++kk)   // 128 keys, 16 per MMA: P columns 8kk..8kk+7
                mma_f16_ts(tmem + 256 + 128 * t, tp + 8 * kk, bd + (uint64_t)(kk * 128),
                           kIdescPV, (j > 0 || kk > 0) ? 1u : 0u);
              mma_commit(&pv_done[t]);
            }
            __syncwarp();
          }
          if (!ok) break;
          release(ring_v(j, nb));                                // V_j
        }
      }
      rc += 2 * nb;
      gt[0] += nt[0];
      gt[1] += nt[1];
      ++qi;
    }
    if (elect_one()) mma_commit(drain);
    drain_wait_a(drain, 0, p.timeout_ns);
  } else {
    // ---------------- softmax, one warpgroup per query tile ----------------
    const int t = (warp - 2) >> 2;
    const int wl = warp & 3;
    const int r = wl * 32 + lane;               // row within the tile = TMEM lane
    const uint32_t lane_off = (uint32_t)(wl * 32) << 16;
    const uint32_t tS = tmem + lane_off;                  // the S buffer (shared)
    const uint32_t tP = tmem + lane_off + 128 + 64 * t;   // P_t
    const uint32_t tO = tmem + lane_off + 256 + 128 * t;
    const float NEG_INF = -INFINITY;
    const int off = p.Skv - p.Sq;
    int gt = 0;               // blocks of this tile before the current item
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int sslot = k % kSched;
      if (!wait_bar(&sched_full[sslot], (uint32_t)((k / kSched) & 1), g, 20, k)) break;
      const int item = sched_item[sslot];
      __syncwarp();
      if (lane == 0) bar_arrive(&sched_empty[sslot]);
      if (item >= p.total_items) break;
      const AttnItem it = attn_item(item, p);
      const int b = it.b, h = it.h;
      const int q = it.q0 + 128 * t + r;          // query index
      float m_ref = NEG_INF;   // running max (log2 domain, scale folded in)
      float l = 0.f;           // running sum of p relative to m_ref
      const int tile_first_row = it.q0 + 128 * t;
      const int nt = it.n_blocks == 0 ? 0 : (t ? it.n_tile1 : it.n_tile0);

      // S_t(j) is copied into registers right after P_t(j-1) is stored, and only then are
      // both announced: the Q·Kᵀ warp then writes the next S (usually the other tile's) into
      // the freed buffer, and the P·V warp lets that product go before this tile's P·V.
      for (int j = 0; j < nt; ++j) {
        if (!wait_bar_warp(&s_full[t], (uint32_t)((gt + j) & 1), g, 21, j)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t s[128];
        tmem_ld32(tS + 0, *reinterpret_cast<uint32_t (*)[32]>(&s[0]));
        tmem_ld32(tS + 32, *reinterpret_cast<uint32_t (*)[32]>(&s[32]));
        tmem_ld32(tS + 64, *reinterpret_cast<uint32_t (*)[32]>(&s[64]));
        tmem_ld32(tS + 96, *reinterpret_cast<uint32_t (*)[32]>(&s[96]));
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (j > 0) bar_arrive(&p_full[t]);
          bar_arrive(s_free);
        }
        const int kbase = j * 128;
        const bool need_mask =
            (kbase + 127 >= p.Skv) || (p.causal && kbase + 127 > tile_first_row + off);
        if (need_mask) {
          const int lim = p.causal ? min(q + off, p.Skv - 1) : p.Skv - 1;
#pragma unroll
          for (int c = 0; c < 128; ++c)
            if (kbase + c > lim) s[c] = __float_as_uint(NEG_INF);
        }
        const float sl = p.scale_log2;
        // Row max: 4 independent chains of 3-input maxima.
        float mxp[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) mxp[i] = __uint_as_float(s[i]);
#pragma unroll
        for (int c = 4; c < 124; c += 8)
#pragma unroll
          for (int i = 0; i < 4; ++i)
            mxp[i] = fmax3(mxp[i], __uint_as_float(s[c + i]), __uint_as_float(s[c + 4 + i]));
#pragma unroll
        for (int i = 0; i < 4; ++i) mxp[i] = fmaxf(mxp[i], __uint_as_float(s[124 + i]));
        const float m_new = fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3])) * sl;
        float alpha = 1.f;
        bool resc = false;
        if (j == 0) {
          m_ref = m_new;
        } else if (m_new > m_ref + 8.f) {
          alpha = fast_exp2(m_ref - m_new);
          m_ref = m_new;
          resc = true;
        }
        // p = 2^(s·scale·log2e - m) for the row, packed pairwise in place over s[0..63]
        // (4 independent sum chains).
        const float m_use = m_ref == NEG_INF ? 0.f : m_ref;
        float sump[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const float p0 = fast_exp2(fmaf(__uint_as_float(s[2 * c]), sl, -m_use));
          const float p1 = fast_exp2(fmaf(__uint_as_float(s[2 * c + 1]), sl, -m_use));
          sump[c & 3] += p0 + p1;
          s[c] = pack2<BF16>(p0, p1);
        }
        const float sum = (sump[0] + sump[1]) + (sump[2] + sump[3]);
        // PV_t(j-1) has finished: P_t may be rewritten and O_t rescaled.
        if (j > 0) {
          if (!wait_bar_warp(&pv_done[t], (uint32_t)((gt + j - 1) & 1), g, 22, j)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (__any_sync(0xffffffffu, resc)) {
#pragma unroll 1
            for (int c = 0; c < D / 16; ++c) {
              uint32_t o[16];
              tmem_ld16(tO + 16 * c, o);
              tmem_wait_ld();
#pragma unroll
              for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
              tmem_st16(tO + 16 * c, o);
            }
          }
        }
        tmem_st32(tP + 0, &s[0]);
        tmem_st32(tP + 32, &s[32]);
        tmem_wait_st();
        l = l * alpha + sum;
        tc_fence_before();
      }
      if (!ok) break;
      if (nt > 0) {
        __syncwarp();
        if (lane == 0) bar_arrive(&p_full[t]);    // the last block's P
      }

      // ---------------- epilogue: O / l -> global, lse ----------------
      // O_t is rewritten by the next item's first P·V only after this warpgroup has
      // produced that item's first P, i.e. after these loads have completed.
      if (nt > 0 && !wait_bar_warp(&pv_done[t], (uint32_t)((gt + nt - 1) & 1), g, 23, 0)) break;
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const bool row_ok = q < p.Sq;
      uint8_t* orow = reinterpret_cast<uint8_t*>(p.O) +
                      2 * ((long long)b * p.o_sb + (long long)h * p.o_sh + (long long)q * p.o_ss);
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        if (nt > 0) {
          tmem_ld32(tO + 32 * c, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = 0u;
        }
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e)
          pk[e] = pack2<BF16>(__uint_as_float(o[2 * e]) * inv, __uint_as_float(o[2 * e + 1]) * inv);
        if (row_ok) {
          uint8_t* dst = orow + c * 64;
          if ((reinterpret_cast<uintptr_t>(dst) & 31) == 0) {
            // 32-byte stores: each lane's store fills a whole 32-byte sector of its row.
            st_global_v8(dst, &pk[0]);
            st_global_v8(dst + 32, &pk[8]);
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e)
              reinterpret_cast<uint4*>(dst)[e] =
                  make_uint4(pk[4 * e], pk[4 * e + 1], pk[4 * e + 2], pk[4 * e + 3]);
          }
        }
      }
      tc_fence_before();
      if (p.lse && row_ok) {
        const float mu = (m_ref == NEG_INF) ? 0.f : m_ref;
        const float v = l > 0.f ? (mu + __log2f(l)) * 0.69314718055994530942f : NEG_INF;
        p.lse[((long long)b * p.Hq + h) * p.Sq + q] = v;
      }
      gt += nt;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kQkWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// seq_kv == 0: every row sees no key, O = 0 and lse = -inf (the empty softmax).
__global__ void attn_empty_kernel(uint16_t* O, long long sb, long long sh, long long ss, int B,
                                  int H, int S, int D, float* lse) {
  const long long rows = (long long)B * H * S;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < rows * D;
       i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / D;
    const int d = (int)(i - row * D);
    const int s = (int)(row % S);
    const long long bh = row / S;
    const int h = (int)(bh % H), b = (int)(bh / H);
    O[b * sb + h * sh + s * ss + d] = 0;
    if (lse && d == 0) lse[row] = -INFINITY;
  }
}

// ----------------------------------------------------------------------------------------
// Host side
// ----------------------------------------------------------------------------------------
namespace {

void packed_or(const int64_t* s, int64_t H, int64_t S, int64_t D, long long out[3]) {
  if (s[0] == 0 && s[1] == 0 && s[2] == 0) {
    out[2] = D;
    out[1] = S * D;
    out[0] = H * S * D;
  } else {
    out[0] = s[0];
    out[1] = s[1];
    out[2] = s[2];
  }
}

template <int D, bool BF16>
int launch_attn(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                const AttnParams& p, int ctas, cudaStream_t stream) {
  auto kern = attn_fwd_kernel<D, BF16>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       AttnCfg<D>::kSmem);
  if (e != cudaSuccess) return fail_cuda(e, "lvb_attention_fwd", "cudaFuncSetAttribute");
  kern<<<ctas, kAttnThreads, AttnCfg<D>::kSmem, stream>>>(tq, tk, tv, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail_cuda(e, "lvb_attention_fwd", "kernel launch");
  return LVB_OK;
}

}  // namespace

int attn_smem_bytes(int D) { return D == 64 ? AttnCfg<64>::kSmem : AttnCfg<128>::kSmem; }

int attn_launch(const lvb_attn_desc* d, const void* Q, const void* K, const void* V, void* O,
                float* lse, cudaStream_t stream, DeviceState* dev) {
  const char* op = "lvb_attention_fwd";
  const int64_t B = d->batch, Hq = d->heads_q, Hkv = d->heads_kv, Sq = d->seq_q, Skv = d->seq_kv,
                D = d->head_dim;
  long long qs[3], ks[3], vs[3], os[3];
  packed_or(d->q_stride, Hq, Sq, D, qs);
  packed_or(d->k_stride, Hkv, Skv, D, ks);
  packed_or(d->v_stride, Hkv, Skv, D, vs);
  packed_or(d->o_stride, Hq, Sq, D, os);
  if (Skv == 0) {
    const long long total = B * Hq * Sq * D;
    const int blocks = (int)std::min<long long>((total + 255) / 256, 8192);
    attn_empty_kernel<<<blocks, 256, 0, stream>>>((uint16_t*)O, os[0], os[1], os[2], (int)B,
                                                  (int)Hq, (int)Sq, (int)D, lse);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? LVB_OK : fail_cuda(e, op, "empty-softmax launch");
  }
  if (attn_decode_applies(d))
    return attn_decode_launch(d, qs, ks, vs, os, Q, K, V, O, lse, stream, dev);
  const uint32_t rowsbox = 128;
  CUtensorMap tq, tk, tv;
  {
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)Sq, (uint64_t)Hq, (uint64_t)B};
    const uint64_t str[3] = {(uint64_t)qs[2], (uint64_t)qs[1], (uint64_t)qs[0]};
    const uint32_t box[4] = {64, rowsbox, 1, 1};
    int st = make_tmap_nd(&tq, Q, 2, 4, dims, str, box, op);
    if (st) return st;
  }
  {
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)Skv, (uint64_t)Hkv, (uint64_t)B};
    const uint64_t strk[3] = {(uint64_t)ks[2], (uint64_t)ks[1], (uint64_t)ks[0]};
    const uint64_t strv[3] = {(uint64_t)vs[2], (uint64_t)vs[1], (uint64_t)vs[0]};
    const uint32_t box[4] = {64, rowsbox, 1, 1};
    int st = make_tmap_nd(&tk, K, 2, 4, dims, strk, box, op);
    if (st) return st;
    st = make_tmap_nd(&tv, V, 2, 4, dims, strv, box, op);
    if (st) return st;
  }
  AttnParams p;
  p.B = (int)B;
  p.Hq = (int)Hq;
  p.Hkv = (int)Hkv;
  p.Sq = (int)Sq;
  p.Skv = (int)Skv;
  p.group = (int)(Hq / Hkv);
  p.num_pairs = (int)((Sq + 255) / 256);
  p.causal = d->causal ? 1 : 0;
  p.scale_log2 = d->scale * 1.4426950408889634f;
  p.O = O;
  p.o_sb = os[0];
  p.o_sh = os[1];
  p.o_ss = os[2];
  p.lse = lse;
  p.status = dev->status;
  p.timeout_ns = wait_timeout_ns();
  const long long items = (long long)p.num_pairs * B * Hq;
  if (items > 2147483647LL - 4096)
    return fail(LVB_ERR_UNSUPPORTED, op, "more than 2^31 query-tile pairs", "split the batch");
  p.total_items = (int)items;
  const int ctas = (int)std::min<long long>(items, std::max(1, dev->sm_count));
  // Causal items differ in length: the last ~two waves of items (whole heads) go
  // longest-first (equal-length items gain nothing from it).
  p.tail_heads = 0;
  if (p.causal) {
    const long long want = (2LL * ctas + p.num_pairs - 1) / p.num_pairs;
    p.tail_heads = (int)std::min<long long>(B * Hq, std::max<long long>(1, want));
  }
  // The item counter: zeroed on the stream before the launch, freed after it.
  void* ws = nullptr;
  cudaError_t e = workspace_alloc(dev, &ws, 16, stream);
  if (e != cudaSuccess) return fail_cuda(e, op, "work counter allocation");
  p.work_counter = reinterpret_cast<int*>(ws);
  e = cudaMemsetAsync(ws, 0, 16, stream);
  int st = e == cudaSuccess ? LVB_OK : fail_cuda(e, op, "work counter reset");
  const bool bf16 = d->dtype == LVB_BF16;
  if (st == LVB_OK) {
    if (D == 128)
      st = bf16 ? launch_attn<128, true>(tq, tk, tv, p, ctas, stream)
                : launch_attn<128, false>(tq, tk, tv, p, ctas, stream);
    else if (D == 64)
      st = bf16 ? launch_attn<64, true>(tq, tk, tv, p, ctas, stream)
                : launch_attn<64, false>(tq, tk, tv, p, ctas, stream);
    else
      st = fail(LVB_ERR_UNSUPPORTED, op, "head_dim must be 64 or 128");
  }
  e = cudaFreeAsync(ws, stream);
  if (st == LVB_OK && e != cudaSuccess) return fail_cuda(e, op, "work counter free");
  return st;
}

}  // namespace lvb
