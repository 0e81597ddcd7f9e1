// Tensor-core paged attention with the softmax split by key halves (head dims up to 128): the tensor path's
// FGW_TENSOR_KERNEL_HALVES.
//
// Same contract, masking rules and epilogues as the other tensor kernels; the reference body it stands for is
// operators/mha/kernels/mha_paged_decode_ascend_v7.py:225-315, 375-465. The schedule:
//   * one 128-row query tile per work item (request, head, split, query tile); the CTA's items form one global
//     sequence of KV tiles g = 0, 1, ...; S is double-buffered in TMEM (S[g % 2]), so QK(g + 2) is issued right
//     after PV(g) and the softmax of tile g + 1 never waits for the tensor core;
//   * two softmax warpgroups: warps 4-7 own keys [0, 64) of every 128-key tile, warps 8-11 keys [64, 128). Each
//     keeps its own running max and sum and its own O accumulator (O_0, O_1 in TMEM), like two interleaved KV
//     splits, so the warpgroups never exchange a row max inside the loop; the epilogue merges the two halves
//     with their LSE weights;
//   * P of each half goes back into the first 32 TMEM columns of that half of S, and PV_h reads it from there
//     (tcgen05.mma with the A operand in tensor memory);
//   * one shared-memory stage per tile holds V(g) and K(g + 2) (stage u = g + 2 holds V(u - 2) and K(u); the first
//     two stages of the sequence hold K only), so the MMA warp waits on one barrier per tile, and a stage is free
//     once QK(u) has completed (the commit that publishes S also releases the stage: QK(u) is issued after
//     PV(u - 2));
//   * the softmax warps hand P(g) to the MMA warp through a named barrier (bar.arrive / bar.sync) instead of an
//     mbarrier the issuing thread polls; the MMA warp runs as a whole warp, one lane issuing;
//   * Q is double-buffered, so the next item's first two QKs run while this item's epilogue reads O.
// TMEM: S0 [0, 128), S1 [128, 256), O_0 [256, 256 + D), O_1 [384, 384 + D) of 512 columns.
//
// Barrier phases. Every parity wait below is on a phase that cannot be two completions old: s_full[b] completes
// once per QK into S[b], and QK(g + 2) needs P(g), which its waiters have not released yet; pv_done completes
// once per tile and a softmax warp that rescales at tile g + 1 has seen S(g + 1), whose QK was issued after
// PV(g - 1), so at most PV(g) is outstanding; o_full completes once per non-empty item and the next item's last
// PV needs this item's epilogue first; full[s] completes once per stage and stage u + 2 reuses the slot only
// after QK(u). The producer waits on s_full for a stage's release, which needs exactly two stages in the ring.
#include <algorithm>

#include "fgw_common.cuh"
#include "fgw_kernels.h"

namespace fgw {

struct HalvesArgs {
  void* out;
  const int32_t* table;
  const int32_t* lengths;
  const int32_t* order;
  float* part_o;
  float* part_lse;
  WorkspaceHeader* ws;
  int batch, sq, heads, dim, width, page, splits, causal, box_rows, write_partials, qtiles;
  long long items;
  // contiguous schedule (one split): per-program first item, unit offset and first unit, the per-item arrival
  // counters and two partial slots of 128 rows per program; whole items below tail_start first
  int contiguous, programs, tail_start;
  const int32_t* prog_item;
  const int32_t* prog_off;
  const long long* prog_u;
  int32_t* counters;
  float* slot_lse;
  float* slot_o;
  float scale_log2;
  uint64_t budget_ns;
};

template <int NB>
struct HalvesShape {
  static constexpr int kBN = 128;                  // keys per KV tile; each softmax warpgroup owns 64
  static constexpr int kTileBytes = 128 * 128;     // one 64-column block of a 128-row operand
  static constexpr int kQBytes = NB * kTileBytes;  // one query tile
  static constexpr int kKBytes = NB * kBN * 128;   // one K (or V) tile
  static constexpr int kStageBytes = 2 * kKBytes;  // V(u - 2) at 0, K(u) at kKBytes
  static constexpr int kStages = 2;                // the s_full release needs exactly two (see above)
  static constexpr int kThreads = 384;
  // registers per thread after the warpgroup split (4 x 32 x 88 + 8 x 32 x 208 = 384 x 168)
  static constexpr int kRegsControl = 88;
  static constexpr int kRegsSoftmax = 208;
  __device__ __forceinline__ static uint32_t o_col(int h) { return 256u + 128u * static_cast<uint32_t>(h); }
  static constexpr int kTmemCols = 512;
  // shared memory carve-up; kX: per half, the row max and row sum of every row, for the epilogue merge
  static constexpr int kQ = 0;
  static constexpr int kStage = kQ + 2 * kQBytes;
  static constexpr int kX = kStage + kStages * kStageBytes;
  static constexpr int kBar = kX + 2 * 2 * 128 * 4;
  // q_full[2], q_empty[2], full[kStages], s_full[2], pv_done, o_full, mma_done
  static constexpr int kNumBars = 4 + kStages + 5;
  static constexpr int kTmemSlot = kBar + kNumBars * 8;
  static constexpr int kBytes = kTmemSlot + 16 + 1024;
  // named barriers: P(g) handed over on kBarP + g % 2 (8 softmax warps arrive, the MMA warp syncs); the two
  // warpgroups exchange their epilogue states on kBarX
  static constexpr uint32_t kBarP = 4;
  static constexpr uint32_t kBarPThreads = 9 * 32;
  static constexpr uint32_t kBarX = 6;
};

struct HalvesItem {
  int b, h, s, q0, len, n_begin, n;
};

__device__ __forceinline__ int halves_visible(int row, int len, int sq, int causal) {
  return causal ? max(len - sq + row + 1, 0) : len;
}

__device__ __forceinline__ void halves_item(const HalvesArgs& a, long long item, HalvesItem& c) {
  const int qt_rev = static_cast<int>(item % a.qtiles);
  long long rest = item / a.qtiles;
  c.s = static_cast<int>(rest % a.splits);
  rest /= a.splits;
  c.h = static_cast<int>(rest % a.heads);
  c.b = a.order[rest / a.heads];
  c.q0 = (a.qtiles - 1 - qt_rev) * 128;  // later query tiles first: they see the most keys when causal
  c.len = a.lengths[c.b];
  const int last = min(c.q0 + 128, a.sq) - 1;
  const int tiles = (halves_visible(last, c.len, a.sq, a.causal) + 127) / 128;
  c.n_begin = static_cast<int>((long long)tiles * c.s / a.splits);
  c.n = static_cast<int>((long long)tiles * (c.s + 1) / a.splits) - c.n_begin;
}

// One run of KV tiles of one item processed by this CTA: a whole item, or, with the contiguous schedule, tiles
// [first, first + count) of an item (a piece when other CTAs hold the rest of it).
struct HalvesSegment {
  long long item;
  bool piece;
  long long item_u;  // first unit of the item in the contiguous cut
  int units;         // units of the whole item (at least 1)
};

struct SegmentWalk {
  long long whole;  // next whole item (strided part)
  long long item;
  int off;
  long long u, u_end;
};

__device__ __forceinline__ void segment_walk_init(const HalvesArgs& a, SegmentWalk& k) {
  k.whole = blockIdx.x;
  k.item = a.contiguous ? a.prog_item[blockIdx.x] : 0;
  k.off = a.contiguous ? a.prog_off[blockIdx.x] : 0;
  k.u = a.contiguous ? a.prog_u[blockIdx.x] : 0;
  k.u_end = a.contiguous ? a.prog_u[blockIdx.x + 1] : 0;
}

// The next segment of this CTA, with `c` the item restricted to the segment's tiles. Every role walks the same
// segments in the same order: whole items first (all of them with the strided schedule), then the CTA's
// contiguous range of units.
__device__ __forceinline__ bool segment_walk_next(const HalvesArgs& a, SegmentWalk& k, HalvesSegment& sg,
                                                  HalvesItem& c) {
  const long long whole_end = a.contiguous ? a.tail_start : a.items;
  if (k.whole < whole_end) {
    sg.item = k.whole;
    sg.piece = false;
    sg.item_u = 0;
    sg.units = 0;
    halves_item(a, k.whole, c);
    k.whole += gridDim.x;
    return true;
  }
  if (!a.contiguous || k.u >= k.u_end) return false;
  halves_item(a, k.item, c);  // one split: the whole item
  const int tiles = c.n;
  const int units = max(tiles, 1);  // an item without keys still costs one unit (its rows are written as zeros)
  const int count = static_cast<int>(min(static_cast<long long>(units - k.off), k.u_end - k.u));
  sg.item = k.item;
  sg.piece = count < units;
  sg.item_u = k.u - k.off;
  sg.units = units;
  c.n_begin = k.off;
  c.n = max(0, min(k.off + count, tiles) - k.off);
  k.u += count;
  k.off += count;
  if (k.off >= units) {
    ++k.item;
    k.off = 0;
  }
  return true;
}

// Walks the CTA's segments that have tiles, tile by tile, `ahead` tiles ahead of a consumer: the producer and the
// MMA warp need the segment of tile g + 2 while they work on tile g.
struct TileCursor {
  SegmentWalk walk;
  HalvesSegment sg;
  HalvesItem c;    // current segment's item, restricted to its tiles
  int j;           // tile within it
  int items_seen;  // segments with tiles entered so far (their Q buffer is (items_seen - 1) % 2)
  bool valid;
};

__device__ __forceinline__ void tile_cursor_advance(const HalvesArgs& a, TileCursor& t) {
  if (t.valid && t.j + 1 < t.c.n) {
    ++t.j;
    return;
  }
  t.valid = false;
  while (segment_walk_next(a, t.walk, t.sg, t.c)) {
    if (t.c.n > 0) {
      t.j = 0;
      ++t.items_seen;
      t.valid = true;
      return;
    }
  }
}

__device__ __forceinline__ void tile_cursor_init(const HalvesArgs& a, TileCursor& t) {
  segment_walk_init(a, t.walk);
  t.j = 0;
  t.items_seen = 0;
  t.valid = false;
  tile_cursor_advance(a, t);
}

// 2^(s * scale - m) for the 64 scores of one half row (32 FP32 pairs, scale-and-subtract two lanes per
// instruction), summed into four partial sums and packed to 16-bit pairs.
template <typename Tr>
__device__ __forceinline__ void halves_exp2_pack(const uint32_t (&sr)[64], float2 scale2, float2 negm2,
                                                 float2 (&acc)[4], uint32_t (&packed)[32]) {
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const float2 x = __ffma2_rn(make_float2(__uint_as_float(sr[2 * i]), __uint_as_float(sr[2 * i + 1])), scale2,
                                negm2);
    const float2 p = make_float2(fast_exp2(x.x), fast_exp2(x.y));
    acc[i % 4] = __fadd2_rn(acc[i % 4], p);
    packed[i] = Tr::pack2(p.x, p.y);
  }
}

__device__ __forceinline__ void named_barrier_arrive(uint32_t id, uint32_t threads) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

template <typename T, int NB>
__global__ void __launch_bounds__(384, 1)
    fmha_halves_sm100_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                             const __grid_constant__ CUtensorMap vmap, const HalvesArgs a) {
  using S = HalvesShape<NB>;
  using Tr = ElemTraits<T>;
  constexpr int BN = S::kBN;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* q_smem = smem + S::kQ;
  uint8_t* st_smem = smem + S::kStage;
  float* xch = reinterpret_cast<float*>(smem + S::kX);  // [half][0: max, 1: sum][row]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kBar);
  uint64_t* q_full = bars + 0;        // [2]
  uint64_t* q_empty = bars + 2;       // [2]
  uint64_t* full = bars + 4;          // [kStages]: a stage's V and K have landed
  uint64_t* s_full = full + S::kStages;  // [2]: S[b] holds a tile's scores (and frees the stage of that QK)
  uint64_t* pv_done = s_full + 2;     // PV of a tile has completed
  uint64_t* o_full = pv_done + 1;     // the last PV of an item has completed
  uint64_t* mma_done = o_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::kTmemSlot);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&s_full[i], 1);
    }
    for (int i = 0; i < S::kStages; ++i) mbar_init(&full[i], 1);
    mbar_init(pv_done, 1);
    mbar_init(o_full, 1);
    mbar_init(mma_done, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, S::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  const int D = a.dim;

  if (warp < 4) setmaxnreg_dec<S::kRegsControl>();  // warpgroup 0: TMA, MMA and two idle warps
  if (warp == 0) {
    // ------------------------------------------------------------------------- TMA producer
    // Stage u (ring slot u % 2) holds V(u - 2) and K(u) of the CTA's tile sequence; Q of each item goes into Q
    // buffer (item % 2) just before the item's first K.
    if (lane == 0) {
      tma_prefetch_desc(&qmap);
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
      bool ok = true;
      const int boxes = BN / a.box_rows;
      const uint32_t box_bytes = a.box_rows * 128;
      auto fail = [&](int site) {
        ok = false;
        record_error(a.ws, FGW_ERR_DEVICE_TIMEOUT, site);
      };
      // the live boxes of tile j of item c, and their loads into dst
      auto live_boxes = [&](const HalvesItem& c, int j) {
        const int tok0 = (c.n_begin + j) * BN;
        int nbox = 0;
        for (int k = 0; k < boxes; ++k) nbox += (tok0 + k * a.box_rows < c.len) ? 1 : 0;
        return nbox;
      };
      auto load_tile = [&](const CUtensorMap* map, const HalvesItem& c, int j, uint8_t* dst, uint64_t* bar,
                           int nbox) {
        const int32_t* row_table = a.table + (long long)c.b * a.width;
        const int tok0 = (c.n_begin + j) * BN;
        for (int k = 0; k < nbox; ++k) {
          const int tok = tok0 + k * a.box_rows;
          const int row = row_table[tok / a.page] * a.page + tok % a.page;
          for (int blk = 0; blk < NB; ++blk) {
            tma_load_3d(dst + blk * BN * 128 + k * box_bytes, map, bar, blk * 64, c.h, row);
          }
        }
      };
      TileCursor kc, vc;  // K(u) and V(u - 2)
      tile_cursor_init(a, kc);
      tile_cursor_init(a, vc);
      uint32_t u = 0;
      while (kc.valid || vc.valid) {
        const int slot = u & 1;
        // the slot's previous stage (u - 2) is free once QK(u - 2) has completed
        if (ok && u >= 2 && !mbar_wait(&s_full[slot], ((u - 2) >> 1) & 1, a.budget_ns)) fail(70);
        const bool has_k = kc.valid;
        const bool has_v = u >= 2 && vc.valid;
        if (has_k && kc.j == 0) {
          // the item's Q, into buffer (items - 1) % 2, once the item two back has issued its last QK
          const int qb = (kc.items_seen - 1) & 1;
          if (ok && kc.items_seen > 2 && !mbar_wait(&q_empty[qb], ((kc.items_seen - 3) >> 1) & 1, a.budget_ns)) {
            fail(71);
          }
          if (ok) {
            mbar_arrive_expect_tx(&q_full[qb], S::kQBytes);
            for (int blk = 0; blk < NB; ++blk) {
              tma_load_4d(q_smem + qb * S::kQBytes + blk * S::kTileBytes, &qmap, &q_full[qb], blk * 64, kc.c.h,
                          kc.c.q0, kc.c.b);
            }
          }
        }
        const int kbox = has_k ? live_boxes(kc.c, kc.j) : 0;
        const int vbox = has_v ? live_boxes(vc.c, vc.j) : 0;
        if (ok) {
          uint8_t* dst = st_smem + slot * S::kStageBytes;
          mbar_arrive_expect_tx(&full[slot], NB * (kbox + vbox) * box_bytes);
          if (has_v) load_tile(&vmap, vc.c, vc.j, dst, &full[slot], vbox);
          if (has_k) load_tile(&kmap, kc.c, kc.j, dst + S::kKBytes, &full[slot], kbox);
        }
        if (has_k) tile_cursor_advance(a, kc);
        if (has_v) tile_cursor_advance(a, vc);
        ++u;
      }
      // leave no copy in flight: the last two stages landed (or their waits gave up)
      for (uint32_t w = (u >= 2 ? u - 2 : 0); w < u; ++w) mbar_wait(&full[w & 1], (w >> 1) & 1, a.budget_ns);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------------- UMMA issuer (whole warp, lane 0
    // issues; the warp takes part in the P named barriers)
    bool ok = true;
    const int fmt = Tr::kUmmaFormat;
    const uint32_t idesc_qk = umma_idesc_f16(fmt, 128, BN, 0, 0);
    const uint32_t idesc_pv = umma_idesc_f16(fmt, 128, D, 0, 1);
    const uint32_t q_lo = umma_desc_lo(smem_u32(q_smem), 16);
    const uint32_t k_lo = umma_desc_lo(smem_u32(st_smem + S::kKBytes), 16);
    const uint32_t v_lo = umma_desc_lo(smem_u32(st_smem), BN * 128);
    constexpr uint32_t kHi = umma_desc_hi(1024, 2);
    const int ksteps_qk = D / 16;
    auto wait_lane0 = [&](uint64_t* bar, uint32_t parity, int site) {
      bool good = true;
      if (lane == 0 && ok) {
        good = mbar_wait(bar, parity, a.budget_ns);
        if (!good) record_error(a.ws, FGW_ERR_DEVICE_TIMEOUT, site);
      }
      ok = __shfl_sync(0xffffffffu, ok && good, 0);
      return ok;
    };
    // S[buf] = Q K^T with Q from buffer qb and K from the stage of slot `slot`; publishes S[buf] (and frees the
    // stage for the producer).
    auto qk = [&](uint32_t buf, int qb, int slot) {
      if (lane == 0) {
        const uint32_t a_base = q_lo + static_cast<uint32_t>((qb * S::kQBytes) >> 4);
        const uint32_t b_base = k_lo + static_cast<uint32_t>((slot * S::kStageBytes) >> 4);
#pragma unroll
        for (int kk = 0; kk < 4 * NB; ++kk) {
          if (kk < ksteps_qk) {
            const uint32_t a_off = static_cast<uint32_t>(((kk >> 2) * S::kTileBytes + (kk & 3) * 32) >> 4);
            const uint32_t b_off = static_cast<uint32_t>(((kk >> 2) * BN * 128 + (kk & 3) * 32) >> 4);
            umma_f16_ss_w(tmem + buf * 128u, a_base + a_off, kHi, b_base + b_off, kHi, idesc_qk, kk > 0 ? 1u : 0u);
          }
        }
        umma_commit(&s_full[buf]);
      }
    };
    // O_h += P_h V_h over keys [64 h, 64 h + 64) for both halves: P_h from the first 32 columns of half h of
    // S[buf], V rows from the stage of slot `slot`.
    auto pv = [&](uint32_t buf, int slot, bool first) {
      if (lane == 0) {
        const uint32_t b_base = v_lo + static_cast<uint32_t>((slot * S::kStageBytes) >> 4);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
#pragma unroll
          for (int k4 = 0; k4 < 4; ++k4) {
            const int kk = 4 * half + k4;  // 16-key step within the tile
            umma_f16_ts_w(tmem + S::o_col(half), tmem + buf * 128u + 64u * half + 8u * k4,
                          b_base + static_cast<uint32_t>((kk * 16 * 128) >> 4), kHi, idesc_pv,
                          (!first || k4 > 0) ? 1u : 0u);
          }
        }
        umma_commit(pv_done);
      }
    };
    TileCursor cur, ahead;  // tile g and tile g + 2
    tile_cursor_init(a, cur);
    tile_cursor_init(a, ahead);
    // prologue: S of the first two tiles
    uint32_t g = 0;
    for (int u = 0; u < 2 && ahead.valid; ++u) {
      const int qb = (ahead.items_seen - 1) & 1;
      if (ahead.j == 0) wait_lane0(&q_full[qb], ((ahead.items_seen - 1) >> 1) & 1, 75);
      wait_lane0(&full[u], 0, 76 + u);
      if (ok) {
        tc_fence_after_sync();
        qk(u, qb, u);
        if (lane == 0 && ahead.j + 1 == ahead.c.n) umma_commit(&q_empty[qb]);
      }
      tile_cursor_advance(a, ahead);
    }
    while (cur.valid) {
      const uint32_t buf = g & 1;
      const uint32_t u = g + 2;  // the stage holding V(g) and K(g + 2)
      const int slot = u & 1;
      __syncwarp();
      named_barrier_sync(S::kBarP + buf, S::kBarPThreads);  // both halves of P(g) are in TMEM
      wait_lane0(&full[slot], (u >> 1) & 1, 78);
      if (ok) {
        tc_fence_after_sync();
        pv(buf, slot, cur.j == 0);
        if (lane == 0 && cur.j + 1 == cur.c.n) umma_commit(o_full);  // the item's O is complete
      }
      if (ahead.valid) {
        // S[buf] takes tile g + 2 (both halves of P(g) are consumed first, in issue order)
        const int qb = (ahead.items_seen - 1) & 1;
        if (ahead.j == 0) wait_lane0(&q_full[qb], ((ahead.items_seen - 1) >> 1) & 1, 79);
        if (ok) {
          tc_fence_after_sync();
          qk(buf, qb, slot);
          if (lane == 0 && ahead.j + 1 == ahead.c.n) umma_commit(&q_empty[qb]);  // every QK of that item issued
        }
        tile_cursor_advance(a, ahead);
      }
      tile_cursor_advance(a, cur);
      ++g;
    }
    if (lane == 0 && ok) {
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, a.budget_ns);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------------------- softmax / epilogue
    // Warpgroup 1 (warps 4-7) owns keys [0, 64) of every tile, warpgroup 2 (warps 8-11) keys [64, 128). A warp
    // may only touch the TMEM lane quarter warp % 4, so each warpgroup covers all 128 rows.
    setmaxnreg_inc<S::kRegsSoftmax>();
    const int half = (warp - 4) / 4;
    const int row = (warp % 4) * 32 + lane;  // TMEM lane = query row within the tile
    const uint32_t lane_base = static_cast<uint32_t>((warp % 4) * 32) << 16;
    const uint32_t o_own = tmem + lane_base + S::o_col(half);
    bool ok = true;
    uint32_t g = 0, items_done = 0;
    auto wait_warp = [&](uint64_t* bar, uint32_t parity, int site) {
      if (ok) {
        ok = __all_sync(0xffffffffu, mbar_wait(bar, parity, a.budget_ns));
        if (!ok && lane == 0) record_error(a.ws, FGW_ERR_DEVICE_TIMEOUT, site);
      }
      return ok;
    };
    SegmentWalk walk;
    segment_walk_init(a, walk);
    HalvesSegment sg;
    HalvesItem c;
    volatile int* merge_flag = reinterpret_cast<volatile int*>(smem + S::kTmemSlot + 4);
    while (segment_walk_next(a, walk, sg, c)) {
      const int q = c.q0 + row;
      const bool row_valid = q < a.sq;
      const int vis = row_valid ? halves_visible(q, c.len, a.sq, a.causal) : 0;
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < c.n; ++j, ++g) {
        const uint32_t buf = g & 1;
        const int tok0 = (c.n_begin + j) * BN;
        wait_warp(&s_full[buf], (g >> 1) & 1, 80 + half);
        const int valid_cols = min(max(vis - tok0 - 64 * half, 0), 64);
        const uint32_t s_addr = tmem + lane_base + buf * 128u + 64u * half;
        uint32_t sr[64];
        if (ok) {
          tc_fence_after_sync();
          tmem_ld32(s_addr, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
          tmem_ld32(s_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 64; ++i) sr[i] = __float_as_uint(-INFINITY);
        }
        if (valid_cols < 64) {
          // ragged / diagonal tile: mask columns at or past this row's visible count
#pragma unroll
          for (int col = 0; col < 64; ++col) {
            if (col >= valid_cols) sr[col] = 0xff800000u;  // -inf
          }
        }
        float mx_raw = -INFINITY;
#pragma unroll
        for (int col = 0; col < 64; col += 4) {
          mx_raw = fmaxf(mx_raw, fmaxf(fmaxf(__uint_as_float(sr[col]), __uint_as_float(sr[col + 1])),
                                       fmaxf(__uint_as_float(sr[col + 2]), __uint_as_float(sr[col + 3]))));
        }
        const float mx = mx_raw * a.scale_log2;  // scale > 0; -inf stays -inf
        float m_new = m;
        bool grow = false;
        if (j == 0) {
          m_new = mx;
        } else if (mx > m + 8.0f) {
          grow = true;
        }
        const bool warp_grow = __any_sync(0xffffffffu, grow);
        float alpha = 1.f;
        if (warp_grow && j > 0) {
          m_new = fmaxf(m, mx);
          alpha = (m == -INFINITY) ? 0.f : fast_exp2(m - m_new);
        }
        const float neg_m = (m_new == -INFINITY) ? 0.f : -m_new;
        // P = 2^(s*scale - m), packed over the first 32 columns of this half of S (the scores are in registers)
        float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
        if (ok) {
          uint32_t packed[32];
          halves_exp2_pack<Tr>(sr, make_float2(a.scale_log2, a.scale_log2), make_float2(neg_m, neg_m), acc, packed);
          tmem_st32(s_addr, packed);
        }
        // O_h may be rescaled only once PV(g - 1) has completed (at most that PV is outstanding here).
        if (warp_grow && j > 0) {
          wait_warp(pv_done, (g - 1) & 1, 82 + half);
          if (ok) {
            tc_fence_after_sync();
            for (int cb = 0; cb < D / 16; ++cb) {
              uint32_t r[16];
              tmem_ld16(o_own + cb * 16, r);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
              tmem_st16(o_own + cb * 16, r);
            }
          }
        }
        // Value rows past the cache end: this half's rows of V(g) are zeroed before its P is released (PV reads
        // them). V(g) is in the stage u = g + 2.
        if (tok0 + BN > c.len) {
          const uint32_t u = g + 2;
          wait_warp(&full[u & 1], (u >> 1) & 1, 84 + half);
          const int vrow = 64 * half + row;
          if (ok && row < 64 && tok0 + vrow >= c.len) {
            uint8_t* dst = st_smem + (u & 1) * S::kStageBytes + vrow * 128;
#pragma unroll
            for (int blk = 0; blk < NB; ++blk) {
#pragma unroll
              for (int ch = 0; ch < 8; ++ch) {
                *reinterpret_cast<uint4*>(dst + blk * BN * 128 + ch * 16) = make_uint4(0, 0, 0, 0);
              }
            }
          }
          fence_proxy_async_smem();
        }
        if (ok) tmem_wait_st();
        tc_fence_before_sync();
        __syncwarp();
        named_barrier_arrive(S::kBarP + buf, S::kBarPThreads);  // every tile, whatever happened above
        const float rowsum = (acc[0].x + acc[0].y) + (acc[1].x + acc[1].y) + (acc[2].x + acc[2].y) +
                             (acc[3].x + acc[3].y);
        l = l * alpha + rowsum;
        m = m_new;
      }
      if (c.n > 0) {
        wait_warp(o_full, items_done & 1, 86 + half);  // the item's last PV has completed
        ++items_done;
      }
      // epilogue: merge the two halves' running states (LSE weights), then each warpgroup normalises and
      // stores alternate 16-column blocks of the row
      xch[(2 * half) * 128 + row] = m;
      xch[(2 * half + 1) * 128 + row] = l;
      __syncwarp();  // the named barriers are the aligned form: the warp arrives converged
      named_barrier_sync(S::kBarX, 256);  // both halves' states are published
      const float m0 = xch[row], l0 = xch[128 + row], m1 = xch[256 + row], l1 = xch[384 + row];
      const float mt = fmaxf(m0, m1);
      const float w0 = (m0 == -INFINITY) ? 0.f : fast_exp2(m0 - mt);
      const float w1 = (m1 == -INFINITY) ? 0.f : fast_exp2(m1 - mt);
      const float lt = l0 * w0 + l1 * w1;
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      const float lse = (c.n > 0 && lt > 0.f) ? mt + fast_log2(lt) : kEmptyLse;
      const long long row_id = row_valid ? ((long long)c.b * a.sq + q) * a.heads + c.h : 0;
      long long my_slot = 0;  // this program's slot for a piece (contiguous schedule)
      if (sg.piece) {
        const long long total = a.prog_u[a.programs];
        const int q_first = program_of(total, a.programs, sg.item_u);
        const int first_extra = sg.item_u != program_start(total, a.programs, q_first) ? 1 : 0;
        my_slot = piece_slot(q_first, first_extra, static_cast<int>(blockIdx.x) - q_first);
        if (row_valid && half == 0) a.slot_lse[my_slot * 128 + row] = lse;
      }
      const bool read_o = c.n > 0 && ok;
      if (read_o) tc_fence_after_sync();
      // this warpgroup's blocks cb = half, half + 2, ...: both O halves of up to four blocks loaded before one wait
      constexpr int kBlocks = NB * 4;  // 16-column blocks of the O accumulators (D / 16 of them hold data)
#pragma unroll
      for (int c0 = 0; c0 < kBlocks; c0 += 4) {
        uint32_t r0[2][16], r1[2][16];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const int cb = c0 + 2 * k + half;
          if (read_o && cb < D / 16) {  // warp-collective: every lane, valid row or not
            tmem_ld16(tmem + lane_base + S::o_col(0) + cb * 16, r0[k]);
            tmem_ld16(tmem + lane_base + S::o_col(1) + cb * 16, r1[k]);
          }
        }
        if (read_o) tmem_wait_ld();
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const int cb = c0 + 2 * k + half;
          if (cb >= D / 16) continue;
          float o[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            o[i] = read_o ? (__uint_as_float(r0[k][i]) * w0 + __uint_as_float(r1[k][i]) * w1) * inv : 0.f;
          }
          if (row_valid && sg.piece) {
            float4* dst = reinterpret_cast<float4*>(a.slot_o + (my_slot * 128 + row) * D + cb * 16);
#pragma unroll
            for (int i = 0; i < 4; ++i) dst[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
          } else if (row_valid && a.write_partials) {
            float4* dst = reinterpret_cast<float4*>(a.part_o + (row_id * a.splits + c.s) * D + cb * 16);
#pragma unroll
            for (int i = 0; i < 4; ++i) dst[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
          } else if (row_valid) {
            uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<T*>(a.out) + row_id * D + cb * 16);
            dst[0] = make_uint4(Tr::pack2(o[0], o[1]), Tr::pack2(o[2], o[3]), Tr::pack2(o[4], o[5]),
                                Tr::pack2(o[6], o[7]));
            dst[1] = make_uint4(Tr::pack2(o[8], o[9]), Tr::pack2(o[10], o[11]), Tr::pack2(o[12], o[13]),
                                Tr::pack2(o[14], o[15]));
          }
        }
      }
      if (row_valid && a.write_partials && half == 0) a.part_lse[row_id * a.splits + c.s] = lse;
      if (sg.piece) {
        // A piece of an item cut between CTAs: its partial (normalised FP32 O and base-2 LSE) went to this
        // program's slot above; it counts itself in on the item's counter, and the piece whose arrival completes
        // the set merges every piece from its slot in piece order (so the result does not depend on which CTA
        // finished last). No CTA waits for another.
        __threadfence();
        __syncwarp();
        named_barrier_sync(S::kBarX, 256);  // both warpgroups have written their blocks
        if (warp == 4 && lane == 0) {
          const long long total = a.prog_u[a.programs];
          const int q_first = program_of(total, a.programs, sg.item_u);
          const int pieces = program_of(total, a.programs, sg.item_u + sg.units - 1) - q_first + 1;
          *merge_flag = atomicAdd(&a.counters[sg.item], 1) + 1 == pieces ? 1 : 0;
        }
        __syncwarp();
        named_barrier_sync(S::kBarX, 256);
        const int merge = *merge_flag;
        if (merge) {
          __threadfence();
          if (warp == 4 && lane == 0) a.counters[sg.item] = 0;  // ready for the next launch
        }
        if (merge && row_valid) {
          const long long total = a.prog_u[a.programs];
          const int q_first = program_of(total, a.programs, sg.item_u);
          const int pieces = program_of(total, a.programs, sg.item_u + sg.units - 1) - q_first + 1;
          const int first_extra = sg.item_u != program_start(total, a.programs, q_first) ? 1 : 0;
          float peak = kEmptyLse;
          for (int k = 0; k < pieces; ++k) {
            peak = fmaxf(peak, __ldcg(&a.slot_lse[piece_slot(q_first, first_extra, k) * 128 + row]));
          }
          float wsum = 0.f;
          for (int k = 0; k < pieces; ++k) {
            const float lk = __ldcg(&a.slot_lse[piece_slot(q_first, first_extra, k) * 128 + row]);
            if (lk > kValidLse) wsum += fast_exp2(lk - peak);
          }
          const float scale = wsum > 0.f ? 1.f / wsum : 0.f;
          for (int cb = half; cb < D / 16; cb += 2) {
            float acc[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) acc[i] = 0.f;
            for (int k = 0; k < pieces; ++k) {
              const long long pr = piece_slot(q_first, first_extra, k) * 128 + row;
              const float lk = __ldcg(&a.slot_lse[pr]);
              if (!(lk > kValidLse)) continue;
              const float w = fast_exp2(lk - peak);
              const float4* src = reinterpret_cast<const float4*>(a.slot_o + pr * D + cb * 16);
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const float4 v = __ldcg(src + i);
                acc[4 * i] += w * v.x;
                acc[4 * i + 1] += w * v.y;
                acc[4 * i + 2] += w * v.z;
                acc[4 * i + 3] += w * v.w;
              }
            }
            uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<T*>(a.out) + row_id * D + cb * 16);
            dst[0] = make_uint4(Tr::pack2(acc[0] * scale, acc[1] * scale), Tr::pack2(acc[2] * scale, acc[3] * scale),
                                Tr::pack2(acc[4] * scale, acc[5] * scale), Tr::pack2(acc[6] * scale, acc[7] * scale));
            dst[1] = make_uint4(Tr::pack2(acc[8] * scale, acc[9] * scale), Tr::pack2(acc[10] * scale, acc[11] * scale),
                                Tr::pack2(acc[12] * scale, acc[13] * scale),
                                Tr::pack2(acc[14] * scale, acc[15] * scale));
          }
        }
      }
      __syncwarp();
      named_barrier_sync(S::kBarX, 256);  // the exchange slots and the merge flag are free for the next segment
    }
  }
  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, S::kTmemCols);
  }
}

template <typename T, int NB>
static cudaError_t launch_halves_t(const LaunchDesc& d, const HalvesArgs& args, const CUtensorMap& qmap,
                                   const CUtensorMap& kmap, const CUtensorMap& vmap) {
  using S = HalvesShape<NB>;
  auto kernel = fmha_halves_sm100_kernel<T, NB>;
  // setmaxnreg.inc only succeeds if the registers the block was launched with cover the new split (see
  // launch_fmha2_t); refuse a build whose allocation would not cover it.
  cudaFuncAttributes attr;
  cudaError_t err = cudaFuncGetAttributes(&attr, kernel);
  if (err != cudaSuccess) return err;
  const int allocated = ((attr.numRegs + 7) / 8) * 8 * S::kThreads;
  if (allocated < 4 * 32 * S::kRegsControl + 8 * 32 * S::kRegsSoftmax) return cudaErrorNotSupported;
  err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kBytes);
  if (err != cudaSuccess) return err;
  const long long cap = d.p.grid_cap > 0 ? d.p.grid_cap : d.sm_count;
  // contiguous schedule: one CTA per program of the plan; strided: persistent CTAs over the items
  const long long grid = args.contiguous ? args.programs
                                         : std::min<long long>(args.items, std::min<long long>(cap, d.sm_count));
  if (grid <= 0) return cudaSuccess;
  kernel<<<(unsigned)grid, S::kThreads, S::kBytes, d.stream>>>(qmap, kmap, vmap, args);
  return cudaGetLastError();
}

cudaError_t launch_tensor_halves(const LaunchDesc& d, bool write_partials, const CUtensorMap& qmap,
                                 const CUtensorMap& kmap, const CUtensorMap& vmap, int box_rows) {
  const fgw_mha_params& p = d.p;
  HalvesArgs args;
  args.out = p.out;
  args.table = p.block_table;
  args.lengths = d.lens;
  args.order = d.order;
  args.part_o = d.part_o;
  args.part_lse = d.part_lse;
  args.ws = d.header;
  args.batch = p.batch;
  args.sq = p.q_len;
  args.heads = p.heads;
  args.dim = p.head_dim;
  args.width = p.table_width;
  args.page = p.page_size;
  args.splits = p.num_splits;
  args.causal = p.causal;
  args.box_rows = box_rows;
  args.write_partials = write_partials ? 1 : 0;
  args.qtiles = (p.q_len + 127) / 128;
  args.items = (long long)p.batch * p.heads * p.num_splits * args.qtiles;
  args.scale_log2 = (1.0f / sqrtf((float)p.head_dim)) * kLog2e;
  args.budget_ns = d.budget_ns;
  args.contiguous = d.contiguous ? 1 : 0;
  args.programs = d.contiguous ? d.programs : 0;
  args.tail_start = d.contiguous ? d.tail_start : 0;
  args.prog_item = d.prog_item;
  args.prog_off = d.prog_off;
  args.prog_u = d.prog_u;
  args.counters = d.counters;
  args.slot_lse = d.slot_lse;
  args.slot_o = d.slot_o;
  const bool bf16 = p.dtype == FGW_DTYPE_BFLOAT16;
  if (p.head_dim <= 64) {
    return bf16 ? launch_halves_t<__nv_bfloat16, 1>(d, args, qmap, kmap, vmap)
                : launch_halves_t<__half, 1>(d, args, qmap, kmap, vmap);
  }
  if (p.head_dim <= 128) {
    return bf16 ? launch_halves_t<__nv_bfloat16, 2>(d, args, qmap, kmap, vmap)
                : launch_halves_t<__half, 2>(d, args, qmap, kmap, vmap);
  }
  return cudaErrorInvalidValue;
}

}  // namespace fgw
