// Tensor-core paged attention with the softmax split by key halves (head dims up to 128): the tensor path's
// FGW_TENSOR_KERNEL_HALVES.
//
// Same contract, masking rules and epilogues as the other tensor kernels; the reference body it stands for is
// operators/mha/kernels/mha_paged_decode_ascend_v7.py:225-315, 375-465. The schedule:
//   * one 128-row query tile per work item (request, head, split, query tile); the CTA's segments (whole items,
//     or pieces of items under the contiguous schedule) form one sequence of KV tiles g = 0, 1, ...; S is
//     double-buffered in TMEM (S[g % 2]), so QK(g + 2) is issued right after PV(g) and the softmax of tile g + 1
//     never waits for the tensor core;
//   * Q lives in TMEM (two buffers: the next segment's Q is written while this one runs) and both products read
//     their A operand from TMEM (tcgen05.mma with A in tensor memory): only K and V come from shared memory. A
//     QK with Q in shared memory reads 8 KB of operands per M128 N128 K16 instruction, all that shared memory
//     delivers (128 bytes per cycle) in the instruction's 64 cycles, leaving none for the row-max exchange; with
//     Q in TMEM it reads 4 KB;
//   * two softmax warpgroups: warps 4-7 own keys [0, 64) of every 128-key tile, warps 8-11 keys [64, 128). They
//     exchange their partial row maxima through shared memory once per tile, so both halves exponentiate against
//     the same running max and accumulate into one O; each keeps its own partial row sum;
//   * P of each half goes back into the first 32 TMEM columns of that half of S, and PV reads it from there;
//   * K and V have rings of their own (K(g) is free once QK(g) has completed, V(g) once PV(g) has), so a tile's
//     loads start two tile periods before they are needed;
//   * the softmax warps hand P(g) to the MMA warp through a named barrier (bar.arrive / bar.sync); the MMA warp
//     runs as a whole warp, one lane issuing.
// TMEM: S0 [0, 128), S1 [128, 256), O [256, 256 + D), Q0 [384, 384 + D / 2), Q1 [448, 448 + D / 2).
//
// Barrier phases. Every parity wait below is on a phase that cannot be two completions old: s_full[b] completes
// once per QK into S[b], and QK(g + 2) needs P(g), which its waiters have not released yet; pv_done completes once
// per tile and a softmax warp that rescales at tile g + 1 has seen S(g + 1), whose QK was issued after PV(g - 1),
// so at most PV(g) is outstanding; o_full completes once per segment with tiles and the next segment's last PV
// needs this segment's epilogue first; a ring's full barrier of slot s is reloaded only after the tile it holds
// has been consumed; q_ready[b] / q_free[b] alternate with the segments.
#include <algorithm>

#include "fgw_common.cuh"
#include "fgw_kernels.h"

namespace fgw {

struct HalvesArgs {
  const void* q;
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
  static constexpr int kBN = 128;                    // keys per KV tile; each softmax warpgroup owns 64
  static constexpr int kTileBytes = NB * kBN * 128;  // one K (or V) tile: NB 64-column blocks of 128 rows
  static constexpr int kStages = NB == 1 ? 6 : 3;    // per ring
  static constexpr int kThreads = 384;
  // registers per thread after the warpgroup split (4 x 32 x 88 + 8 x 32 x 208 = 384 x 168)
  static constexpr int kRegsControl = 88;
  static constexpr int kRegsSoftmax = 208;
  static constexpr uint32_t kColO = 256;
  __device__ __forceinline__ static uint32_t q_col(int b) { return 384u + 64u * static_cast<uint32_t>(b); }
  static constexpr int kTmemCols = 512;
  // shared memory: K ring, V ring, the partial row maxima of both halves (two tiles' worth) and row sums
  static constexpr int kK = 0;
  static constexpr int kV = kK + kStages * kTileBytes;
  static constexpr int kXMax = kV + kStages * kTileBytes;  // [2 tiles][2 halves][128 rows] float
  static constexpr int kXSum = kXMax + 2 * 2 * 128 * 4;    // [2 halves][128 rows] float
  static constexpr int kBar = kXSum + 2 * 128 * 4;
  // k_full[S], k_empty[S], v_full[S], v_empty[S], s_full[2], q_ready[2], q_free[2], pv_done, o_full, mma_done
  static constexpr int kNumBars = 4 * kStages + 9;
  static constexpr int kTmemSlot = kBar + kNumBars * 8;
  static constexpr int kBytes = kTmemSlot + 16 + 1024;
  // named barriers: P(g) handed over on kBarP + g % 2 (8 softmax warps arrive, the MMA warp syncs); the two
  // warpgroups exchange row maxima and sums on kBarX
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
  long long round;  // next round of whole items (strided part, snake order)
  long long item;
  int off;
  long long u, u_end;
};

__device__ __forceinline__ void segment_walk_init(const HalvesArgs& a, SegmentWalk& k) {
  k.round = 0;
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
  const long long whole = snake_item(k.round);
  if (whole < whole_end) {
    sg.item = whole;
    sg.piece = false;
    sg.item_u = 0;
    sg.units = 0;
    halves_item(a, whole, c);
    ++k.round;
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

// Walks the CTA's segments that have tiles, tile by tile: the producer and the MMA warp keep one cursor on the
// tile they consume and one two tiles ahead.
struct TileCursor {
  SegmentWalk walk;
  HalvesSegment sg;
  HalvesItem c;  // current segment's item, restricted to its tiles
  int j;         // tile within it
  int seg;       // index of the current segment among those with tiles (its Q buffer is seg % 2)
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
      ++t.seg;
      t.valid = true;
      return;
    }
  }
}

__device__ __forceinline__ void tile_cursor_init(const HalvesArgs& a, TileCursor& t) {
  segment_walk_init(a, t.walk);
  t.j = 0;
  t.seg = -1;
  t.valid = false;
  tile_cursor_advance(a, t);
}

// 2^(s * scale - m) for the 64 scores of one half row (32 FP32 pairs, scale-and-subtract two lanes per
// instruction), packed to 16-bit pairs and summed, as rounded, into four partial sums.
template <typename Tr>
__device__ __forceinline__ void halves_exp2_pack(const uint32_t (&sr)[64], float2 scale2, float2 negm2,
                                                 float2 (&acc)[4], uint32_t (&packed)[32]) {
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const float2 x = __ffma2_rn(make_float2(__uint_as_float(sr[2 * i]), __uint_as_float(sr[2 * i + 1])), scale2,
                                negm2);
    packed[i] = Tr::pack2(fast_exp2(x.x), fast_exp2(x.y));
    // the row sum adds the rounded values PV multiplies (with the lazily rescaled running max a row's largest P
    // may exceed 1 and round; normalising by the unrounded sum would leave that rounding in the output)
    acc[i % 4] = Tr::add2(acc[i % 4], packed[i]);
  }
}

template <typename T, int NB>
__global__ void __launch_bounds__(384, 1)
    fmha_halves_sm100_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                             const HalvesArgs a) {
  using S = HalvesShape<NB>;
  using Tr = ElemTraits<T>;
  constexpr int BN = S::kBN;
  constexpr int NS = S::kStages;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* k_smem = smem + S::kK;
  uint8_t* v_smem = smem + S::kV;
  float* xmax = reinterpret_cast<float*>(smem + S::kXMax);  // [tile parity][half][row]
  float* xsum = reinterpret_cast<float*>(smem + S::kXSum);  // [half][row]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kBar);
  uint64_t* k_full = bars;
  uint64_t* k_empty = k_full + NS;
  uint64_t* v_full = k_empty + NS;
  uint64_t* v_empty = v_full + NS;
  uint64_t* s_full = v_empty + NS;  // [2]: S[b] holds a tile's scores
  uint64_t* q_ready = s_full + 2;   // [2]: Q buffer b holds the segment's query tile
  uint64_t* q_free = q_ready + 2;   // [2]: every QK reading Q buffer b has completed
  uint64_t* pv_done = q_free + 2;   // PV of a tile has completed
  uint64_t* o_full = pv_done + 1;   // the last PV of a segment has completed
  uint64_t* mma_done = o_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::kTmemSlot);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&q_ready[i], 8);  // every softmax warp writes its rows' half of Q
      mbar_init(&q_free[i], 1);
    }
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
  grid_dependency_wait();  // the plan's lengths, order and counters from here on

  if (warp < 4) setmaxnreg_dec<S::kRegsControl>();  // warpgroup 0: TMA, MMA and two idle warps
  if (warp == 0) {
    // ------------------------------------------------------------------------- TMA producer
    // K(t) into K-ring slot t % NS, V(t) into V-ring slot t % NS, in the order K0, K1, V0, K2, V1, K3, ...: the
    // order the MMA warp consumes them (QK(g + 2) follows PV(g)).
    if (lane == 0) {
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
      bool ok = true;
      const int boxes = BN / a.box_rows;
      const uint32_t box_bytes = a.box_rows * 128;
      auto load = [&](const CUtensorMap* map, const HalvesItem& c, int j, uint8_t* ring, uint64_t* full,
                      uint64_t* empty, uint32_t t, int site) {
        const int slot = t % NS;
        if (ok && !mbar_wait(&empty[slot], ((t / NS) & 1) ^ 1, a.budget_ns)) {
          ok = false;
          record_error(a.ws, FGW_ERR_DEVICE_TIMEOUT, site);
        }
        if (!ok) return;
        const int tok0 = (c.n_begin + j) * BN;
        int nbox = 0;
        for (int k = 0; k < boxes; ++k) nbox += (tok0 + k * a.box_rows < c.len) ? 1 : 0;
        mbar_arrive_expect_tx(&full[slot], NB * nbox * box_bytes);
        uint8_t* dst = ring + slot * S::kTileBytes;
        const int32_t* row_table = a.table + (long long)c.b * a.width;
        for (int k = 0; k < nbox; ++k) {
          const int tok = tok0 + k * a.box_rows;
          const int row = row_table[tok / a.page] * a.page + tok % a.page;
          for (int blk = 0; blk < NB; ++blk) {
            tma_load_3d(dst + blk * BN * 128 + k * box_bytes, map, &full[slot], blk * 64, c.h, row);
          }
        }
      };
      TileCursor kc, vc;
      tile_cursor_init(a, kc);
      tile_cursor_init(a, vc);
      uint32_t kt = 0, vt = 0;
      for (int i = 0; i < 2 && kc.valid; ++i, ++kt) {
        load(&kmap, kc.c, kc.j, k_smem, k_full, k_empty, kt, 70);
        tile_cursor_advance(a, kc);
      }
      while (vc.valid) {
        load(&vmap, vc.c, vc.j, v_smem, v_full, v_empty, vt, 71);
        tile_cursor_advance(a, vc);
        ++vt;
        if (kc.valid) {
          load(&kmap, kc.c, kc.j, k_smem, k_full, k_empty, kt, 72);
          tile_cursor_advance(a, kc);
          ++kt;
        }
      }
      // leave no copy in flight: the last loads of both rings landed (or their waits gave up)
      for (uint32_t t = (kt > NS ? kt - NS : 0); t < kt; ++t) mbar_wait(&k_full[t % NS], (t / NS) & 1, a.budget_ns);
      for (uint32_t t = (vt > NS ? vt - NS : 0); t < vt; ++t) mbar_wait(&v_full[t % NS], (t / NS) & 1, a.budget_ns);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------------- UMMA issuer (whole warp, lane 0
    // issues; the warp takes part in the P named barriers)
    bool ok = true;
    const int fmt = Tr::kUmmaFormat;
    const uint32_t idesc_qk = umma_idesc_f16(fmt, 128, BN, 0, 0);
    const uint32_t idesc_pv = umma_idesc_f16(fmt, 128, D, 0, 1);
    const uint32_t k_lo = umma_desc_lo(smem_u32(k_smem), 16);
    const uint32_t v_lo = umma_desc_lo(smem_u32(v_smem), BN * 128);
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
    // S[buf] = Q K^T with Q from TMEM buffer qb and K from ring slot `slot`; publishes S[buf], frees the K slot.
    auto qk = [&](uint32_t buf, int qb, int slot) {
      if (lane == 0) {
        const uint32_t b_base = k_lo + static_cast<uint32_t>((slot * S::kTileBytes) >> 4);
#pragma unroll
        for (int kk = 0; kk < 4 * NB; ++kk) {
          if (kk < ksteps_qk) {
            const uint32_t b_off = static_cast<uint32_t>(((kk >> 2) * BN * 128 + (kk & 3) * 32) >> 4);
            umma_f16_ts_w(tmem + buf * 128u, tmem + S::q_col(qb) + 8u * kk, b_base + b_off, kHi, idesc_qk,
                          kk > 0 ? 1u : 0u);
          }
        }
        umma_commit(&s_full[buf]);
        umma_commit(&k_empty[slot]);
      }
    };
    // O += P V over the tile's 128 keys: P of key half h from the first 32 columns of half h of S[buf], V rows
    // from ring slot `slot`; frees the V slot.
    auto pv = [&](uint32_t buf, int slot, bool first) {
      if (lane == 0) {
        const uint32_t b_base = v_lo + static_cast<uint32_t>((slot * S::kTileBytes) >> 4);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // 16-key steps
          const uint32_t a_col = buf * 128u + 64u * (kk >> 2) + 8u * (kk & 3);
          umma_f16_ts_w(tmem + S::kColO, tmem + a_col, b_base + static_cast<uint32_t>((kk * 16 * 128) >> 4), kHi,
                        idesc_pv, (!first || kk > 0) ? 1u : 0u);
        }
        umma_commit(pv_done);
        umma_commit(&v_empty[slot]);
      }
    };
    TileCursor cur, ahead;  // tile g and tile g + 2
    tile_cursor_init(a, cur);
    tile_cursor_init(a, ahead);
    // QK of the tile `ahead` points at (index u) into S[u % 2]
    auto issue_qk = [&](uint32_t u) {
      const int qb = ahead.seg & 1;
      if (ahead.j == 0) wait_lane0(&q_ready[qb], (ahead.seg >> 1) & 1, 75);
      wait_lane0(&k_full[u % NS], (u / NS) & 1, 76);
      if (ok) {
        tc_fence_after_sync();
        qk(u & 1, qb, u % NS);
        if (lane == 0 && ahead.j + 1 == ahead.c.n) umma_commit(&q_free[qb]);  // every QK of the segment issued
      }
      tile_cursor_advance(a, ahead);
    };
    for (uint32_t u = 0; u < 2 && ahead.valid; ++u) issue_qk(u);  // prologue: S of the first two tiles
    uint32_t g = 0;
    while (cur.valid) {
      const uint32_t buf = g & 1;
      __syncwarp();
      named_barrier_sync(S::kBarP + buf, S::kBarPThreads);  // both halves of P(g) are in TMEM
      wait_lane0(&v_full[g % NS], (g / NS) & 1, 77);
      if (ok) {
        tc_fence_after_sync();
        pv(buf, g % NS, cur.j == 0);
        if (lane == 0 && cur.j + 1 == cur.c.n) umma_commit(o_full);  // the segment's O is complete
      }
      if (ahead.valid) issue_qk(g + 2);  // S[buf] takes tile g + 2 (P(g) is consumed first, in issue order)
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
    // Warpgroup 1 (warps 4-7) owns keys [0, 64) of every tile and the first half of the columns of Q and O;
    // warpgroup 2 (warps 8-11) keys [64, 128) and the second half. A warp may only touch the TMEM lane quarter
    // warp % 4, so each warpgroup covers all 128 rows.
    setmaxnreg_inc<S::kRegsSoftmax>();
    const int half = (warp - 4) / 4;
    const int row = (warp % 4) * 32 + lane;  // TMEM lane = query row within the tile
    const uint32_t lane_base = static_cast<uint32_t>((warp % 4) * 32) << 16;
    const int dh = D / 2;  // this warpgroup's elements of each Q row
    // this warpgroup's columns of O: [o_lo, o_lo + o_n), split on a 16-column boundary (TMEM loads of 16 columns)
    const int o_split = min(D, (D / 2 + 15) / 16 * 16);
    const int o_lo = half ? o_split : 0;
    const int o_n = half ? D - o_split : o_split;
    const uint32_t o_own = tmem + lane_base + S::kColO + static_cast<uint32_t>(o_lo);
    bool ok = true;
    uint32_t g = 0, segs_done = 0;
    auto wait_warp = [&](uint64_t* bar, uint32_t parity, int site) {
      if (ok) {
        ok = __all_sync(0xffffffffu, mbar_wait(bar, parity, a.budget_ns));
        if (!ok && lane == 0) record_error(a.ws, FGW_ERR_DEVICE_TIMEOUT, site);
      }
      return ok;
    };
    // Q of the next segment with tiles, into TMEM buffer (its index) % 2: this thread's row, this warpgroup's half
    // of the head dimension, as packed 16-bit pairs (element 2c in the low half of column c), the layout of an A
    // operand read from TMEM. Rows past the query length are zeros.
    TileCursor qcur;
    tile_cursor_init(a, qcur);
    auto write_next_q = [&]() {
      if (!qcur.valid) return;
      const int qb = qcur.seg & 1;
      if (qcur.seg >= 2) wait_warp(&q_free[qb], ((qcur.seg - 2) >> 1) & 1, 88);
      const int qrow = qcur.c.q0 + row;
      const uint4* src = reinterpret_cast<const uint4*>(
          reinterpret_cast<const T*>(a.q) +
          (((long long)qcur.c.b * a.sq + min(qrow, a.sq - 1)) * a.heads + qcur.c.h) * D + dh * half);
      const uint32_t dst = tmem + lane_base + S::q_col(qb) + static_cast<uint32_t>(dh / 2 * half);
      if (ok) {
        for (int w = 0; w < dh / 8; ++w) {  // 8 elements (4 columns) per step
          const uint4 v = qrow < a.sq ? src[w] : make_uint4(0, 0, 0, 0);
          tmem_st4(dst + 4 * w, v.x, v.y, v.z, v.w);
        }
        tmem_wait_st();
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&q_ready[qb]);
      // past the segment's tiles: the next segment with tiles
      qcur.j = qcur.c.n - 1;
      tile_cursor_advance(a, qcur);
    };
    write_next_q();  // segment 0
    SegmentWalk walk;
    segment_walk_init(a, walk);
    HalvesSegment sg;
    HalvesItem c;
    volatile int* merge_flag = reinterpret_cast<volatile int*>(smem + S::kTmemSlot + 4);
    while (segment_walk_next(a, walk, sg, c)) {
      if (c.n > 0) write_next_q();  // the following segment's Q, while this one runs
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
        // the row's maximum over both key halves
        xmax[((g & 1) * 2 + half) * 128 + row] = mx_raw;
        __syncwarp();
        named_barrier_sync(S::kBarX, 256);
        mx_raw = fmaxf(mx_raw, xmax[((g & 1) * 2 + (half ^ 1)) * 128 + row]);
        const float mx = mx_raw * a.scale_log2;  // scale > 0; -inf stays -inf
        float m_new = m;
        bool grow = false;
        if (j == 0) {
          m_new = mx;
        } else if (mx > m + 8.0f) {
          grow = true;
        }
        // the same rows, maxima and running max in both warpgroups: both take the same decision
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
        // this warpgroup's columns of O may be rescaled only once PV(g - 1) has completed (at most that PV is
        // outstanding here)
        if (warp_grow && j > 0) {
          wait_warp(pv_done, (g - 1) & 1, 82 + half);
          if (ok) {
            tc_fence_after_sync();
            for (int cb = 0; cb < o_n / 16; ++cb) {
              uint32_t r[16];
              tmem_ld16(o_own + cb * 16, r);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
              tmem_st16(o_own + cb * 16, r);
            }
          }
        }
        // Value rows past the cache end: this half's rows of V(g) are zeroed before P is released (PV reads them)
        if (tok0 + BN > c.len) {
          wait_warp(&v_full[g % NS], (g / NS) & 1, 84 + half);
          const int vrow = 64 * half + row;
          if (ok && row < 64 && tok0 + vrow >= c.len) {
            uint8_t* dst = v_smem + (g % NS) * S::kTileBytes + vrow * 128;
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
        wait_warp(o_full, segs_done & 1, 86 + half);  // the segment's last PV has completed
        ++segs_done;
      }
      // epilogue: the row sum over both halves, then each warpgroup normalises and stores its half of the row
      xsum[half * 128 + row] = l;
      __syncwarp();  // the named barriers are the aligned form: the warp arrives converged
      named_barrier_sync(S::kBarX, 256);
      const float lt = l + xsum[(half ^ 1) * 128 + row];
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      const float lse = (c.n > 0 && lt > 0.f) ? m + fast_log2(lt) : kEmptyLse;
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
      for (int cb = 0; cb < o_n / 16; ++cb) {
        float o[16];
        if (read_o) {  // warp-collective: every lane, valid row or not
          uint32_t r[16];
          tmem_ld16(o_own + cb * 16, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = __uint_as_float(r[i]) * inv;
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = 0.f;
        }
        const int col = o_lo + cb * 16;
        if (row_valid && sg.piece) {
          float4* dst = reinterpret_cast<float4*>(a.slot_o + (my_slot * 128 + row) * D + col);
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
        } else if (row_valid && a.write_partials) {
          float4* dst = reinterpret_cast<float4*>(a.part_o + (row_id * a.splits + c.s) * D + col);
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
        } else if (row_valid) {
          uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<T*>(a.out) + row_id * D + col);
          dst[0] = make_uint4(Tr::pack2(o[0], o[1]), Tr::pack2(o[2], o[3]), Tr::pack2(o[4], o[5]),
                              Tr::pack2(o[6], o[7]));
          dst[1] = make_uint4(Tr::pack2(o[8], o[9]), Tr::pack2(o[10], o[11]), Tr::pack2(o[12], o[13]),
                              Tr::pack2(o[14], o[15]));
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
        named_barrier_sync(S::kBarX, 256);  // both warpgroups have written their halves
        const long long total = a.prog_u[a.programs];
        const int q_first = program_of(total, a.programs, sg.item_u);
        const int pieces = program_of(total, a.programs, sg.item_u + sg.units - 1) - q_first + 1;
        const int first_extra = sg.item_u != program_start(total, a.programs, q_first) ? 1 : 0;
        if (warp == 4 && lane == 0) *merge_flag = atomicAdd(&a.counters[sg.item], 1) + 1 == pieces ? 1 : 0;
        __syncwarp();
        named_barrier_sync(S::kBarX, 256);
        const int merge = *merge_flag;
        if (merge) {
          __threadfence();
          if (warp == 4 && lane == 0) a.counters[sg.item] = 0;  // ready for the next launch
        }
        if (merge && row_valid) {
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
          for (int cb = 0; cb < o_n / 16; ++cb) {
            const int col = o_lo + cb * 16;
            float acc[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) acc[i] = 0.f;
            for (int k = 0; k < pieces; ++k) {
              const long long pr = piece_slot(q_first, first_extra, k) * 128 + row;
              const float lk = __ldcg(&a.slot_lse[pr]);
              if (!(lk > kValidLse)) continue;
              const float w = fast_exp2(lk - peak);
              const float4* src = reinterpret_cast<const float4*>(a.slot_o + pr * D + col);
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const float4 v = __ldcg(src + i);
                acc[4 * i] += w * v.x;
                acc[4 * i + 1] += w * v.y;
                acc[4 * i + 2] += w * v.z;
                acc[4 * i + 3] += w * v.w;
              }
            }
            uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<T*>(a.out) + row_id * D + col);
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
static cudaError_t launch_halves_t(const LaunchDesc& d, const HalvesArgs& args, const CUtensorMap& kmap,
                                   const CUtensorMap& vmap) {
  using S = HalvesShape<NB>;
  auto kernel = fmha_halves_sm100_kernel<T, NB>;
  // setmaxnreg.inc only succeeds if the registers the block was launched with cover the new split (see
  // launch_fmha2_t); refuse a build whose allocation would not cover it.
  int regs = 0;
  cudaError_t err = prepare_kernel(reinterpret_cast<const void*>(kernel), S::kBytes, d.device, &regs);
  if (err != cudaSuccess) return err;
  const int allocated = ((regs + 7) / 8) * 8 * S::kThreads;
  if (allocated < 4 * 32 * S::kRegsControl + 8 * 32 * S::kRegsSoftmax) return cudaErrorNotSupported;
  const long long cap = d.p.grid_cap > 0 ? d.p.grid_cap : d.sm_count;
  // contiguous schedule: one CTA per program of the plan; strided: persistent CTAs over the items
  const long long grid = args.contiguous ? args.programs
                                         : std::min<long long>(args.items, std::min<long long>(cap, d.sm_count));
  if (grid <= 0) return cudaSuccess;
  return launch_after_plan(kernel, (unsigned)grid, S::kThreads, S::kBytes, d.stream, kmap, vmap, args);
}

cudaError_t launch_tensor_halves(const LaunchDesc& d, bool write_partials, const CUtensorMap& kmap,
                                 const CUtensorMap& vmap, int box_rows) {
  const fgw_mha_params& p = d.p;
  HalvesArgs args;
  args.q = p.q;
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
    return bf16 ? launch_halves_t<__nv_bfloat16, 1>(d, args, kmap, vmap)
                : launch_halves_t<__half, 1>(d, args, kmap, vmap);
  }
  if (p.head_dim <= 128) {
    return bf16 ? launch_halves_t<__nv_bfloat16, 2>(d, args, kmap, vmap)
                : launch_halves_t<__half, 2>(d, args, kmap, vmap);
  }
  return cudaErrorInvalidValue;
}

}  // namespace fgw
