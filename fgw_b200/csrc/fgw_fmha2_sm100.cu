// Two-query-tile tensor-core paged attention for head dims up to 128 (the long-query workhorse).
//
// Same contract and masking rules as fmha_sm100_kernel (fgw_fmha_sm100.cu), which it replaces for D <= 128;
// the reference body it stands for is operators/mha/kernels/mha_paged_decode_ascend_v7.py:225-315, 375-465.
// What changes is the schedule:
//   * a work item is a pair of 128-row query tiles (A, B) of one (request, head, split); both share every
//     K/V tile, so K/V shared-memory traffic per FLOP halves;
//   * two softmax warpgroups (warps 4-7 for A, 8-11 for B) ping-pong on the tensor core. The MMA warp
//     issues, per KV tile j:  PV_A(j), QK_A(j+1), PV_B(j), QK_B(j+1)  so the softmax of A(j+1)
//     overlaps PV_B(j) + QK_B(j+1) and the softmax of B(j) overlaps PV_A(j) + QK_A(j+1);
//   * P never touches shared memory: each softmax thread writes its bf16/fp16 P row back into the TMEM
//     columns of the S row it has just consumed, and PV reads P straight from TMEM (tcgen05.mma with the
//     A operand in tensor memory);
//   * P_t(j) is released in two halves of 64 keys, so PV over the first half overlaps the exponentials of
//     the second;
//   * a commit after QK_t(j+1) also covers the earlier PV_t(j), so a softmax thread that has seen S_t(j+1)
//     may rescale O_t in TMEM without a separate wait.
// TMEM: S_A [0,128), S_B [128,256), O_A [256,256+D), O_B [384,384+D) of 512 columns.
#include <algorithm>

#include "fgw_common.cuh"
#include "fgw_kernels.h"

namespace fgw {

struct Fmha2Args {
  void* out;
  const int32_t* table;
  const int32_t* lengths;
  const int32_t* order;
  float* part_o;
  float* part_lse;
  WorkspaceHeader* ws;
  int batch, sq, heads, dim, width, page, splits, causal, box_rows, write_partials, qpairs;
  long long items;
  // contiguous schedule (see fgw_schedule): per-program start item / unit offset / first unit, the
  // per-item arrival counters and the two partial slots of every program
  int contiguous, programs;
  int tail_start;  // items below it are whole items of the full waves, dealt strided (tail schedule)
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
struct Fmha2Shape {
  static constexpr int kBN = 128;
  static constexpr int kTileBytes = 128 * 128;           // one 64-col block of a 128-row operand
  static constexpr int kQBytes = NB * kTileBytes;        // one 128-row query tile
  static constexpr int kKVBytes = NB * kBN * 128;        // one K (or V) stage
  static constexpr int kStages = NB == 1 ? 4 : 2;
  static constexpr int kThreads = 384;
  // registers per thread after the warpgroup split (4 x 32 x 88 + 8 x 32 x 208 = 384 x 168)
  static constexpr int kRegsControl = 88;
  static constexpr int kRegsSoftmax = 208;
  // full tiles evaluate one exponential pair in kFmaEvery on the FMA pipe (0: all on the SFU)
  static constexpr int kFmaEvery = 0;
  // TMEM column of S_t / O_t for query tile t
  __device__ __forceinline__ static uint32_t s_col(int t) { return static_cast<uint32_t>(t) * 128u; }
  __device__ __forceinline__ static uint32_t o_col(int t) { return 256u + static_cast<uint32_t>(t) * 128u; }
  static constexpr int kTmemCols = 512;
  // shared memory carve-up
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + 2 * kQBytes;
  static constexpr int kV = kK + kStages * kKVBytes;
  static constexpr int kBar = kV + kStages * kKVBytes;
  // q_full, q_empty, k_full[S], k_empty[S], v_full[S], v_empty[S], s_full[2], p_full[2], pv_done[2],
  // o_empty[2], mma_done, p_half[2]
  static constexpr int kNumBars = 2 + 4 * kStages + 8 + 1 + 2;
  static constexpr int kTmemSlot = kBar + kNumBars * 8;
  static constexpr int kBytes = kTmemSlot + 16 + 1024;
};

// max(a, b, c) in one instruction (sm_100 three-input max; NaN-free inputs here)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

struct PairItem {
  int b, h, s, q0, len, n_begin, n, n_tile[2];
};

__device__ __forceinline__ int visible_upto(int row, int len, int sq, int causal) {
  return causal ? max(len - sq + row + 1, 0) : len;
}

__device__ __forceinline__ void pair_item(const Fmha2Args& a, long long item, PairItem& c) {
  const int p_rev = static_cast<int>(item % a.qpairs);
  long long rest = item / a.qpairs;
  c.s = static_cast<int>(rest % a.splits);
  rest /= a.splits;
  c.h = static_cast<int>(rest % a.heads);
  c.b = a.order[rest / a.heads];
  c.q0 = (a.qpairs - 1 - p_rev) * 256;  // later pairs first: they see the most keys when causal
  c.len = a.lengths[c.b];
  const int last = min(c.q0 + 256, a.sq) - 1;
  const int tiles = (visible_upto(last, c.len, a.sq, a.causal) + 127) / 128;
  c.n_begin = static_cast<int>((long long)tiles * c.s / a.splits);
  const int n_end = static_cast<int>((long long)tiles * (c.s + 1) / a.splits);
  c.n = n_end - c.n_begin;
  const int last_a = min(c.q0 + 128, a.sq) - 1;
  const int tiles_a = (visible_upto(last_a, c.len, a.sq, a.causal) + 127) / 128;
  c.n_tile[0] = max(0, min(n_end, tiles_a) - c.n_begin);
  c.n_tile[1] = (c.q0 + 128 < a.sq) ? c.n : 0;
}

// 2^(s * scale - m) for 64 consecutive scores (32 FP32 pairs, scale-and-subtract two lanes per
// instruction), summed into four independent partial sums and packed to 16-bit pairs. With kFmaEvery = k > 0,
// one pair in k is evaluated by poly_exp2_pair on the FMA pipe so that the SFU and FMA pipes share the
// work; only used on tiles without masked (-inf) scores, since poly_exp2_pair clamps its input.
template <typename Tr, int kFmaEvery>
__device__ __forceinline__ void exp2_pack_half(const uint32_t* sr, float2 scale2, float2 negm2, float2 (&acc)[4],
                                               uint32_t (&packed)[32]) {
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const float2 x = __ffma2_rn(make_float2(__uint_as_float(sr[2 * i]), __uint_as_float(sr[2 * i + 1])), scale2, negm2);
    float2 p;
    if (kFmaEvery > 0 && (i % (kFmaEvery > 0 ? kFmaEvery : 1)) == kFmaEvery - 1) {
      p = poly_exp2_pair(x);
    } else {
      p = make_float2(fast_exp2(x.x), fast_exp2(x.y));
    }
    packed[i] = Tr::pack2(p.x, p.y);
    // the row sum adds the rounded values PV multiplies: with the lazily rescaled running max a row's largest P
    // may exceed 1 and round, and normalising by the unrounded sum would leave that rounding in the output. The
    // 16-bit values go straight into FP32 adds (the same sums as unpacking first, two instructions fewer per
    // pair: config 2 89.1 against 91.1 us)
    acc[i % 4] = Tr::add2(acc[i % 4], packed[i]);
  }
}

// One run of KV tiles of one work item processed by this CTA. With the strided schedule a segment is a
// whole item; with the contiguous schedule it may be a piece of an item cut between programs.
struct Segment {
  PairItem c;        // n_begin / n / n_tile[] restricted to the segment's KV tiles
  int item;
  bool piece;        // the item's other tiles belong to other programs
  long long item_u;  // first unit of the item (contiguous schedule)
  long long u0;      // first unit of this segment (contiguous schedule)
  int units;         // units of the whole item (contiguous schedule)
};

struct SegmentCursor {
  long long round;  // next round of whole items (strided part, snake order)
  long long item;
  int off;
  long long u, u_end;
};

__device__ __forceinline__ void cursor_init(const Fmha2Args& a, SegmentCursor& k) {
  k.round = 0;
  if (a.contiguous) {
    k.item = a.prog_item[blockIdx.x];
    k.off = a.prog_off[blockIdx.x];
    k.u = a.prog_u[blockIdx.x];
    k.u_end = a.prog_u[blockIdx.x + 1];
  } else {
    k.item = 0;
    k.off = 0;
    k.u = k.u_end = 0;
  }
}

// Every role of the CTA walks the same segments in the same order: whole items first (all of them with the
// strided schedule, those of the full waves with the tail schedule), then its contiguous range of units.
__device__ __forceinline__ bool next_segment(const Fmha2Args& a, SegmentCursor& k, Segment& sg) {
  const long long whole_end = a.contiguous ? a.tail_start : a.items;
  const long long whole = snake_item(k.round);
  if (whole < whole_end) {
    sg.item = static_cast<int>(whole);
    pair_item(a, whole, sg.c);
    sg.piece = false;
    sg.item_u = sg.u0 = 0;
    sg.units = 0;
    ++k.round;
    return true;
  }
  if (!a.contiguous) return false;
  if (k.u >= k.u_end) return false;
  sg.item = static_cast<int>(k.item);
  pair_item(a, k.item, sg.c);  // one split: the whole item
  const int tiles = sg.c.n;
  sg.units = max(tiles, 1);    // an item without keys still costs one unit (its rows are written as zeros)
  const int first = k.off;
  const int count = static_cast<int>(min(static_cast<long long>(sg.units - first), k.u_end - k.u));
  sg.u0 = k.u;
  sg.item_u = k.u - first;
  sg.piece = count < sg.units;
  const int tiles_a = sg.c.n_tile[0];
  const bool has_b = sg.c.n_tile[1] > 0;
  const int real = max(0, min(first + count, tiles) - first);
  sg.c.n_begin = first;
  sg.c.n = real;
  sg.c.n_tile[0] = max(0, min(first + count, tiles_a) - first);
  sg.c.n_tile[1] = has_b ? real : 0;
  k.u += count;
  k.off += count;
  if (k.off >= sg.units) {
    ++k.item;
    k.off = 0;
  }
  return true;
}

template <typename T, int NB>
__global__ void __launch_bounds__(384, 1)
    fmha2_sm100_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                       const __grid_constant__ CUtensorMap vmap, const Fmha2Args a) {
  using S = Fmha2Shape<NB>;
  using Tr = ElemTraits<T>;
  constexpr int BN = S::kBN;
  constexpr int NS = S::kStages;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* q_smem = smem + S::kQ;
  uint8_t* k_smem = smem + S::kK;
  uint8_t* v_smem = smem + S::kV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kBar);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;
  uint64_t* k_empty = k_full + NS;
  uint64_t* v_full = k_empty + NS;
  uint64_t* v_empty = v_full + NS;
  uint64_t* s_full = v_empty + NS;  // [2]
  uint64_t* p_full = s_full + 2;    // [2]
  uint64_t* pv_done = p_full + 2;   // [2]
  uint64_t* o_empty = pv_done + 2;  // [2]
  uint64_t* mma_done = o_empty + 2;
  uint64_t* p_half = mma_done + 1;  // [2]: the first 64 keys of P_t are in TMEM
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::kTmemSlot);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < NS; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 4);   // one arrival per softmax warp
      mbar_init(&p_half[t], 4);
      mbar_init(&pv_done[t], 1);
      mbar_init(&o_empty[t], 4);
    }
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
    // The whole warp walks the segments converged; lane 0 issues the copies. The block-table entries of an item
    // are read 32 pages at a time, one per lane, before the item's first wait, and broadcast per box, so no
    // table read sits between an empty-slot wait and the copy it gates (config 2: 103.4 against 105.5 us with a
    // lone lane 0 reading the table per box).
    {
      if (lane == 0) {
        tma_prefetch_desc(&qmap);
        tma_prefetch_desc(&kmap);
        tma_prefetch_desc(&vmap);
      }
      bool ok = true;
      uint32_t kc = 0, vc = 0, qc = 0;
      const int boxes = BN / a.box_rows;
      const uint32_t box_bytes = a.box_rows * 128;
      auto wait_or_fail = [&](uint64_t* bar, uint32_t parity, int site) {
        if (ok && !__all_sync(0xffffffffu, mbar_wait(bar, parity, a.budget_ns))) {
          ok = false;
          if (lane == 0) record_error(a.ws, FGW_ERR_DEVICE_TIMEOUT, site);
        }
        return ok;
      };
      SegmentCursor cur;
      cursor_init(a, cur);
      Segment sg;
      while (__shfl_sync(0xffffffffu, static_cast<int>(next_segment(a, cur, sg)), 0)) {
        PairItem c = sg.c;  // the fields this role branches on, made warp-uniform
        c.n = __shfl_sync(0xffffffffu, c.n, 0);
        c.n_tile[1] = __shfl_sync(0xffffffffu, c.n_tile[1], 0);
        if (c.n <= 0) continue;
        const int32_t* row_table = a.table + (long long)c.b * a.width;
        TableWindow table;
        table.init(row_table, a.width, (c.n_begin * BN) / a.page, lane);
        if (wait_or_fail(q_empty, (qc & 1) ^ 1, 40) && lane == 0) {
          const int tiles_q = c.n_tile[1] > 0 ? 2 : 1;
          mbar_arrive_expect_tx(q_full, tiles_q * S::kQBytes);
          for (int t = 0; t < tiles_q; ++t) {
            for (int blk = 0; blk < NB; ++blk) {
              tma_load_4d(q_smem + t * S::kQBytes + blk * S::kTileBytes, &qmap, q_full, blk * 64, c.h,
                          c.q0 + 128 * t, c.b);
            }
          }
        }
        ++qc;
        for (int j = 0; j < c.n; ++j) {
          const int tok0 = (c.n_begin + j) * BN;
          int nbox = 0;
          for (int k = 0; k < boxes; ++k) nbox += (tok0 + k * a.box_rows < c.len) ? 1 : 0;
          // K tile, then V tile of KV step j
#pragma unroll
          for (int which = 0; which < 2; ++which) {
            const uint32_t cnt = which == 0 ? kc : vc;
            uint64_t* full = which == 0 ? k_full : v_full;
            uint64_t* empty = which == 0 ? k_empty : v_empty;
            const CUtensorMap* map = which == 0 ? &kmap : &vmap;
            uint8_t* ring = which == 0 ? k_smem : v_smem;
            const int st = cnt % NS;
            if (wait_or_fail(&empty[st], ((cnt / NS) & 1) ^ 1, 41 + which)) {
              if (lane == 0) mbar_arrive_expect_tx(&full[st], NB * nbox * box_bytes);
              uint8_t* dst = ring + st * S::kKVBytes;
              for (int k = 0; k < nbox; ++k) {
                const int tok = tok0 + k * a.box_rows;
                const int pg = tok / a.page;  // < width: only boxes before the cache end are loaded
                const int row = table.page(pg, lane) * a.page + tok % a.page;
                if (lane == 0) {
                  for (int blk = 0; blk < NB; ++blk) {
                    tma_load_3d(dst + blk * BN * 128 + k * box_bytes, map, &full[st], blk * 64, c.h, row);
                  }
                }
              }
            }
          }
          ++kc;
          ++vc;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------------- UMMA issuer
    // The whole warp runs this role converged, with its loop state kept warp-uniform (segment fields are
    // broadcast from lane 0), and every tcgen05 issue is predicated on one elected lane. Against a lone lane 0
    // running the same code this measured 105.4 against 111.6 us on config 2 (619 against 654 us at Q = 32768).
    {
      const uint32_t leader = elect_one_sync();
      const uint32_t tmem_u = __shfl_sync(0xffffffffu, tmem, 0);
      bool ok = true;
      uint32_t kc = 0, vc = 0, qc = 0;
      uint32_t pbits = 0, obits = 0;  // bit t: phase parity of p_full[t] / o_empty[t] uses
      const int fmt = Tr::kUmmaFormat;
      const uint32_t idesc_qk = umma_idesc_f16(fmt, 128, BN, 0, 0);
      const uint32_t idesc_pv = umma_idesc_f16(fmt, 128, D, 0, 1);
      // Descriptor words: each issue below only adds a constant to a low word.
      uint32_t q_lo = umma_desc_lo(smem_u32(q_smem), 16);
      uint32_t k_lo = umma_desc_lo(smem_u32(k_smem), 16);
      uint32_t v_lo = umma_desc_lo(smem_u32(v_smem), BN * 128);
      constexpr uint32_t kHi = umma_desc_hi(1024, 2);
      const int ksteps_qk = D / 16;
      auto wait_or_fail = [&](uint64_t* bar, uint32_t parity, int site) {
        if (ok && !__all_sync(0xffffffffu, mbar_wait(bar, parity, a.budget_ns))) {
          ok = false;
          if (lane == 0) record_error(a.ws, FGW_ERR_DEVICE_TIMEOUT, site);
        }
        return ok;
      };
      // Several phases (null entries are skipped), waited for in turn with try_wait, which suspends the warp
      // until the phase completes or a hardware time limit passes: the buffers first, the tile's P (b0), the one
      // usually still pending, last. With the converged warp this measured 97.3 against 101.4 us on config 2
      // (578 against 611 us at Q = 32768) over polling all four with test_wait in one loop.
      auto wait_all_or_fail = [&](uint64_t* b0, uint32_t p0, uint64_t* b1, uint32_t p1, uint64_t* b2, uint32_t p2,
                                  uint64_t* b3, uint32_t p3, int site) {
        if (!ok) return false;
        const bool got = (b1 == nullptr || mbar_wait(b1, p1, a.budget_ns)) &&
                         (b2 == nullptr || mbar_wait(b2, p2, a.budget_ns)) &&
                         (b3 == nullptr || mbar_wait(b3, p3, a.budget_ns)) &&
                         (b0 == nullptr || mbar_wait(b0, p0, a.budget_ns));
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          if (lane == 0) record_error(a.ws, FGW_ERR_DEVICE_TIMEOUT, site);
        }
        return ok;
      };
      // S_t = Q_t K^T into TMEM, K from stage `st` (already waited for).
      auto qk = [&](int t, int st) {
        const uint32_t a_lo = q_lo + static_cast<uint32_t>((t * S::kQBytes) >> 4);
        const uint32_t b_lo = k_lo + static_cast<uint32_t>((st * S::kKVBytes) >> 4);
#pragma unroll
        for (int kk = 0; kk < 4 * NB; ++kk) {
          if (kk < ksteps_qk) {
            umma_f16_ss_e(leader, tmem_u + S::s_col(t), a_lo + (((kk >> 2) * S::kTileBytes + (kk & 3) * 32) >> 4), kHi,
                          b_lo + (((kk >> 2) * BN * 128 + (kk & 3) * 32) >> 4), kHi, idesc_qk, kk > 0 ? 1u : 0u);
          }
        }
        umma_commit_e(leader, &s_full[t]);
      };
      // O_t += P_t V: P_t read from TMEM (packed into the first 64 columns of S_t), V from stage `st`.
      // The P column and V descriptor advance by one step per MMA through opaque registers: with all eight
      // operand pairs formed up front the issuer needs more than the control warpgroup's registers and
      // spills, and the reloads sit between the MMA issues.
      auto pv = [&](int t, int st, bool first, int k0) {
        uint32_t b_lo = v_lo + static_cast<uint32_t>((st * S::kKVBytes) >> 4) + k0 * ((16 * 128) >> 4);
        uint32_t p_col = tmem_u + S::s_col(t) + k0 * 8;
        const uint32_t o_tmem = tmem_u + S::o_col(t);
#pragma unroll
        for (int kk = k0; kk < k0 + BN / 32; ++kk) {
          umma_f16_ts_e(leader, o_tmem, p_col, b_lo, kHi, idesc_pv, (!first || kk > 0) ? 1u : 0u);
          p_col += 8;
          b_lo += (16 * 128) >> 4;
          asm volatile("" : "+r"(p_col), "+r"(b_lo));
        }
      };
      SegmentCursor cur;
      cursor_init(a, cur);
      Segment sg;
      while (__shfl_sync(0xffffffffu, static_cast<int>(next_segment(a, cur, sg)), 0)) {
        PairItem c = sg.c;  // the fields this role branches on, made warp-uniform
        c.n = __shfl_sync(0xffffffffu, c.n, 0);
        c.n_tile[0] = __shfl_sync(0xffffffffu, c.n_tile[0], 0);
        c.n_tile[1] = __shfl_sync(0xffffffffu, c.n_tile[1], 0);
        if (c.n <= 0) continue;
        // prologue: S_A(0), S_B(0) once Q and K(0) are in
        int kst = kc % NS;
        if (wait_all_or_fail(q_full, qc & 1, &k_full[kst], (kc / NS) & 1, nullptr, 0, nullptr, 0, 50)) {
          tc_fence_after_sync();
          for (int t = 0; t < 2; ++t) {
            if (c.n_tile[t] > 0) qk(t, kst);
          }
          umma_commit_e(leader, &k_empty[kst]);
        }
        ++qc;
        ++kc;
        if (c.n == 1 && ok) umma_commit_e(leader, q_empty);
        for (int j = 0; j < c.n; ++j) {
          // Opaque to the compiler, so the descriptor sums are formed where they are used instead of being
          // hoisted out of the loops (which would keep one register per stage and step live).
          asm volatile("" : "+r"(q_lo), "+r"(k_lo), "+r"(v_lo));
          const int vst = vc % NS;
          const uint32_t v_par = (vc / NS) & 1;
          ++vc;
          const bool more = j + 1 < c.n;
          const int knext = kc % NS;
          const uint32_t k_par = (kc / NS) & 1;
          bool v_seen = false, k_seen = !more;
#pragma unroll 1
          for (int t = 0; t < 2; ++t) {
            const int nt = t ? c.n_tile[1] : c.n_tile[0];
            const bool pv_t = j < nt;
            const bool qk_t = more && j + 1 < nt;
            if (pv_t || qk_t) {
              // the first half of this tile's P, the V tile, the next K tile and (first tile of an item) an empty O
              const bool ready = wait_all_or_fail(pv_t ? &p_half[t] : nullptr, (pbits >> t) & 1,
                                                  (pv_t && !v_seen) ? &v_full[vst] : nullptr, v_par,
                                                  (qk_t && !k_seen) ? &k_full[knext] : nullptr, k_par,
                                                  (pv_t && j == 0) ? &o_empty[t] : nullptr,
                                                  ((obits >> t) & 1) ^ 1, 53 + t);
              v_seen = v_seen || pv_t;
              k_seen = k_seen || qk_t;
              if (ready) {
                tc_fence_after_sync();
                if (pv_t) {
                  // PV over the first 64 keys once that half of P is stored, the rest once all of it is (config 2:
                  // 97.3 against 99.3 us, Q = 32768: 555 against 580 us, over waiting for the whole of P)
                  pv(t, vst, j == 0, 0);
                  if (wait_all_or_fail(&p_full[t], (pbits >> t) & 1, nullptr, 0, nullptr, 0, nullptr, 0, 55 + t)) {
                    tc_fence_after_sync();
                    pv(t, vst, false, BN / 32);
                    if (j + 1 == nt) umma_commit_e(leader, &pv_done[t]);
                  }
                }
                if (qk_t) qk(t, knext);
              }
            }
            if (pv_t) pbits ^= 1u << t;
          }
          if (ok) umma_commit_e(leader, &v_empty[vst]);
          if (more) {
            if (ok) umma_commit_e(leader, &k_empty[knext]);
            ++kc;
            if (j + 2 == c.n && ok) umma_commit_e(leader, q_empty);  // every QK of this item is now issued
          }
        }
        if (c.n_tile[0] > 0) obits ^= 1u;
        if (c.n_tile[1] > 0) obits ^= 2u;
      }
      if (ok) {
        umma_commit_e(leader, mma_done);
        __all_sync(0xffffffffu, mbar_wait(mma_done, 0, a.budget_ns));
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------------- softmax / epilogue
    // Warpgroup 1 (warps 4-7) owns query tile A, warpgroup 2 (warps 8-11) tile B. A warp may only
    // touch the TMEM lane quarter warp % 4, so each warpgroup covers all 128 rows.
    setmaxnreg_inc<S::kRegsSoftmax>();
    const int t = (warp - 4) / 4;                    // query tile A (0) or B (1)
    const int row = (warp % 4) * 32 + lane;          // TMEM lane = query row within the tile
    const uint32_t lane_base = static_cast<uint32_t>((warp % 4) * 32) << 16;
    const uint32_t s_addr = tmem + lane_base + S::s_col(t);
    const uint32_t o_addr = tmem + lane_base + S::o_col(t);
    bool ok = true;
    uint32_t sc = 0, pd = 0, vbase = 0;
    auto wait_warp = [&](uint64_t* bar, uint32_t parity, int site) {
      if (ok) {
        ok = __all_sync(0xffffffffu, mbar_wait(bar, parity, a.budget_ns));
        if (!ok && lane == 0) record_error(a.ws, FGW_ERR_DEVICE_TIMEOUT, site);
      }
      return ok;
    };
    volatile int* merge_flag = reinterpret_cast<volatile int*>(smem + S::kTmemSlot + 4);
    SegmentCursor cur;
    cursor_init(a, cur);
    Segment sg;
    while (next_segment(a, cur, sg)) {
      const PairItem& c = sg.c;
      const int q = c.q0 + 128 * t + row;
      const bool row_valid = q < a.sq;
      const int vis = row_valid ? visible_upto(q, c.len, a.sq, a.causal) : 0;
      const int n_t = t == 0 ? c.n_tile[0] : c.n_tile[1];
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < n_t; ++j) {
        const int tok0 = (c.n_begin + j) * BN;
        wait_warp(&s_full[t], sc & 1, 60 + t);
        ++sc;
        const int valid_cols = min(max(vis - tok0, 0), BN);
        const bool tail = valid_cols < BN;  // masking only on tail / diagonal tiles
        // The whole S row in registers with one wait.
        uint32_t sr[BN];
        if (ok) {
          tc_fence_after_sync();
#pragma unroll
          for (int cb = 0; cb < BN / 64; ++cb) {  // two 64-column loads (Q32768: 544 against 550 us with four of 32)
            tmem_ld64(s_addr + cb * 64, *reinterpret_cast<uint32_t(*)[64]>(&sr[cb * 64]));
          }
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < BN; ++i) sr[i] = __float_as_uint(-INFINITY);
        }
        if (tail) {
          // ragged / diagonal tile: mask columns at or past this row's visible count
#pragma unroll
          for (int col = 0; col < BN; ++col) {
            if (col >= valid_cols) sr[col] = 0xff800000u;  // -inf
          }
        }
        auto sval = [&](int col) -> float { return __uint_as_float(sr[col]); };
        // four independent chains of three-input maxima (two new scores per instruction)
        float mq0 = -INFINITY, mq1 = -INFINITY, mq2 = -INFINITY, mq3 = -INFINITY;
#pragma unroll
        for (int col = 0; col < BN; col += 8) {
          mq0 = fmax3(mq0, sval(col), sval(col + 1));
          mq1 = fmax3(mq1, sval(col + 2), sval(col + 3));
          mq2 = fmax3(mq2, sval(col + 4), sval(col + 5));
          mq3 = fmax3(mq3, sval(col + 6), sval(col + 7));
        }
        const float mx_raw = fmax3(mq0, mq1, fmaxf(mq2, mq3));
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
          if (ok) {
            // The commit that published S_t(j) also covers PV_t(j-1): O_t is stable.
            for (int cb = 0; cb < D / 16; ++cb) {
              uint32_t r[16];
              tmem_ld16(o_addr + cb * 16, r);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
              tmem_st16(o_addr + cb * 16, r);
            }
          }
        }
        const float neg_m = (m_new == -INFINITY) ? 0.f : -m_new;
        // P = 2^(s*scale - m): the packed 16-bit pairs overwrite the first 64 S columns (the whole row is
        // already in registers).
        float rowsum = 0.f;
        // Tiles inside the cache release P in two halves; a tile reaching past the cache end releases both at
        // once, after the value rows past the end are zeroed.
        const bool early = tok0 + BN <= c.len;
        bool half_sent = false;
        if (ok) {
          const float2 scale2 = make_float2(a.scale_log2, a.scale_log2);
          const float2 negm2 = make_float2(neg_m, neg_m);
          // four independent partial sums keep the add chain short
          float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                           make_float2(0.f, 0.f)};
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            uint32_t packed[32];
            // One inlined copy of the exponential loop when every pair goes to the SFU: the per-tile code of
            // the softmax, MMA and TMA warps shares the SM's instruction caches, and the duplicate copy measured
            // ~2 % slower (111.6 against 113.7 us on config 2).
            if (S::kFmaEvery == 0 || tail) {
              exp2_pack_half<Tr, 0>(&sr[half * 64], scale2, negm2, acc, packed);
            } else {
              exp2_pack_half<Tr, S::kFmaEvery>(&sr[half * 64], scale2, negm2, acc, packed);
            }
            tmem_st32(s_addr + half * 32, packed);
            if (half == 0 && early) {
              // the first 64 keys of P are in TMEM: PV over them may start while the rest is exponentiated
              tmem_wait_st();
              tc_fence_before_sync();
              __syncwarp();
              if (lane == 0) mbar_arrive(&p_half[t]);
              half_sent = true;
            }
          }
          tmem_wait_st();
          rowsum = (acc[0].x + acc[0].y) + (acc[1].x + acc[1].y) + (acc[2].x + acc[2].y) + (acc[3].x + acc[3].y);
        }
        // Value rows past the cache end: the first tile to use this V stage zeroes them before it
        // releases P (the PV reads them).
        const bool mine = (t == 0) ? true : (j >= c.n_tile[0]);
        if (tok0 + BN > c.len && mine) {
          const uint32_t vcount = vbase + j;
          const int vst = vcount % NS;
          wait_warp(&v_full[vst], (vcount / NS) & 1, 62);
          if (ok && tok0 + row >= c.len) {
            uint8_t* vrow = v_smem + vst * S::kKVBytes + row * 128;
#pragma unroll
            for (int blk = 0; blk < NB; ++blk) {
#pragma unroll
              for (int ch = 0; ch < 8; ++ch) {
                *reinterpret_cast<uint4*>(vrow + blk * BN * 128 + ch * 16) = make_uint4(0, 0, 0, 0);
              }
            }
          }
          fence_proxy_async_smem();
        }
        tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) {
          if (!half_sent) mbar_arrive(&p_half[t]);
          mbar_arrive(&p_full[t]);
        }
        l = l * alpha + rowsum;
        m = m_new;
      }
      if (c.n > 0) vbase += c.n;
      // epilogue
      float inv = 0.f;
      if (n_t > 0) {
        wait_warp(&pv_done[t], pd & 1, 63);
        ++pd;
        inv = l > 0.f ? 1.f / l : 0.f;
        if (ok) tc_fence_after_sync();
      }
      const long long row_id = row_valid ? ((long long)c.b * a.sq + q) * a.heads + c.h : 0;
      const float own_lse = (n_t > 0 && l > 0.f) ? m + fast_log2(l) : kEmptyLse;
      // this row's O block cb (16 columns), normalised, from TMEM
      auto load_o = [&](int cb, float (&o)[16]) {
        if (n_t > 0 && ok) {
          uint32_t r[16];
          tmem_ld16(o_addr + cb * 16, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = __uint_as_float(r[i]) * inv;
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = 0.f;
        }
      };
      auto store_row = [&](int cb, const float (&o)[16], float scale) {
        uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<T*>(a.out) + row_id * D + cb * 16);
        dst[0] = make_uint4(Tr::pack2(o[0] * scale, o[1] * scale), Tr::pack2(o[2] * scale, o[3] * scale),
                            Tr::pack2(o[4] * scale, o[5] * scale), Tr::pack2(o[6] * scale, o[7] * scale));
        dst[1] = make_uint4(Tr::pack2(o[8] * scale, o[9] * scale), Tr::pack2(o[10] * scale, o[11] * scale),
                            Tr::pack2(o[12] * scale, o[13] * scale), Tr::pack2(o[14] * scale, o[15] * scale));
      };
      if (!sg.piece) {
        for (int cb = 0; cb < D / 16; ++cb) {
          float o[16];
          load_o(cb, o);  // warp-collective: every lane, valid row or not
          if (row_valid && a.write_partials) {
            float4* dst = reinterpret_cast<float4*>(a.part_o + (row_id * a.splits + c.s) * D + cb * 16);
#pragma unroll
            for (int i = 0; i < 4; ++i) dst[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
          } else if (row_valid) {
            store_row(cb, o, 1.f);
          }
        }
        if (row_valid && a.write_partials) a.part_lse[row_id * a.splits + c.s] = own_lse;
      } else {
        // A piece of an item cut between programs. Every piece writes its partial (FP32 O and base-2 LSE) to
        // its program's slot (2 p for the piece a program starts with, 2 p + 1 for the one it ends with), then
        // counts itself in on the item's arrival counter; the piece whose count completes the set merges all
        // pieces from their slots in piece order, so the result does not depend on which CTA finished last.
        // No CTA ever waits for another. A slot holds O in groups of four columns ([D / 4][256 rows][4]), so the
        // 32 rows of a warp write, and read back, 512 contiguous bytes per group with one 16-byte access each.
        const long long total = a.prog_u[a.programs];
        const int q_first = program_of(total, a.programs, sg.item_u);
        const int pieces = program_of(total, a.programs, sg.item_u + sg.units - 1) - q_first + 1;
        const int first_extra = sg.item_u != program_start(total, a.programs, q_first) ? 1 : 0;
        const int own = blockIdx.x - q_first;
        const int r = 128 * t + row;  // this thread's row in the pair item
        // slot of piece k (piece k >= 1 sits 2k - first_extra slots after piece 0's)
        auto piece_slot = [&](int k) -> long long {
          return 2ll * q_first + first_extra + (k == 0 ? 0 : 2 * k - first_extra);
        };
        auto slot_group = [&](long long slot, int g) -> float4* {  // columns [4 g, 4 g + 4) of this row
          return reinterpret_cast<float4*>(a.slot_o) + (slot * (D / 4) + g) * kPairRows + r;
        };
        const long long my_slot = piece_slot(own);
        for (int cb = 0; cb < D / 16; ++cb) {
          float o[16];
          load_o(cb, o);  // warp-collective: every lane, valid row or not
          if (row_valid) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              *slot_group(my_slot, cb * 4 + i) = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
            }
          }
        }
        if (row_valid) a.slot_lse[my_slot * kPairRows + r] = own_lse;
        // O_t is out of TMEM: the next segment's first PV may overwrite it while this piece counts in and merges
        if (n_t > 0) {
          tc_fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(&o_empty[t]);
        }
        named_barrier_sync(1, 256);  // both warpgroups have written their rows
        if (warp == 4 && lane == 0) {
          __threadfence();
          *merge_flag = atomicAdd(&a.counters[sg.item], 1) + 1 == pieces ? 1 : 0;
        }
        named_barrier_sync(1, 256);
        const int merge = *merge_flag;
        named_barrier_sync(1, 256);  // read by all before the next write
        if (merge) {
          __threadfence();
          if (warp == 4 && lane == 0) a.counters[sg.item] = 0;  // ready for the next launch
          // base-2 LSE merge (the split merge's arithmetic, merge_kernel in fgw_aux.cu), in piece order; each
          // round loads 32 values of every piece with independent 16-byte loads, so a round costs one L2 round
          // trip per piece instead of one per piece and value
          if (row_valid) {
            auto lse_of = [&](int k) { return __ldcg(&a.slot_lse[piece_slot(k) * kPairRows + r]); };
            float peak = kEmptyLse;
            for (int k = 0; k < pieces; ++k) peak = fmaxf(peak, lse_of(k));
            float wsum = 0.f;
            for (int k = 0; k < pieces; ++k) {
              const float lse = lse_of(k);
              if (lse > kValidLse) wsum += fast_exp2(lse - peak);
            }
            const float scale = wsum > 0.f ? 1.f / wsum : 0.f;
            // two column blocks (32 values) per round; a piece's weight is reloaded with its values, so nothing
            // is indexed by piece in registers
            auto piece_weight = [&](int k) -> float {
              const float lse = lse_of(k);
              return lse > kValidLse ? fast_exp2(lse - peak) : 0.f;
            };
            for (int cb = 0; cb < D / 16; cb += 2) {
              const bool second = cb + 1 < D / 16;
              float acc0[16], acc1[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) acc0[i] = acc1[i] = 0.f;
              for (int k = 0; k < pieces; ++k) {
                const float wk = piece_weight(k);
                if (wk == 0.f) continue;
                const long long slot = piece_slot(k);
                float4 v[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                  v[i] = (i < 4 || second) ? __ldcg(slot_group(slot, cb * 4 + i)) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  acc0[4 * i] = fmaf(wk, v[i].x, acc0[4 * i]);
                  acc0[4 * i + 1] = fmaf(wk, v[i].y, acc0[4 * i + 1]);
                  acc0[4 * i + 2] = fmaf(wk, v[i].z, acc0[4 * i + 2]);
                  acc0[4 * i + 3] = fmaf(wk, v[i].w, acc0[4 * i + 3]);
                  acc1[4 * i] = fmaf(wk, v[4 + i].x, acc1[4 * i]);
                  acc1[4 * i + 1] = fmaf(wk, v[4 + i].y, acc1[4 * i + 1]);
                  acc1[4 * i + 2] = fmaf(wk, v[4 + i].z, acc1[4 * i + 2]);
                  acc1[4 * i + 3] = fmaf(wk, v[4 + i].w, acc1[4 * i + 3]);
                }
              }
              store_row(cb, acc0, scale);
              if (second) store_row(cb + 1, acc1, scale);
            }
          }
        }
        continue;  // this segment's O_t was released above
      }
      if (n_t > 0) {
        tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&o_empty[t]);
      }
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
static cudaError_t launch_fmha2_t(const LaunchDesc& d, const Fmha2Args& args, const CUtensorMap& qmap,
                                  const CUtensorMap& kmap, const CUtensorMap& vmap) {
  using S = Fmha2Shape<NB>;
  auto kernel = fmha2_sm100_kernel<T, NB>;
  // setmaxnreg.inc only succeeds if the registers the block was launched with cover the new split:
  // warpgroup 0 drops to kRegsControl per thread, the two softmax warpgroups rise to kRegsSoftmax. Refuse
  // to launch a build whose allocation would not cover that (the increase would otherwise never complete).
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
  return launch_after_plan(kernel, (unsigned)grid, S::kThreads, S::kBytes, d.stream, qmap, kmap, vmap, args);
}

cudaError_t launch_tensor_pairs(const LaunchDesc& d, bool write_partials, const CUtensorMap& qmap,
                                const CUtensorMap& kmap, const CUtensorMap& vmap, int box_rows) {
  const fgw_mha_params& p = d.p;
  Fmha2Args args;
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
  args.qpairs = (p.q_len + 255) / 256;
  args.items = (long long)p.batch * p.heads * p.num_splits * args.qpairs;
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
    return bf16 ? launch_fmha2_t<__nv_bfloat16, 1>(d, args, qmap, kmap, vmap)
                : launch_fmha2_t<__half, 1>(d, args, qmap, kmap, vmap);
  }
  if (p.head_dim <= 128) {
    return bf16 ? launch_fmha2_t<__nv_bfloat16, 2>(d, args, qmap, kmap, vmap)
                : launch_fmha2_t<__half, 2>(d, args, qmap, kmap, vmap);
  }
  return cudaErrorInvalidValue;
}

}  // namespace fgw
