// Tensor-core paged attention with the softmax split by key halves (head dims up to 128). Opt-in:
// launched only when FGW_MHA_TENSOR_KERNEL=halves is set in the environment; the two-query-tile kernel
// (fgw_fmha2_sm100.cu) stays the default, since it is still the faster one on the long-query workload.
//
// Same contract, masking rules and epilogues as the other tensor kernels; the reference body it stands for
// is operators/mha/kernels/mha_paged_decode_ascend_v7.py:225-315, 375-465. What changes is how the softmax
// meets the tensor core:
//   * one 128-row query tile per work item (request, head, split, query tile); S is double-buffered in
//     TMEM, so QK of tile j + 2 is issued as soon as both halves of P(j) are consumed and the softmax of
//     tile j + 1 never waits for the tensor core;
//   * two softmax warpgroups: warps 4-7 own keys [0, 64) of every 128-key tile, warps 8-11 keys [64, 128).
//     Each keeps its own running max and sum and its own O accumulator (O_0, O_1 in TMEM), like two
//     interleaved KV splits, so the warpgroups never exchange a row max inside the loop; the epilogue
//     merges the two halves with their LSE weights;
//   * P of each half goes back into the first 32 TMEM columns of that half of S, and PV_h reads it from
//     there (tcgen05.mma with the A operand in tensor memory).
// TMEM: S0 [0, 128), S1 [128, 256), O_0 [256, 256 + D), O_1 [384, 384 + D) of 512 columns.
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
  float scale_log2;
  uint64_t budget_ns;
};

template <int NB>
struct HalvesShape {
  static constexpr int kBN = 128;                 // keys per KV tile; each softmax warpgroup owns 64
  static constexpr int kTileBytes = 128 * 128;    // one 64-column block of a 128-row operand
  static constexpr int kQBytes = NB * kTileBytes;
  static constexpr int kKVBytes = NB * kBN * 128;  // one K (or V) stage
  static constexpr int kStages = NB == 1 ? 4 : 2;
  static constexpr int kThreads = 384;
  // registers per thread after the warpgroup split (4 x 32 x 88 + 8 x 32 x 208 = 384 x 168)
  static constexpr int kRegsControl = 88;
  static constexpr int kRegsSoftmax = 208;
  // first TMEM column of O_h
  __device__ __forceinline__ static uint32_t o_col(int h) { return 256u + 128u * static_cast<uint32_t>(h); }
  static constexpr int kTmemCols = 512;
  // shared memory carve-up; kX: per half, the row max and row sum of every row, for the epilogue merge
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + kQBytes;
  static constexpr int kV = kK + kStages * kKVBytes;
  static constexpr int kX = kV + kStages * kKVBytes;
  static constexpr int kBar = kX + 2 * 2 * 128 * 4;
  // q_full, q_empty, k_full[S], k_empty[S], v_full[S], v_empty[S], s_full[2], p_full[2], pv_done[2],
  // o_empty, mma_done
  static constexpr int kNumBars = 2 + 4 * kStages + 8;
  static constexpr int kTmemSlot = kBar + kNumBars * 8;
  static constexpr int kBytes = kTmemSlot + 16 + 1024;
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

template <typename T, int NB>
__global__ void __launch_bounds__(384, 1)
    fmha_halves_sm100_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                             const __grid_constant__ CUtensorMap vmap, const HalvesArgs a) {
  using S = HalvesShape<NB>;
  using Tr = ElemTraits<T>;
  constexpr int BN = S::kBN;
  constexpr int NS = S::kStages;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* q_smem = smem + S::kQ;
  uint8_t* k_smem = smem + S::kK;
  uint8_t* v_smem = smem + S::kV;
  float* xch = reinterpret_cast<float*>(smem + S::kX);  // [half][0: max, 1: sum][row]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kBar);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;
  uint64_t* k_empty = k_full + NS;
  uint64_t* v_full = k_empty + NS;
  uint64_t* v_empty = v_full + NS;
  uint64_t* s_full = v_empty + NS;   // [2]: S buffer b holds a tile's scores
  uint64_t* p_full = s_full + 2;     // [2]: half h of P is in TMEM
  uint64_t* pv_done = p_full + 2;    // [2]: PV_h of a tile has completed
  uint64_t* o_empty = pv_done + 2;   // the epilogue has read O_0 and O_1
  uint64_t* mma_done = o_empty + 1;
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
      mbar_init(&p_full[t], 4);  // one arrival per warp of the half's warpgroup
      mbar_init(&pv_done[t], 1);
    }
    mbar_init(o_empty, 8);  // every softmax warp
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
  const long long grid = gridDim.x;

  if (warp < 4) setmaxnreg_dec<S::kRegsControl>();  // warpgroup 0: TMA, MMA and two idle warps
  if (warp == 0) {
    // ------------------------------------------------------------------------- TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&qmap);
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
      bool ok = true;
      uint32_t kc = 0, vc = 0, qc = 0;
      const int boxes = BN / a.box_rows;
      const uint32_t box_bytes = a.box_rows * 128;
      for (long long item = blockIdx.x; item < a.items; item += grid) {
        HalvesItem c;
        halves_item(a, item, c);
        if (c.n <= 0) continue;
        if (ok && !mbar_wait(q_empty, (qc & 1) ^ 1, a.budget_ns)) {
          ok = false;
          record_error(a.ws, FGW_ERR_DEVICE_TIMEOUT, 70);
        }
        if (ok) {
          mbar_arrive_expect_tx(q_full, S::kQBytes);
          for (int blk = 0; blk < NB; ++blk) {
            tma_load_4d(q_smem + blk * S::kTileBytes, &qmap, q_full, blk * 64, c.h, c.q0, c.b);
          }
        }
        ++qc;
        const int32_t* row_table = a.table + (long long)c.b * a.width;
        for (int j = 0; j < c.n; ++j) {
          const int tok0 = (c.n_begin + j) * BN;
          int nbox = 0;
          for (int k = 0; k < boxes; ++k) nbox += (tok0 + k * a.box_rows < c.len) ? 1 : 0;
#pragma unroll
          for (int which = 0; which < 2; ++which) {  // K tile, then V tile of KV step j
            const uint32_t cnt = which == 0 ? kc : vc;
            uint64_t* full = which == 0 ? k_full : v_full;
            uint64_t* empty = which == 0 ? k_empty : v_empty;
            const CUtensorMap* map = which == 0 ? &kmap : &vmap;
            uint8_t* ring = which == 0 ? k_smem : v_smem;
            const int st = cnt % NS;
            if (ok && !mbar_wait(&empty[st], ((cnt / NS) & 1) ^ 1, a.budget_ns)) {
              ok = false;
              record_error(a.ws, FGW_ERR_DEVICE_TIMEOUT, 71 + which);
            }
            if (ok) {
              mbar_arrive_expect_tx(&full[st], NB * nbox * box_bytes);
              uint8_t* dst = ring + st * S::kKVBytes;
              for (int k = 0; k < nbox; ++k) {
                const int tok = tok0 + k * a.box_rows;
                const int row = row_table[tok / a.page] * a.page + tok % a.page;
                for (int blk = 0; blk < NB; ++blk) {
                  tma_load_3d(dst + blk * BN * 128 + k * box_bytes, map, &full[st], blk * 64, c.h, row);
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
    if (lane == 0) {
      bool ok = true;
      uint32_t kc = 0, vc = 0, qc = 0, oc = 0, pc = 0, g = 0;  // g: tiles so far (S buffer g % 2)
      const int fmt = Tr::kUmmaFormat;
      const uint32_t idesc_qk = umma_idesc_f16(fmt, 128, BN, 0, 0);
      const uint32_t idesc_pv = umma_idesc_f16(fmt, 128, D, 0, 1);
      const uint32_t q_lo = umma_desc_lo(smem_u32(q_smem), 16);
      const uint32_t k_lo = umma_desc_lo(smem_u32(k_smem), 16);
      const uint32_t v_lo = umma_desc_lo(smem_u32(v_smem), BN * 128);
      constexpr uint32_t kHi = umma_desc_hi(1024, 2);
      const int ksteps_qk = D / 16;
      auto wait_all_or_fail = [&](uint64_t* b0, uint32_t p0, uint64_t* b1, uint32_t p1, uint64_t* b2, uint32_t p2,
                                  int site) {
        if (ok && !mbar_wait_all(b0, p0, b1, p1, b2, p2, nullptr, 0, a.budget_ns)) {
          ok = false;
          record_error(a.ws, FGW_ERR_DEVICE_TIMEOUT, site);
        }
        return ok;
      };
      // S[buf] = Q K^T, K from stage `st` (already waited for); publishes S[buf] and frees the K stage.
      auto qk = [&](uint32_t buf, int st) {
        const uint32_t b_lo = k_lo + static_cast<uint32_t>((st * S::kKVBytes) >> 4);
#pragma unroll
        for (int kk = 0; kk < 4 * NB; ++kk) {
          if (kk < ksteps_qk) {
            const uint32_t a_off = static_cast<uint32_t>(((kk >> 2) * S::kTileBytes + (kk & 3) * 32) >> 4);
            const uint32_t b_off = static_cast<uint32_t>(((kk >> 2) * BN * 128 + (kk & 3) * 32) >> 4);
            umma_f16_ss_w(tmem + buf * 128u, q_lo + a_off, kHi, b_lo + b_off, kHi, idesc_qk, kk > 0 ? 1u : 0u);
          }
        }
        umma_commit(&s_full[buf]);
        umma_commit(&k_empty[st]);
      };
      // O_h += P_h V_h over keys [64 h, 64 h + 64): P_h from the first 32 columns of half h of S[buf], V rows
      // from stage `st`.
      auto pv = [&](uint32_t buf, int half, int st, bool first) {
        const uint32_t b_lo = v_lo + static_cast<uint32_t>((st * S::kKVBytes) >> 4);
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) {
          const int kk = 4 * half + k4;  // 16-key step within the tile
          umma_f16_ts_w(tmem + S::o_col(half), tmem + buf * 128u + 64u * half + 8u * k4,
                        b_lo + static_cast<uint32_t>((kk * 16 * 128) >> 4), kHi, idesc_pv,
                        (!first || k4 > 0) ? 1u : 0u);
        }
        umma_commit(&pv_done[half]);
      };
      for (long long item = blockIdx.x; item < a.items; item += grid) {
        HalvesItem c;
        halves_item(a, item, c);
        if (c.n <= 0) continue;
        // prologue: S of the item's first two tiles
        for (int j = 0; j < 2 && j < c.n; ++j) {
          const int st = kc % NS;
          if (wait_all_or_fail(j == 0 ? q_full : nullptr, qc & 1, &k_full[st], (kc / NS) & 1, nullptr, 0, 75 + j)) {
            tc_fence_after_sync();
            qk((g + j) & 1, st);
          }
          ++kc;
        }
        ++qc;
        if (c.n <= 2 && ok) umma_commit(q_empty);  // every QK of this item is issued
        for (int j = 0; j < c.n; ++j, ++g) {
          const uint32_t buf = g & 1;
          const int vst = vc % NS;
          const uint32_t v_par = (vc / NS) & 1;
          ++vc;
          for (int half = 0; half < 2; ++half) {
            // this half of P(j), the V tile (once) and, on an item's first tile, O read out by the epilogue
            if (wait_all_or_fail(&p_full[half], pc & 1, half == 0 ? &v_full[vst] : nullptr, v_par,
                                 (half == 0 && j == 0) ? o_empty : nullptr, (oc & 1) ^ 1, 77 + half)) {
              tc_fence_after_sync();
              pv(buf, half, vst, j == 0);
            }
          }
          ++pc;
          if (ok) umma_commit(&v_empty[vst]);
          if (j + 2 < c.n) {
            // both halves of P(j) are consumed (in issue order): S[buf] takes tile j + 2
            const int st = kc % NS;
            if (wait_all_or_fail(&k_full[st], (kc / NS) & 1, nullptr, 0, nullptr, 0, 79)) {
              tc_fence_after_sync();
              qk(buf, st);
            }
            ++kc;
            if (j + 3 == c.n && ok) umma_commit(q_empty);
          }
        }
        ++oc;
      }
      if (ok) {
        umma_commit(mma_done);
        mbar_wait(mma_done, 0, a.budget_ns);
      }
    }
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
    uint32_t g = 0, pvc = 0, vbase = 0;
    auto wait_warp = [&](uint64_t* bar, uint32_t parity, int site) {
      if (ok) {
        ok = __all_sync(0xffffffffu, mbar_wait(bar, parity, a.budget_ns));
        if (!ok && lane == 0) record_error(a.ws, FGW_ERR_DEVICE_TIMEOUT, site);
      }
      return ok;
    };
    for (long long item = blockIdx.x; item < a.items; item += grid) {
      HalvesItem c;
      halves_item(a, item, c);
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
        // O_h may be rescaled only once PV_h(j - 1) has completed. The wait happens on every tile, so this
        // warpgroup is never more than one phase behind the barrier.
        if (j > 0) {
          wait_warp(&pv_done[half], pvc & 1, 82 + half);
          ++pvc;
          if (warp_grow && ok) {
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
        // Value rows past the cache end: this half's rows are zeroed before its P is released (PV_h reads them).
        if (tok0 + BN > c.len) {
          const uint32_t vcount = vbase + j;
          const int vst = vcount % NS;
          wait_warp(&v_full[vst], (vcount / NS) & 1, 84 + half);
          const int vrow = 64 * half + row;
          if (ok && row < 64 && tok0 + vrow >= c.len) {
            uint8_t* dst = v_smem + vst * S::kKVBytes + vrow * 128;
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
        if (lane == 0) mbar_arrive(&p_full[half]);
        const float rowsum = (acc[0].x + acc[0].y) + (acc[1].x + acc[1].y) + (acc[2].x + acc[2].y) +
                             (acc[3].x + acc[3].y);
        l = l * alpha + rowsum;
        m = m_new;
      }
      if (c.n > 0) {
        vbase += c.n;
        wait_warp(&pv_done[half], pvc & 1, 86 + half);  // PV_h of the item's last tile
        ++pvc;
      }
      // epilogue: merge the two halves' running states (LSE weights), then each warpgroup normalises and
      // stores alternate 16-column blocks of the row
      xch[(2 * half) * 128 + row] = m;
      xch[(2 * half + 1) * 128 + row] = l;
      named_barrier_sync(2, 256);  // both halves' states, and both PV_h of the last tile, are complete
      const float m0 = xch[row], l0 = xch[128 + row], m1 = xch[256 + row], l1 = xch[384 + row];
      const float mt = fmaxf(m0, m1);
      const float w0 = (m0 == -INFINITY) ? 0.f : fast_exp2(m0 - mt);
      const float w1 = (m1 == -INFINITY) ? 0.f : fast_exp2(m1 - mt);
      const float lt = l0 * w0 + l1 * w1;
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      const float lse = (c.n > 0 && lt > 0.f) ? mt + fast_log2(lt) : kEmptyLse;
      const long long row_id = row_valid ? ((long long)c.b * a.sq + q) * a.heads + c.h : 0;
      if (c.n > 0 && ok) tc_fence_after_sync();
      for (int cb = half; cb < D / 16; cb += 2) {
        float o[16];
        if (c.n > 0 && ok) {  // warp-collective: every lane, valid row or not
          uint32_t r0[16], r1[16];
          tmem_ld16(tmem + lane_base + S::o_col(0) + cb * 16, r0);
          tmem_ld16(tmem + lane_base + S::o_col(1) + cb * 16, r1);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = (__uint_as_float(r0[i]) * w0 + __uint_as_float(r1[i]) * w1) * inv;
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = 0.f;
        }
        if (row_valid && a.write_partials) {
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
      if (row_valid && a.write_partials && half == 0) a.part_lse[row_id * a.splits + c.s] = lse;
      named_barrier_sync(2, 256);  // the exchange slots are free for the next item
      if (c.n > 0) {
        tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(o_empty);
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
  const long long grid = std::min<long long>(args.items, std::min<long long>(cap, d.sm_count));
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
