// Tensor-core (tcgen05 + TMEM + TMA) paged attention for long query blocks.
//
// Replaces the reference's Cube QK^T -> softmax -> PV body (operators/mha/kernels/
// mha_paged_decode_ascend_v7.py:225-315 partial, :375-465 direct; general D/page/causal form in
// mha_paged_decode_ascend_cube_general.py:49-157). B200 design:
//   * persistent CTAs (<= one per SM) walk work items (request, head, split, 128-row query tile)
//     round-robin in descending-cache-length order;
//   * warp 0 (converged, lane 0 issuing) runs TMA: the query tile straight from Q[B,Sq,H,D] through a 4-D
//     tensor map (rows past Sq are zero-filled, so no head-major copy of Q is needed, cf. v7.py:472), and K/V
//     tiles of BN tokens as one 3-D box per (64-column block, page slice) addressed through the block table;
//   * warp 1 (converged, one elected lane issuing) runs tcgen05.mma: S = Q K^T into one of two TMEM
//     buffers, then O += P V into a TMEM accumulator; QK of tile j+1 is issued before PV of tile j so the
//     tensor core works while the softmax warps handle tile j;
//   * warps 4..7 own one query row per thread (TMEM lane = row): load the S row, mask tails and the
//     right-aligned causal diagonal, run the base-2 online softmax, write P (bf16/fp16, 128B-swizzled
//     K-major) to shared memory, rescale O in TMEM only when the row max grew by more than 2^8, and
//     finally normalise O and store the output row (or an FP32 partial + base-2 LSE).
// Value rows of the tile past the cache end are zeroed in shared memory before PV, so NaN-filled
// unread rows can never reach the accumulator (0 * NaN): the reference guards the same way
// (cube_general.py:93-109).
#include <algorithm>

#include "fgw_common.cuh"
#include "fgw_kernels.h"

namespace fgw {

struct TensorArgs {
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

// NB: 64-column blocks of the head dimension (D <= 64 * NB).
template <int NB>
struct TensorShape {
  static constexpr int kBM = 128;                       // query rows per tile (UMMA M)
  static constexpr int kBN = NB <= 2 ? 128 : 64;        // KV tokens per tile
  static constexpr int kBlockBytes = 128 * 128;         // one 64-col block of a 128-row operand
  static constexpr int kQBytes = NB * kBM * 128;
  static constexpr int kKVBytes = NB * kBN * 128;       // one K (or V) stage
  static constexpr int kPBytes = kBM * kBN * 2;
  static constexpr int kStages = NB == 1 ? 4 : (NB == 3 ? 3 : 2);
  static constexpr int kThreads = 256;
  static constexpr int kSCols = kBN;                    // TMEM columns of one S buffer
  static constexpr int kOCol = 2 * kBN;                 // first TMEM column of O
  static constexpr int kTmemCols = 512;
};

template <int NB>
struct TensorSmem {
  using S = TensorShape<NB>;
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + S::kQBytes;
  static constexpr int kV = kK + S::kStages * S::kKVBytes;
  static constexpr int kP = kV + S::kStages * S::kKVBytes;
  static constexpr int kBar = kP + S::kPBytes;
  // barriers: q_full, q_empty, k_full[st], k_empty[st], v_full[st], v_empty[st], s_full[2], p_full,
  //           pv_done, o_empty, mma_done
  static constexpr int kNumBars = 2 + 4 * S::kStages + 2 + 4;
  static constexpr int kTmemSlot = kBar + kNumBars * 8;
  static constexpr int kBytes = kTmemSlot + 16 + 1024;  // + alignment slack
};

struct ItemCoords {
  int b, h, s, qt, q0, n_begin, n_end, len;
};

__device__ __forceinline__ void tensor_item(const TensorArgs& a, long long item, int bn, ItemCoords& c) {
  const int qt_rev = static_cast<int>(item % a.qtiles);
  long long rest = item / a.qtiles;
  c.s = static_cast<int>(rest % a.splits);
  rest /= a.splits;
  c.h = static_cast<int>(rest % a.heads);
  c.b = a.order[rest / a.heads];
  c.qt = a.qtiles - 1 - qt_rev;  // later query tiles first: they see the most keys when causal
  c.q0 = c.qt * 128;
  c.len = a.lengths[c.b];
  const int last_row = min(c.q0 + 128, a.sq) - 1;
  const int vis_max = a.causal ? max(c.len - a.sq + last_row + 1, 0) : c.len;
  const int tiles = (vis_max + bn - 1) / bn;
  c.n_begin = static_cast<int>((long long)tiles * c.s / a.splits);
  c.n_end = static_cast<int>((long long)tiles * (c.s + 1) / a.splits);
}

template <typename T, int NB>
__global__ void __launch_bounds__(256, 1)
    fmha_sm100_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap, const TensorArgs a) {
  using S = TensorShape<NB>;
  using L = TensorSmem<NB>;
  using Tr = ElemTraits<T>;
  constexpr int BN = S::kBN;
  constexpr int NS = S::kStages;

  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128B-swizzled operand tiles.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* q_smem = smem + L::kQ;
  uint8_t* k_smem = smem + L::kK;
  uint8_t* v_smem = smem + L::kV;
  uint8_t* p_smem = smem + L::kP;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;
  uint64_t* k_empty = k_full + NS;
  uint64_t* v_full = k_empty + NS;
  uint64_t* v_empty = v_full + NS;
  uint64_t* s_full = v_empty + NS;  // [2]
  uint64_t* p_full = s_full + 2;
  uint64_t* pv_done = p_full + 1;
  uint64_t* o_empty = pv_done + 1;
  uint64_t* mma_done = o_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kTmemSlot);

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
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(p_full, 128);
    mbar_init(pv_done, 1);
    mbar_init(o_empty, 128);
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
  const int grid = gridDim.x;
  const int D = a.dim;
  grid_dependency_wait();  // the plan's lengths, order and counters from here on

  if (warp == 0) {
    // ------------------------------------------------------------------------- TMA producer
    // Converged warp, lane 0 issues; the item's block-table entries are read 32 pages at a time (one per lane)
    // ahead of the waits and broadcast per box (as in the two-tile kernel, fgw_fmha2_sm100.cu).
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
      for (long long item = blockIdx.x; item < a.items; item += grid) {
        ItemCoords c;
        tensor_item(a, item, BN, c);
        c.n_begin = __shfl_sync(0xffffffffu, c.n_begin, 0);
        c.n_end = __shfl_sync(0xffffffffu, c.n_end, 0);
        if (c.n_end <= c.n_begin) continue;
        const int32_t* row_table = a.table + (long long)c.b * a.width;
        TableWindow table;
        table.init(row_table, a.width, (c.n_begin * BN) / a.page, lane);
        // Q tile: wait until the previous item's last QK has read it.
        if (wait_or_fail(q_empty, (qc & 1) ^ 1, 10) && lane == 0) {
          mbar_arrive_expect_tx(q_full, NB * S::kBlockBytes);
          for (int blk = 0; blk < NB; ++blk) {
            tma_load_4d(q_smem + blk * S::kBlockBytes, &qmap, q_full, blk * 64, c.h, c.q0, c.b);
          }
        }
        ++qc;
        const int end_tok = c.len;
        for (int j = c.n_begin; j < c.n_end; ++j) {
          const int tok0 = j * BN;
          int nbox = 0;
          for (int k = 0; k < boxes; ++k) nbox += (tok0 + k * a.box_rows < end_tok) ? 1 : 0;
          // K tile, then V tile
#pragma unroll
          for (int which = 0; which < 2; ++which) {
            const uint32_t cnt = which == 0 ? kc : vc;
            uint64_t* full = which == 0 ? k_full : v_full;
            uint64_t* empty = which == 0 ? k_empty : v_empty;
            const CUtensorMap* map = which == 0 ? &kmap : &vmap;
            uint8_t* ring = which == 0 ? k_smem : v_smem;
            const int st = cnt % NS;
            if (wait_or_fail(&empty[st], ((cnt / NS) & 1) ^ 1, 11 + which)) {
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
    // Converged warp with warp-uniform loop state; every tcgen05 issue is predicated on one elected lane, and
    // the waits are try_wait (as in the two-tile kernel).
    {
      const uint32_t leader = elect_one_sync();
      const uint32_t tmem_u = __shfl_sync(0xffffffffu, tmem, 0);
      bool ok = true;
      uint32_t kc = 0, vc = 0, qc = 0, sc = 0, pc = 0, oc = 0;
      const int fmt = Tr::kUmmaFormat;
      const uint32_t idesc_qk = umma_idesc_f16(fmt, 128, BN, 0, 0);
      const uint32_t idesc_pv = umma_idesc_f16(fmt, 128, D, 0, 1);
      const uint32_t q_base = smem_u32(q_smem);
      const uint32_t k_base = smem_u32(k_smem);
      const uint32_t v_base = smem_u32(v_smem);
      const uint32_t p_base = smem_u32(p_smem);
      const int ksteps_qk = D / 16;
      const int ksteps_pv = BN / 16;

      auto wait_or_fail = [&](uint64_t* bar, uint32_t parity, int site) {
        if (ok && !__all_sync(0xffffffffu, mbar_wait(bar, parity, a.budget_ns))) {
          ok = false;
          if (lane == 0) record_error(a.ws, FGW_ERR_DEVICE_TIMEOUT, site);
        }
        return ok;
      };
      auto issue_qk = [&](uint32_t s_buf) {
        const int st = kc % NS;
        if (wait_or_fail(&k_full[st], (kc / NS) & 1, 21)) {
          tc_fence_after_sync();
          const uint32_t kst = k_base + st * S::kKVBytes;
          for (int kk = 0; kk < ksteps_qk; ++kk) {
            const uint32_t off = (kk & 3) * 32;  // 16 elements further along the 128-byte swizzled row
            const uint64_t adesc = umma_smem_desc(q_base + (kk >> 2) * S::kBlockBytes + off, 16, 1024, 2);
            const uint64_t bdesc = umma_smem_desc(kst + (kk >> 2) * BN * 128 + off, 16, 1024, 2);
            umma_f16_ss_e(leader, tmem_u + s_buf * S::kSCols, static_cast<uint32_t>(adesc),
                          static_cast<uint32_t>(adesc >> 32), static_cast<uint32_t>(bdesc),
                          static_cast<uint32_t>(bdesc >> 32), idesc_qk, kk > 0 ? 1u : 0u);
          }
          umma_commit_e(leader, &k_empty[st]);
          umma_commit_e(leader, &s_full[s_buf]);
        }
        ++kc;
      };
      auto issue_pv = [&](bool first) {
        const int st = vc % NS;
        bool ready = wait_or_fail(&v_full[st], (vc / NS) & 1, 23);
        if (first) ready = ready && wait_or_fail(o_empty, (oc & 1) ^ 1, 24);
        ready = ready && wait_or_fail(p_full, pc & 1, 22);
        if (ready) {
          tc_fence_after_sync();
          const uint32_t vst = v_base + st * S::kKVBytes;
          for (int kk = 0; kk < ksteps_pv; ++kk) {
            const uint64_t adesc = umma_smem_desc(p_base + (kk >> 2) * S::kBlockBytes + (kk & 3) * 32, 16, 1024, 2);
            const uint64_t bdesc = umma_smem_desc(vst + kk * 16 * 128, BN * 128, 1024, 2);
            umma_f16_ss_e(leader, tmem_u + S::kOCol, static_cast<uint32_t>(adesc), static_cast<uint32_t>(adesc >> 32),
                          static_cast<uint32_t>(bdesc), static_cast<uint32_t>(bdesc >> 32), idesc_pv,
                          (!first || kk > 0) ? 1u : 0u);
          }
          umma_commit_e(leader, &v_empty[st]);
          umma_commit_e(leader, pv_done);
        }
        ++vc;
        ++pc;
      };

      for (long long item = blockIdx.x; item < a.items; item += grid) {
        ItemCoords c;
        tensor_item(a, item, BN, c);
        const int n = __shfl_sync(0xffffffffu, c.n_end - c.n_begin, 0);
        if (n <= 0) continue;
        const bool have_q = wait_or_fail(q_full, qc & 1, 20);
        (void)have_q;
        issue_qk(sc & 1);
        ++sc;
        for (int j = 0; j < n; ++j) {
          if (j + 1 < n) {
            issue_qk(sc & 1);
            ++sc;
          }
          if (j + 1 == n && ok) umma_commit_e(leader, q_empty);  // every QK of this item has been issued
          issue_pv(j == 0);
        }
        ++qc;
        ++oc;
      }
      // Drain: make sure every UMMA issued above has completed before TMEM is released.
      if (ok) {
        umma_commit_e(leader, mma_done);
        __all_sync(0xffffffffu, mbar_wait(mma_done, 0, a.budget_ns));
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------------- softmax / epilogue
    const int row = threadIdx.x - 128;                 // 0..127, = TMEM lane
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>((warp - 4) * 32) << 16);
    bool ok = true;
    uint32_t vc = 0, sc = 0, pc = 0;
    auto wait_warp = [&](uint64_t* bar, uint32_t parity, int site) {
      if (ok) {
        ok = __all_sync(0xffffffffu, mbar_wait(bar, parity, a.budget_ns));
        if (!ok && lane == 0) record_error(a.ws, FGW_ERR_DEVICE_TIMEOUT, site);
      }
      return ok;
    };
    for (long long item = blockIdx.x; item < a.items; item += grid) {
      ItemCoords c;
      tensor_item(a, item, BN, c);
      const int q = c.q0 + row;
      const bool row_valid = q < a.sq;
      const int vis = row_valid ? (a.causal ? max(c.len - a.sq + q + 1, 0) : c.len) : 0;
      const int n = c.n_end - c.n_begin;
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < n; ++j) {
        const int tok0 = (c.n_begin + j) * BN;
        const uint32_t s_buf = sc & 1;
        wait_warp(&s_full[s_buf], (sc >> 1) & 1, 30);
        ++sc;
        float s[BN];
        if (ok) {
          tc_fence_after_sync();
#pragma unroll
          for (int cb = 0; cb < BN / 32; ++cb) {
            uint32_t r[32];
            tmem_ld32(lane_addr + s_buf * S::kSCols + cb * 32, r);
#pragma unroll
            for (int i = 0; i < 32; ++i) s[cb * 32 + i] = __uint_as_float(r[i]);
          }
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < BN; ++i) s[i] = 0.f;
        }
        // mask + row max in the base-2 score domain
        const int valid_cols = min(max(vis - tok0, 0), BN);
        float mx = -INFINITY;
        if (valid_cols == BN) {
#pragma unroll
          for (int i = 0; i < BN; ++i) {
            s[i] *= a.scale_log2;
            mx = fmaxf(mx, s[i]);
          }
        } else {
#pragma unroll
          for (int i = 0; i < BN; ++i) {
            s[i] = i < valid_cols ? s[i] * a.scale_log2 : -INFINITY;
            mx = fmaxf(mx, s[i]);
          }
        }
        // Decide whether O must be rescaled (warp-uniform: the TMEM accesses are warp-collective).
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
        const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
        uint32_t packed[BN / 2];
        // four independent partial sums of pairs keep the add chain short
        float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
        for (int i = 0; i < BN / 2; ++i) {
          packed[i] = Tr::pack2(fast_exp2(s[2 * i] - m_use), fast_exp2(s[2 * i + 1] - m_use));
          // the row sum adds the rounded values PV multiplies (the lazily rescaled max lets P exceed 1 and round)
          acc[i % 4] = Tr::add2(acc[i % 4], packed[i]);
        }
        const float rowsum =
            (acc[0].x + acc[0].y) + (acc[1].x + acc[1].y) + (acc[2].x + acc[2].y) + (acc[3].x + acc[3].y);
        // PV of the previous tile must be finished before P is overwritten and O is rescaled.
        if (j > 0) wait_warp(pv_done, (pc - 1) & 1, 31);
        if (ok && warp_grow && j > 0) {
          tc_fence_after_sync();
          for (int cb = 0; cb < D / 16; ++cb) {
            uint32_t r[16];
            tmem_ld16(lane_addr + S::kOCol + cb * 16, r);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
            tmem_st16(lane_addr + S::kOCol + cb * 16, r);
          }
          tmem_wait_st();
        }
        // P row -> shared memory, 128B-swizzled K-major blocks of 64 tokens.
#pragma unroll
        for (int blk = 0; blk < BN / 64; ++blk) {
          uint8_t* rowp = p_smem + blk * S::kBlockBytes + row * 128;
#pragma unroll
          for (int ch = 0; ch < 8; ++ch) {
            const int base = blk * 32 + ch * 4;
            uint4 v4 = make_uint4(packed[base], packed[base + 1], packed[base + 2], packed[base + 3]);
            *reinterpret_cast<uint4*>(rowp + ((ch ^ (row & 7)) * 16)) = v4;
          }
        }
        // Value rows past the cache end: zero them before PV reads the tile.
        const int vst = vc % NS;
        ++vc;
        if (tok0 + BN > c.len) {
          wait_warp(&v_full[vst], ((vc - 1) / NS) & 1, 32);
          if (ok && row < BN && tok0 + row >= c.len) {
            uint8_t* vrow = v_smem + vst * S::kKVBytes + row * 128;
#pragma unroll
            for (int blk = 0; blk < NB; ++blk) {
#pragma unroll
              for (int ch = 0; ch < 8; ++ch) {
                *reinterpret_cast<uint4*>(vrow + blk * BN * 128 + ch * 16) = make_uint4(0, 0, 0, 0);
              }
            }
          }
        }
        fence_proxy_async_smem();
        tc_fence_before_sync();
        mbar_arrive(p_full);
        ++pc;
        l = l * alpha + rowsum;
        m = m_new;
      }
      // Epilogue: wait for the last PV, normalise and store this row.
      float inv = 0.f;
      if (n > 0) {
        wait_warp(pv_done, (pc - 1) & 1, 33);
        inv = l > 0.f ? 1.f / l : 0.f;
      }
      const long long row_id = row_valid ? ((long long)c.b * a.sq + q) * a.heads + c.h : 0;
      if (n > 0 && ok) tc_fence_after_sync();
      for (int cb = 0; cb < D / 16; ++cb) {
        float o[16];
        if (n > 0 && ok) {
          uint32_t r[16];
          tmem_ld16(lane_addr + S::kOCol + cb * 16, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = __uint_as_float(r[i]) * inv;
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = 0.f;
        }
        if (!row_valid) continue;
        if (a.write_partials) {
          float4* dst = reinterpret_cast<float4*>(a.part_o + (row_id * a.splits + c.s) * D + cb * 16);
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
        } else {
          uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<T*>(a.out) + row_id * D + cb * 16);
          dst[0] = make_uint4(Tr::pack2(o[0], o[1]), Tr::pack2(o[2], o[3]), Tr::pack2(o[4], o[5]),
                              Tr::pack2(o[6], o[7]));
          dst[1] = make_uint4(Tr::pack2(o[8], o[9]), Tr::pack2(o[10], o[11]), Tr::pack2(o[12], o[13]),
                              Tr::pack2(o[14], o[15]));
        }
      }
      if (row_valid && a.write_partials) {
        a.part_lse[row_id * a.splits + c.s] = (n > 0 && l > 0.f) ? m + fast_log2(l) : kEmptyLse;
      }
      if (n > 0) {
        tc_fence_before_sync();
        mbar_arrive(o_empty);
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

// --------------------------------------------------------------------------------------------- host
static int gcd_int(int x, int y) {
  while (y) {
    const int t = x % y;
    x = y;
    y = t;
  }
  return x;
}

static bool make_q_map(CUtensorMap* map, const fgw_mha_params& p) {
  const cuuint64_t dims[4] = {(cuuint64_t)p.head_dim, (cuuint64_t)p.heads, (cuuint64_t)p.q_len,
                              (cuuint64_t)p.batch};
  const cuuint64_t strides[3] = {(cuuint64_t)p.head_dim * 2, (cuuint64_t)p.heads * p.head_dim * 2,
                                 (cuuint64_t)p.q_len * p.heads * p.head_dim * 2};
  const cuuint32_t box[4] = {64, 1, 128, 1};
  const cuuint32_t estride[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt =
      p.dtype == FGW_DTYPE_BFLOAT16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return encode_tiled_cached(map, dt, 4, const_cast<void*>(p.q), dims, strides, box, estride,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static bool make_kv_sw_map(CUtensorMap* map, const void* base, const fgw_mha_params& p, int box_rows) {
  const cuuint64_t dims[3] = {(cuuint64_t)p.head_dim, (cuuint64_t)p.heads, (cuuint64_t)p.pool_rows};
  const cuuint64_t strides[2] = {(cuuint64_t)p.head_dim * 2, (cuuint64_t)p.heads * p.head_dim * 2};
  const cuuint32_t box[3] = {64, 1, (cuuint32_t)box_rows};
  const cuuint32_t estride[3] = {1, 1, 1};
  const CUtensorMapDataType dt =
      p.dtype == FGW_DTYPE_BFLOAT16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return encode_tiled_cached(map, dt, 3, const_cast<void*>(base), dims, strides, box, estride,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename T, int NB>
static cudaError_t launch_tensor_t(const LaunchDesc& d, const TensorArgs& args, const CUtensorMap& qmap,
                                   const CUtensorMap& kmap, const CUtensorMap& vmap) {
  using L = TensorSmem<NB>;
  auto kernel = fmha_sm100_kernel<T, NB>;
  cudaError_t err = prepare_kernel(reinterpret_cast<const void*>(kernel), L::kBytes, d.device, nullptr);
  if (err != cudaSuccess) return err;
  const long long cap = d.p.grid_cap > 0 ? d.p.grid_cap : d.sm_count;
  const long long grid = std::min<long long>(args.items, std::min<long long>(cap, d.sm_count));
  if (grid <= 0) return cudaSuccess;
  return launch_after_plan(kernel, (unsigned)grid, TensorShape<NB>::kThreads, L::kBytes, d.stream, qmap, kmap, vmap,
                           args);
}

cudaError_t launch_tensor(const LaunchDesc& d, bool write_partials) {
  const fgw_mha_params& p = d.p;
  const int nb = (p.head_dim + 63) / 64;
  const int bn = nb <= 2 ? 128 : 64;
  TensorArgs args;
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
  args.box_rows = gcd_int(p.page_size, bn);
  args.write_partials = write_partials ? 1 : 0;
  args.qtiles = (p.q_len + 127) / 128;
  args.items = (long long)p.batch * p.heads * p.num_splits * args.qtiles;
  args.scale_log2 = (1.0f / sqrtf((float)p.head_dim)) * kLog2e;
  args.budget_ns = d.budget_ns;
  CUtensorMap qmap, kmap, vmap;
  if (!make_q_map(&qmap, p) || !make_kv_sw_map(&kmap, p.k_cache, p, args.box_rows) ||
      !make_kv_sw_map(&vmap, p.v_cache, p, args.box_rows)) {
    return cudaErrorInvalidValue;
  }
  if (d.tensor_kernel == FGW_TENSOR_KERNEL_HALVES) {
    if (nb > 2) return cudaErrorNotSupported;
    return launch_tensor_halves(d, write_partials, kmap, vmap, args.box_rows);  // Q goes to TMEM, not via TMA
  }
  if (d.tensor_kernel == FGW_TENSOR_KERNEL_PAIRS) {
    if (nb > 2) return cudaErrorNotSupported;
    return launch_tensor_pairs(d, write_partials, qmap, kmap, vmap, args.box_rows);
  }
  const bool bf16 = p.dtype == FGW_DTYPE_BFLOAT16;
  switch (nb) {
    case 1:
      return bf16 ? launch_tensor_t<__nv_bfloat16, 1>(d, args, qmap, kmap, vmap)
                  : launch_tensor_t<__half, 1>(d, args, qmap, kmap, vmap);
    case 2:
      return bf16 ? launch_tensor_t<__nv_bfloat16, 2>(d, args, qmap, kmap, vmap)
                  : launch_tensor_t<__half, 2>(d, args, qmap, kmap, vmap);
    case 3:
      return bf16 ? launch_tensor_t<__nv_bfloat16, 3>(d, args, qmap, kmap, vmap)
                  : launch_tensor_t<__half, 3>(d, args, qmap, kmap, vmap);
    case 4:
      return bf16 ? launch_tensor_t<__nv_bfloat16, 4>(d, args, qmap, kmap, vmap)
                  : launch_tensor_t<__half, 4>(d, args, qmap, kmap, vmap);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace fgw
