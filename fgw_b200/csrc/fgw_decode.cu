// Warp-level, HBM-streaming paged attention for short query blocks (decode, q_len ~ 1).
//
// Replaces the reference's SIMT split-KV kernels (operators/mha/kernels/mha_paged_decode_ascend_v2.py:34-129,
// v1 for one split) and the Q~1 use of the v7 Cube kernel. Design for B200:
//   * one persistent CTA per SM walks its share of the work items (request, query-row block, split, head),
//     requests in descending-cache-length order (LPT): with one split the items' KV stages, laid end to end,
//     are cut into one equal range per CTA (contiguous schedule; an item cut between CTAs is merged in place by
//     the CTA completing it) when asked for, otherwise whole items are dealt in snake order (snake_item);
//   * a producer warp streams each item's live KV pages into a shared-memory ring with TMA,
//     one 3-D box {head_dim, 1, rows} per (page slice, K or V), driven by the block table;
//   * eight consumer warps split a tile's tokens into groups of LPT lanes; each group owns
//     whole tokens, reduces q.k across its lanes with shuffles and keeps an online-softmax
//     state (max, sum, accumulator) in base 2;
//   * states are merged across groups (shuffles) and warps (shared memory) at the end of the item,
//     which writes the final output (one split) or an FP32 partial plus base-2 LSE.
// Masked tokens never touch the accumulator, so NaN-filled rows past a cache's end cannot leak
// (0 * NaN would): the reference relies on the same guard (v2.py:107-109, cube_general.py:93-109).
#include <algorithm>

#include "fgw_common.cuh"
#include "fgw_kernels.h"

namespace fgw {

struct DecodeArgs {
  const void* q;
  void* out;
  const int32_t* table;
  const int32_t* lengths;
  const int32_t* order;
  float* part_o;
  float* part_lse;
  WorkspaceHeader* ws;
  int batch, sq, heads, width, page, splits, causal, row_blocks, box_rows, write_partials;
  // fused split merge: arrivals per (request, row block, head) group; the CTA completing a group merges it
  int fused_merge;
  int32_t* merge_counters;
  // contiguous schedule (one split): per-program first item, unit offset and first unit, the per-item arrival
  // counters and the two partial slots of every program (kRows rows each); whole items below tail_start first
  int contiguous, programs, tail_start;
  const int32_t* prog_item;
  const int32_t* prog_off;
  const long long* prog_u;
  int32_t* counters;
  float* slot_lse;
  float* slot_o;
  long long items;
  float scale_log2;
  uint64_t budget_ns;
};

template <int D>
struct DecodeShape {
  static constexpr int kChunks = D / 8;                    // 16-byte chunks per row
  static constexpr int kLpt = kChunks >= 8 ? 8 : (kChunks >= 4 ? 4 : 2);  // lanes per token
  static constexpr int kCpl = (kChunks + kLpt - 1) / kLpt;  // chunks per lane
  static constexpr int kGpw = 32 / kLpt;                   // token groups per warp
  // consumer warps: the consumers are latency-bound, so small rows get 12 (the register budget of 416
  // threads still covers them); 8 above D = 128
  static constexpr int kWarps = D <= 128 ? 12 : 8;
  static constexpr int kGroups = kWarps * kGpw;
  static constexpr int kTile = kGroups * ((64 + kGroups - 1) / kGroups);  // tokens per stage: >= 64, whole groups
  static constexpr int kTpg = kTile / kGroups;             // tokens per group per tile
  static constexpr int kRows = (kCpl * 8 >= 32) ? 1 : ((kCpl * 8 >= 16) ? 2 : 4);  // query rows per item
  static constexpr int kThreads = (kWarps + 1) * 32;
};

template <typename T, int D>
struct DecodeSmem {
  using S = DecodeShape<D>;
  static constexpr int kStageBytes = 2 * S::kTile * D * (int)sizeof(T);
  static constexpr int kStages = std::min(8, std::max(2, (192 * 1024) / kStageBytes));
  static constexpr int kRedFloats = S::kWarps * S::kRows * (D + 2);
  static constexpr int kItemSlots = 4;  // whole items handed from the producer to the consumers (dynamic deal)
  static constexpr int kItemBytes = kItemSlots * 8 * 3 + 8;
  static constexpr int kBytes = kStages * kStageBytes + 2 * kStages * 8 + kRedFloats * 4 + kItemBytes + 64;
};

__device__ __forceinline__ void decode_item(long long item, int heads, int splits, int row_blocks,
                                            const int32_t* order, int& b, int& rb, int& s, int& h) {
  h = static_cast<int>(item % heads);
  long long rest = item / heads;
  s = static_cast<int>(rest % splits);
  rest /= splits;
  rb = static_cast<int>(rest % row_blocks);
  b = order[rest / row_blocks];
}

// One run of KV stages of one work item processed by this CTA: a whole item (its split's range), or, with the
// contiguous schedule, units [first, first + count) of an item, which is a piece when other CTAs hold the rest.
struct DecodeSegment {
  long long item;
  int first, count;  // count < 0: whole item, the split's range of stages
  bool piece;
  long long item_u;  // first unit of the item in the contiguous cut
  int units;         // units of the whole item (at least 1)
};

struct DecodeCursor {
  long long round;  // next round of whole items (strided part, snake order)
  long long item;
  int off;
  long long u, u_end;
};

// KV units of a decode item (stages seen by its last query row, at least 1): the plan's stream_item_units.
template <int D>
__device__ __forceinline__ int decode_units(const DecodeArgs& a, long long item) {
  using S = DecodeShape<D>;
  int b, rb, s, h;
  decode_item(item, a.heads, a.splits, a.row_blocks, a.order, b, rb, s, h);
  const int len = a.lengths[b];
  const int last = min(rb * S::kRows + S::kRows, a.sq) - 1;
  const int visible = a.causal ? max(len - a.sq + last + 1, 0) : len;
  return max((visible + S::kTile - 1) / S::kTile, 1);
}

template <bool kContiguous>
__device__ __forceinline__ void decode_cursor_init(const DecodeArgs& a, DecodeCursor& k) {
  k.round = 0;
  k.item = kContiguous ? a.prog_item[blockIdx.x] : 0;
  k.off = kContiguous ? a.prog_off[blockIdx.x] : 0;
  k.u = kContiguous ? a.prog_u[blockIdx.x] : 0;
  k.u_end = kContiguous ? a.prog_u[blockIdx.x + 1] : 0;
}

// The producer and the consumers walk the same segments in the same order: whole items first (all of them
// with the strided schedule), then the CTA's contiguous range of units. The schedule is a template parameter, so
// the strided kernel carries none of the contiguous schedule's state (the consumers run at the register limit).
template <int D, bool kContiguous>
__device__ __forceinline__ bool decode_next(const DecodeArgs& a, DecodeCursor& k, DecodeSegment& sg) {
  const long long whole = snake_item(k.round);
  if (whole < (kContiguous ? static_cast<long long>(a.tail_start) : a.items)) {
    sg.item = whole;
    sg.first = 0;
    sg.count = -1;
    sg.piece = false;
    sg.item_u = 0;
    sg.units = 0;
    ++k.round;
    return true;
  }
  if (!kContiguous || k.u >= k.u_end) return false;
  const int units = decode_units<D>(a, k.item);
  const int count = static_cast<int>(min(static_cast<long long>(units - k.off), k.u_end - k.u));
  sg.item = k.item;
  sg.first = k.off;
  sg.count = count;
  sg.piece = count < units;
  sg.item_u = k.u - k.off;
  sg.units = units;
  k.u += count;
  k.off += count;
  if (k.off >= units) {
    ++k.item;
    k.off = 0;
  }
  return true;
}

// Stages [t_begin, t_end) of a segment over an item with `tiles` stages.
__device__ __forceinline__ void segment_range(const DecodeSegment& sg, int tiles, int s, int splits, int& t_begin,
                                              int& t_end) {
  if (sg.count < 0) {
    t_begin = static_cast<int>((long long)tiles * s / splits);
    t_end = static_cast<int>((long long)tiles * (s + 1) / splits);
  } else {
    t_begin = min(sg.first, tiles);
    t_end = min(sg.first + sg.count, tiles);
  }
}

template <typename T, int D, bool kContiguous>
__global__ void __launch_bounds__(DecodeShape<D>::kThreads, 1)
    decode_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                  const DecodeArgs a) {
  using S = DecodeShape<D>;
  using M = DecodeSmem<T, D>;
  using Tr = ElemTraits<T>;
  constexpr int kRows = S::kRows;
  constexpr int kStages = M::kStages;

  constexpr int kItemSlots = M::kItemSlots;

  extern __shared__ __align__(128) uint8_t smem[];
  T* ring = reinterpret_cast<T*>(smem);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * M::kStageBytes);
  uint64_t* empty = full + kStages;
  float* red = reinterpret_cast<float*>(empty + kStages);
  // dynamic deal: item indices from the producer to the consumers, and the consumers' shared abort flag
  long long* item_slot = reinterpret_cast<long long*>(red + M::kRedFloats);
  uint64_t* item_full = reinterpret_cast<uint64_t*>(item_slot + kItemSlots);
  uint64_t* item_empty = item_full + kItemSlots;
  volatile int* item_abort = reinterpret_cast<volatile int*>(item_empty + kItemSlots);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], S::kWarps);
    }
    for (int i = 0; i < kItemSlots; ++i) {
      mbar_init(&item_full[i], 1);
      mbar_init(&item_empty[i], S::kWarps);
    }
    *item_abort = 0;
    fence_barrier_init();
  }
  __syncthreads();
  grid_dependency_wait();  // the plan's lengths, order and counters from here on

  if (warp == S::kWarps) {
    // ----------------------------------------------------------------- producer warp
    if (lane == 0) {
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
      const uint64_t policy = l2_policy_evict_first();
      bool ok = true;
      uint32_t it = 0;
      const int boxes = S::kTile / a.box_rows;
      const uint32_t box_bytes = a.box_rows * D * sizeof(T);
      DecodeCursor cur;
      decode_cursor_init<kContiguous>(a, cur);
      DecodeSegment sg;
      // Dynamic deal (whole items): the items, longest request first with heads innermost, go one at a time to
      // whichever CTA asks next (a global counter), so the CTAs finish within one item of each other and the
      // items in flight at any moment are consecutive ones (the heads of a few requests, read together). The
      // index is drawn one item ahead and handed to the consumers through the item ring.
      unsigned long long drawn = kContiguous ? 0ull : atomicAdd(&a.ws->next_item, 1ull);
      uint32_t n_items = 0;
      while (true) {
        if constexpr (kContiguous) {
          if (!decode_next<D, true>(a, cur, sg)) break;
        } else {
          const long long item = (ok && drawn < static_cast<unsigned long long>(a.items)) ? static_cast<long long>(drawn)
                                                                                         : -1ll;
          if (item >= 0) drawn = atomicAdd(&a.ws->next_item, 1ull);
          const int slot = n_items % kItemSlots;
          if (!mbar_wait(&item_empty[slot], ((n_items / kItemSlots) & 1) ^ 1, a.budget_ns)) {
            ok = false;
            record_error(a.ws, FGW_ERR_DEVICE_TIMEOUT, 3);
            break;  // unpublished: the consumers' bounded wait for this slot gives up
          }
          item_slot[slot] = item;
          mbar_arrive(&item_full[slot]);
          ++n_items;
          if (item < 0) break;
          sg.item = item;
          sg.first = 0;
          sg.count = -1;
          sg.piece = false;
          sg.item_u = 0;
          sg.units = 0;
        }
        int b, rb, s, h;
        decode_item(sg.item, a.heads, a.splits, a.row_blocks, a.order, b, rb, s, h);
        const int len = a.lengths[b];
        const int last_row = min(rb * kRows + kRows, a.sq) - 1;
        const int end_tok = a.causal ? max(len - a.sq + last_row + 1, 0) : len;
        const int tiles = (end_tok + S::kTile - 1) / S::kTile;
        int t_begin, t_end;
        segment_range(sg, tiles, s, a.splits, t_begin, t_end);
        const int32_t* row_table = a.table + (long long)b * a.width;
        for (int t = t_begin; t < t_end; ++t, ++it) {
          const int stage = it % kStages;
          const uint32_t phase = (it / kStages) & 1;
          if (ok && !mbar_wait(&empty[stage], phase ^ 1, a.budget_ns)) {
            ok = false;
            record_error(a.ws, FGW_ERR_DEVICE_TIMEOUT, 1);
          }
          if (!ok) continue;
          const int tok0 = t * S::kTile;
          int nb = 0;
          for (int k = 0; k < boxes; ++k) nb += (tok0 + k * a.box_rows < end_tok) ? 1 : 0;
          mbar_arrive_expect_tx(&full[stage], 2u * nb * box_bytes);
          T* kdst = ring + (size_t)stage * (2 * S::kTile * D);
          T* vdst = kdst + S::kTile * D;
          for (int k = 0; k < nb; ++k) {
            const int tok = tok0 + k * a.box_rows;
            const int row = row_table[tok / a.page] * a.page + tok % a.page;
            tma_load_3d_hint(kdst + k * a.box_rows * D, &kmap, &full[stage], 0, h, row, policy);
            tma_load_3d_hint(vdst + k * a.box_rows * D, &vmap, &full[stage], 0, h, row, policy);
          }
        }
      }
      if constexpr (!kContiguous) {
        // The CTA that draws last resets the deal for the next launch (the plan launch also zeroes it).
        __threadfence();
        if (atomicAdd(&a.ws->finished, 1u) == gridDim.x - 1) {
          a.ws->next_item = 0ull;
          a.ws->finished = 0u;
        }
      }
      // Leave no copy in flight: wait for the stages still owed to the consumers.
      if (!ok) {
        for (uint32_t j = 0; j < (uint32_t)kStages && j < it; ++j) {
          const uint32_t k = it - 1 - j;
          mbar_wait(&full[k % kStages], (k / kStages) & 1, a.budget_ns);
        }
      }
    }
    return;
  }

  // ------------------------------------------------------------------- consumer warps
  const int group_in_warp = lane / S::kLpt;
  const int lane_in_group = lane % S::kLpt;
  const int group = warp * S::kGpw + group_in_warp;
  const uint32_t group_mask = (S::kLpt == 32 ? 0xffffffffu : ((1u << S::kLpt) - 1u)) << (group_in_warp * S::kLpt);
  const uint32_t consumer_threads = S::kWarps * 32;
  bool ok = true;
  uint32_t it = 0;

  DecodeCursor cur;
  decode_cursor_init<kContiguous>(a, cur);
  DecodeSegment sg;
  uint32_t n_items = 0;
  while (true) {
    if constexpr (kContiguous) {
      if (!decode_next<D, true>(a, cur, sg)) break;
    } else {
      // The next item from the producer. Every consumer warp leaves or stays together (the item loop has
      // consumer-wide named barriers): a warp whose bounded wait gave up raises the shared abort flag before
      // the barrier, and all of them read the flag after it.
      const int slot = n_items % kItemSlots;
      const bool seen = mbar_wait(&item_full[slot], (n_items / kItemSlots) & 1, a.budget_ns);
      if (!__all_sync(0xffffffffu, seen) && lane == 0) {
        *item_abort = 1;
        record_error(a.ws, FGW_ERR_DEVICE_TIMEOUT, 4);
      }
      __syncwarp();
      named_barrier_sync(2, consumer_threads);
      const long long item = *item_abort ? -1ll : *reinterpret_cast<volatile long long*>(&item_slot[slot]);
      __syncwarp();
      named_barrier_sync(2, consumer_threads);  // every warp has read the flag before any can raise it again
      if (lane == 0) mbar_arrive(&item_empty[slot]);
      ++n_items;
      if (item < 0) break;
      sg.item = item;
      sg.first = 0;
      sg.count = -1;
      sg.piece = false;
      sg.item_u = 0;
      sg.units = 0;
    }
    int b, rb, s, h;
    decode_item(sg.item, a.heads, a.splits, a.row_blocks, a.order, b, rb, s, h);
    const int len = a.lengths[b];
    const int q0 = rb * kRows;
    int vis[kRows];
    int end_tok = 0;
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      const int qi = q0 + r;
      vis[r] = qi < a.sq ? (a.causal ? max(len - a.sq + qi + 1, 0) : len) : 0;
      end_tok = max(end_tok, vis[r]);
    }
    const int tiles = (end_tok + S::kTile - 1) / S::kTile;
    int t_begin, t_end;
    segment_range(sg, tiles, s, a.splits, t_begin, t_end);
    const int nrows = min(kRows, a.sq - q0);  // query rows of this item that exist

    // Query rows for this lane's chunks, pre-scaled into the base-2 score domain.
    float qv[kRows][S::kCpl * 8];
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      const int qi = min(q0 + r, a.sq - 1);
      const T* qrow = reinterpret_cast<const T*>(a.q) + (((long long)b * a.sq + qi) * a.heads + h) * D;
#pragma unroll
      for (int c = 0; c < S::kCpl; ++c) {
        const int ci = lane_in_group + c * S::kLpt;
        uint4 raw = make_uint4(0, 0, 0, 0);
        if (ci < S::kChunks) raw = *reinterpret_cast<const uint4*>(qrow + ci * 8);
        const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = Tr::unpack2(w[e]);
          qv[r][c * 8 + 2 * e] = f.x * a.scale_log2;
          qv[r][c * 8 + 2 * e + 1] = f.y * a.scale_log2;
        }
      }
    }
    float m[kRows], l[kRows], acc[kRows][S::kCpl * 8];
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      m[r] = -INFINITY;
      l[r] = 0.f;
#pragma unroll
      for (int e = 0; e < S::kCpl * 8; ++e) acc[r][e] = 0.f;
    }

    for (int t = t_begin; t < t_end; ++t, ++it) {
      const int stage = it % kStages;
      const uint32_t phase = (it / kStages) & 1;
      if (ok) {
        // Keep `ok` warp-uniform: the group shuffles below need every lane of the group.
        ok = __all_sync(0xffffffffu, mbar_wait(&full[stage], phase, a.budget_ns));
        if (!ok && lane == 0) record_error(a.ws, FGW_ERR_DEVICE_TIMEOUT, 2);
      }
      if (ok) {
        const T* ktile = ring + (size_t)stage * (2 * S::kTile * D);
        const T* vtile = ktile + S::kTile * D;
        const int tok0 = t * S::kTile;
        // Scores of this group's kTpg tokens of the tile, computed independently (each dot product in four
        // partial sums), then one max / rescale per tile, then the V rows (each loaded once for every query
        // row). Tokens at or past end_tok are never used: their shared-memory rows were not loaded.
        float sc[S::kTpg][kRows];
        bool live[S::kTpg];
#pragma unroll
        for (int j = 0; j < S::kTpg; ++j) {
          const int tt = group + j * S::kGroups;
          live[j] = tok0 + tt < end_tok;  // uniform within the group
          float kf[S::kCpl * 8];
#pragma unroll
          for (int c = 0; c < S::kCpl; ++c) {
            const int ci = lane_in_group + c * S::kLpt;
            uint4 raw = make_uint4(0, 0, 0, 0);
            if (ci < S::kChunks && live[j]) raw = *reinterpret_cast<const uint4*>(ktile + tt * D + ci * 8);
            const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = Tr::unpack2(w[e]);
              kf[c * 8 + 2 * e] = f.x;
              kf[c * 8 + 2 * e + 1] = f.y;
            }
          }
#pragma unroll
          for (int r = 0; r < kRows; ++r) {
            float dot = 0.f;
            if (r < nrows) {  // uniform: rows past the query length take no work
              float part[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
              for (int e = 0; e < S::kCpl * 8; ++e) part[e % 4] = fmaf(qv[r][e], kf[e], part[e % 4]);
              dot = (part[0] + part[1]) + (part[2] + part[3]);
              // Only this group's lanes take part: groups leave the tile independently.
#pragma unroll
              for (int off = S::kLpt / 2; off > 0; off >>= 1) dot += __shfl_xor_sync(group_mask, dot, off);
            }
            sc[j][r] = dot;
          }
        }
        float pr[S::kTpg][kRows];
#pragma unroll
        for (int r = 0; r < kRows; ++r) {
          float mt = m[r];
#pragma unroll
          for (int j = 0; j < S::kTpg; ++j) {
            const bool use = live[j] && r < nrows && tok0 + group + j * S::kGroups < vis[r];
            if (use) mt = fmaxf(mt, sc[j][r]);
          }
          if (mt > m[r]) {
            const float corr = fast_exp2(m[r] - mt);  // exp2(-inf) = 0 on the first key
            l[r] *= corr;
#pragma unroll
            for (int e = 0; e < S::kCpl * 8; ++e) acc[r][e] *= corr;
            m[r] = mt;
          }
#pragma unroll
          for (int j = 0; j < S::kTpg; ++j) {
            const bool use = live[j] && r < nrows && tok0 + group + j * S::kGroups < vis[r];
            pr[j][r] = use ? fast_exp2(sc[j][r] - m[r]) : 0.f;
            l[r] += pr[j][r];
          }
        }
#pragma unroll
        for (int j = 0; j < S::kTpg; ++j) {
          if (!live[j]) continue;  // uniform within the group
          const int tt = group + j * S::kGroups;
          float vf[S::kCpl * 8];
#pragma unroll
          for (int c = 0; c < S::kCpl; ++c) {
            const int ci = lane_in_group + c * S::kLpt;
            uint4 raw = make_uint4(0, 0, 0, 0);
            if (ci < S::kChunks) raw = *reinterpret_cast<const uint4*>(vtile + tt * D + ci * 8);
            const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = Tr::unpack2(w[e]);
              vf[c * 8 + 2 * e] = f.x;
              vf[c * 8 + 2 * e + 1] = f.y;
            }
          }
#pragma unroll
          for (int r = 0; r < kRows; ++r) {
            // masked tokens (p = 0) stay out of the accumulator entirely: V rows past a cache's end may be NaN
            if (pr[j][r] != 0.f) {
#pragma unroll
              for (int e = 0; e < S::kCpl * 8; ++e) acc[r][e] = fmaf(pr[j][r], vf[e], acc[r][e]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
    }

    // Merge group states inside the warp (groups differ in the high lane bits).
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
#pragma unroll
      for (int off = S::kLpt; off < 32; off <<= 1) {
        const float mo = __shfl_xor_sync(0xffffffffu, m[r], off);
        const float lo = __shfl_xor_sync(0xffffffffu, l[r], off);
        const float mn = fmaxf(m[r], mo);
        const float ca = (m[r] == -INFINITY) ? 0.f : fast_exp2(m[r] - mn);
        const float cb = (mo == -INFINITY) ? 0.f : fast_exp2(mo - mn);
        l[r] = l[r] * ca + lo * cb;
#pragma unroll
        for (int e = 0; e < S::kCpl * 8; ++e) {
          const float ao = __shfl_xor_sync(0xffffffffu, acc[r][e], off);
          acc[r][e] = acc[r][e] * ca + ao * cb;
        }
        m[r] = mn;
      }
    }
    // Group 0 of each warp publishes the warp state: red[warp][row][0..D) acc, [D] max, [D+1] sum.
    if (group_in_warp == 0) {
#pragma unroll
      for (int r = 0; r < kRows; ++r) {
        float* dst = red + (warp * kRows + r) * (D + 2);
#pragma unroll
        for (int c = 0; c < S::kCpl; ++c) {
          const int ci = lane_in_group + c * S::kLpt;
          if (ci < S::kChunks) {
#pragma unroll
            for (int e = 0; e < 8; ++e) dst[ci * 8 + e] = acc[r][c * 8 + e];
          }
        }
        if (lane_in_group == 0) {
          dst[D] = m[r];
          dst[D + 1] = l[r];
        }
      }
    }
    named_barrier_sync(1, consumer_threads);
    // A piece of an item cut between CTAs (contiguous schedule) writes its partial to its program's slot.
    long long my_slot = 0;
    int pieces = 1, q_first = 0, first_extra = 0;
    if (kContiguous && sg.piece) {
      const long long total = a.prog_u[a.programs];
      q_first = program_of(total, a.programs, sg.item_u);
      pieces = program_of(total, a.programs, sg.item_u + sg.units - 1) - q_first + 1;
      first_extra = sg.item_u != program_start(total, a.programs, q_first) ? 1 : 0;
      my_slot = piece_slot(q_first, first_extra, static_cast<int>(blockIdx.x) - q_first);
    }
    for (int idx = threadIdx.x; idx < kRows * D; idx += consumer_threads) {
      const int r = idx / D;
      const int d = idx % D;
      const int qi = q0 + r;
      if (qi >= a.sq) continue;
      float mx = -INFINITY;
#pragma unroll
      for (int w = 0; w < S::kWarps; ++w) mx = fmaxf(mx, red[(w * kRows + r) * (D + 2) + D]);
      float num = 0.f, den = 0.f;
      if (mx != -INFINITY) {
#pragma unroll
        for (int w = 0; w < S::kWarps; ++w) {
          const float* src = red + (w * kRows + r) * (D + 2);
          const float mw = src[D];
          const float f = (mw == -INFINITY) ? 0.f : fast_exp2(mw - mx);
          num = fmaf(src[d], f, num);
          den = fmaf(src[D + 1], f, den);
        }
      }
      const long long row_id = ((long long)b * a.sq + qi) * a.heads + h;
      const float val = den > 0.f ? num / den : 0.f;
      if (kContiguous && sg.piece) {
        a.slot_o[(my_slot * kRows + r) * D + d] = val;
        if (d == 0) a.slot_lse[my_slot * kRows + r] = den > 0.f ? mx + fast_log2(den) : kEmptyLse;
      } else if (a.write_partials) {
        a.part_o[(row_id * a.splits + s) * D + d] = val;
        if (d == 0) a.part_lse[row_id * a.splits + s] = den > 0.f ? mx + fast_log2(den) : kEmptyLse;
      } else {
        reinterpret_cast<T*>(a.out)[row_id * D + d] = Tr::from_float(val);
      }
    }
    if (kContiguous && sg.piece) {
      // Piece merge in place: every piece publishes its partial, then counts itself in on the item's counter;
      // the piece whose arrival completes the set merges all pieces from their slots in piece order (the split
      // merge's arithmetic), so the output does not depend on which CTA finished last. No CTA waits for another.
      __shared__ int piece_merge_here;
      __threadfence();
      named_barrier_sync(1, consumer_threads);
      if (threadIdx.x == 0) piece_merge_here = atomicAdd(&a.counters[sg.item], 1) + 1 == pieces;
      named_barrier_sync(1, consumer_threads);
      if (piece_merge_here) {
        __threadfence();
        if (threadIdx.x == 0) a.counters[sg.item] = 0;  // ready for the next launch
        for (int idx = threadIdx.x; idx < kRows * D; idx += consumer_threads) {
          const int r = idx / D;
          const int d = idx % D;
          const int qi = q0 + r;
          if (qi >= a.sq) continue;
          float peak = kEmptyLse, total = 0.f, accm = 0.f;
          constexpr int kChunk = 8;  // pieces whose loads are in flight together
          for (int k0 = 0; k0 < pieces; k0 += kChunk) {
            float lse[kChunk], o[kChunk];
#pragma unroll
            for (int c = 0; c < kChunk; ++c) {
              if (k0 + c < pieces) {
                const long long slot = piece_slot(q_first, first_extra, k0 + c);
                lse[c] = __ldcg(a.slot_lse + slot * kRows + r);
                o[c] = __ldcg(a.slot_o + (slot * kRows + r) * D + d);
              }
            }
#pragma unroll
            for (int c = 0; c < kChunk; ++c) {
              if (k0 + c < pieces) {
                float w_old, w_new;
                merge_split_weights(lse[c], peak, total, w_old, w_new);
                accm = merge_split_accumulate(accm, w_old, w_new, o[c]);
              }
            }
          }
          const long long row_id = ((long long)b * a.sq + qi) * a.heads + h;
          reinterpret_cast<T*>(a.out)[row_id * D + d] = Tr::from_float(merge_split_finish(accm, total));
        }
      }
    }
    if (a.fused_merge) {
      // Split merge in place: every split's CTA publishes its partial, then counts itself in on the
      // group's counter; the one whose arrival completes the set merges all the group's partials in
      // split order (the arithmetic of merge_kernel, so the output is the same bits whichever CTA merges).
      // No CTA ever waits for another.
      __shared__ int merge_here;
      __threadfence();
      named_barrier_sync(1, consumer_threads);
      if (threadIdx.x == 0) {
        const long long g = ((long long)b * a.row_blocks + rb) * a.heads + h;
        merge_here = atomicAdd(&a.merge_counters[g], 1) == a.splits - 1;
      }
      named_barrier_sync(1, consumer_threads);
      if (merge_here) {
        __threadfence();
        for (int idx = threadIdx.x; idx < kRows * D; idx += consumer_threads) {
          const int r = idx / D;
          const int d = idx % D;
          const int qi = q0 + r;
          if (qi >= a.sq) continue;
          const long long row_id = ((long long)b * a.sq + qi) * a.heads + h;
          const float* lse_row = a.part_lse + row_id * a.splits;
          const float* o_row = a.part_o + row_id * a.splits * D + d;
          // through L2 (ld.global.cg): other CTAs of this launch wrote these partials
          float peak = kEmptyLse, total = 0.f, accm = 0.f;
          constexpr int kChunk = 16;  // splits whose loads are in flight together
          for (int s0 = 0; s0 < a.splits; s0 += kChunk) {
            float lse[kChunk], o[kChunk];
#pragma unroll
            for (int c = 0; c < kChunk; ++c) {
              if (s0 + c < a.splits) {
                lse[c] = __ldcg(lse_row + s0 + c);
                o[c] = __ldcg(o_row + (long long)(s0 + c) * D);
              }
            }
#pragma unroll
            for (int c = 0; c < kChunk; ++c) {
              if (s0 + c < a.splits) {
                float w_old, w_new;
                merge_split_weights(lse[c], peak, total, w_old, w_new);
                accm = merge_split_accumulate(accm, w_old, w_new, o[c]);
              }
            }
          }
          reinterpret_cast<T*>(a.out)[row_id * D + d] = Tr::from_float(merge_split_finish(accm, total));
        }
      }
    }
    named_barrier_sync(1, consumer_threads);
  }
}

template <typename T, int D>
static cudaError_t launch_decode_t(const LaunchDesc& d, const DecodeArgs& args, const CUtensorMap& kmap,
                                   const CUtensorMap& vmap) {
  using S = DecodeShape<D>;
  using M = DecodeSmem<T, D>;
  auto kernel = args.contiguous ? decode_kernel<T, D, true> : decode_kernel<T, D, false>;
  cudaError_t err = prepare_kernel(reinterpret_cast<const void*>(kernel), M::kBytes, d.device, nullptr);
  if (err != cudaSuccess) return err;
  long long grid = args.items;
  const long long cap = d.p.grid_cap > 0 ? d.p.grid_cap : d.sm_count;
  grid = args.contiguous ? args.programs : std::min(grid, cap);
  if (grid <= 0) return cudaSuccess;
  return launch_after_plan(kernel, (unsigned)grid, S::kThreads, M::kBytes, d.stream, kmap, vmap, args);
}

// Tokens per pipeline stage of the decode kernel for this head dimension (the TMA box rows must divide it).
int decode_tile_tokens(int head_dim) {
  switch (head_dim) {
#define FGW_TILE_CASE(DD) \
  case DD:                \
    return DecodeShape<DD>::kTile;
    FGW_TILE_CASE(16)
    FGW_TILE_CASE(32)
    FGW_TILE_CASE(48)
    FGW_TILE_CASE(64)
    FGW_TILE_CASE(80)
    FGW_TILE_CASE(96)
    FGW_TILE_CASE(112)
    FGW_TILE_CASE(128)
    FGW_TILE_CASE(144)
    FGW_TILE_CASE(160)
    FGW_TILE_CASE(176)
    FGW_TILE_CASE(192)
    FGW_TILE_CASE(208)
    FGW_TILE_CASE(224)
    FGW_TILE_CASE(240)
    FGW_TILE_CASE(256)
#undef FGW_TILE_CASE
    default:
      return 64;
  }
}

int decode_rows_per_item(int head_dim) {
  switch (head_dim) {
#define FGW_ROWS_CASE(DD) \
  case DD:                \
    return DecodeShape<DD>::kRows;
    FGW_ROWS_CASE(16)
    FGW_ROWS_CASE(32)
    FGW_ROWS_CASE(48)
    FGW_ROWS_CASE(64)
    FGW_ROWS_CASE(80)
    FGW_ROWS_CASE(96)
    FGW_ROWS_CASE(112)
    FGW_ROWS_CASE(128)
    FGW_ROWS_CASE(144)
    FGW_ROWS_CASE(160)
    FGW_ROWS_CASE(176)
    FGW_ROWS_CASE(192)
    FGW_ROWS_CASE(208)
    FGW_ROWS_CASE(224)
    FGW_ROWS_CASE(240)
    FGW_ROWS_CASE(256)
#undef FGW_ROWS_CASE
    default:
      return 1;
  }
}

static int gcd_int(int x, int y) {
  while (y) {
    const int t = x % y;
    x = y;
    y = t;
  }
  return x;
}

static bool make_kv_map(CUtensorMap* map, const void* base, const fgw_mha_params& p, int box_rows) {
  const cuuint64_t dims[3] = {(cuuint64_t)p.head_dim, (cuuint64_t)p.heads, (cuuint64_t)p.pool_rows};
  const cuuint64_t strides[2] = {(cuuint64_t)p.head_dim * 2, (cuuint64_t)p.heads * p.head_dim * 2};
  const cuuint32_t box[3] = {(cuuint32_t)p.head_dim, 1, (cuuint32_t)box_rows};
  const cuuint32_t estride[3] = {1, 1, 1};
  const CUtensorMapDataType dt =
      p.dtype == FGW_DTYPE_BFLOAT16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = encode_tiled_cached(map, dt, 3, const_cast<void*>(base), dims, strides, box, estride,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

cudaError_t launch_decode(const LaunchDesc& d, bool write_partials, bool fused_merge) {
  const fgw_mha_params& p = d.p;
  const int rows = decode_rows_per_item(p.head_dim);
  DecodeArgs args;
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
  args.width = p.table_width;
  args.page = p.page_size;
  args.splits = p.num_splits;
  args.causal = p.causal;
  args.row_blocks = (p.q_len + rows - 1) / rows;
  args.box_rows = gcd_int(gcd_int(p.page_size, decode_tile_tokens(p.head_dim)), 256);  // divides page and tile
  args.write_partials = write_partials ? 1 : 0;
  args.fused_merge = (write_partials && fused_merge && d.merge_counters != nullptr) ? 1 : 0;
  args.merge_counters = d.merge_counters;
  args.contiguous = d.contiguous ? 1 : 0;
  args.programs = d.contiguous ? d.programs : 0;
  args.tail_start = d.contiguous ? d.tail_start : 0;
  args.prog_item = d.prog_item;
  args.prog_off = d.prog_off;
  args.prog_u = d.prog_u;
  args.counters = d.counters;
  args.slot_lse = d.slot_lse;
  args.slot_o = d.slot_o;
  args.items = (long long)p.batch * args.row_blocks * p.num_splits * p.heads;
  args.scale_log2 = (1.0f / sqrtf((float)p.head_dim)) * kLog2e;
  args.budget_ns = d.budget_ns;

  CUtensorMap kmap, vmap;
  if (!make_kv_map(&kmap, p.k_cache, p, args.box_rows) || !make_kv_map(&vmap, p.v_cache, p, args.box_rows)) {
    return cudaErrorInvalidValue;
  }
  const bool bf16 = p.dtype == FGW_DTYPE_BFLOAT16;
  switch (p.head_dim) {
#define FGW_DECODE_CASE(DD)                                                          \
  case DD:                                                                           \
    return bf16 ? launch_decode_t<__nv_bfloat16, DD>(d, args, kmap, vmap)            \
                : launch_decode_t<__half, DD>(d, args, kmap, vmap);
    FGW_DECODE_CASE(16)
    FGW_DECODE_CASE(32)
    FGW_DECODE_CASE(48)
    FGW_DECODE_CASE(64)
    FGW_DECODE_CASE(80)
    FGW_DECODE_CASE(96)
    FGW_DECODE_CASE(112)
    FGW_DECODE_CASE(128)
    FGW_DECODE_CASE(144)
    FGW_DECODE_CASE(160)
    FGW_DECODE_CASE(176)
    FGW_DECODE_CASE(192)
    FGW_DECODE_CASE(208)
    FGW_DECODE_CASE(224)
    FGW_DECODE_CASE(240)
    FGW_DECODE_CASE(256)
#undef FGW_DECODE_CASE
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace fgw
