// Planning and merge kernels.
//
// plan_kernel: clears the workspace error word, clamps cache lengths into [0, width * page]
//   and orders request rows by descending length, so persistent CTAs walking the work list
//   round-robin start with the longest requests (longest-processing-time-first). This is the
//   length-aware part of the reference's persistent scheduler (v7.py:112-113, 260-270), moved
//   onto the device so no length ever has to cross to the host.
//   With the contiguous schedule it also lays the work items (the two-tile kernel's, or the decode kernel's)
//   end to end and cuts them into one equal range of KV units per program (StreamPlanArgs below).
// merge_kernel: LSE-weighted merge of split-KV partials, one warp per output row; replaces the
//   reference merge prim_funcs (v7.py:317-371, cube_general.py:224-279). Partials carry a base-2
//   LSE; the empty-split sentinel and validity threshold keep the reference's -1e30 / -1e29. The
//   arithmetic is merge_split_* (fgw_common.cuh), shared with the decode kernel's fused merge.
//   plan_kernel also zeroes the decode kernel's per-group arrival counters when it merges in place.
#include "fgw_common.cuh"
#include "fgw_kernels.h"

namespace fgw {

constexpr int kPlanSortMax = 8192;

// Contiguous schedule, planned on the device from the clamped lengths: the work items of the two-tile
// kernel in its item order (under the tail schedule only those of the last, partial wave), each counting
// max(KV tiles, 1) units; program p gets units [p * (total / G) + min(p, total % G), ...) as in the
// reference's balanced plan (static_schedule.py:64-66).
struct StreamPlanArgs {
  // tensor path: items of `block_rows` query rows (256: the two-tile kernel, 128: the key-halves kernel),
  // `qblocks` of them per (request, head)
  int enabled, items, programs, heads, sq, causal, qblocks, block_rows;
  // decode path (decode != 0): items are (request, query-row block, head) with `rows` query rows each and
  // `tile`-token KV units (the decode kernel's stage), `row_blocks` blocks per request
  int decode, rows, tile, row_blocks;
  int first;  // first item of the cut range (0, or the items of the full waves under the tail schedule)
  int32_t* prog_item;
  int32_t* prog_off;
  long long* prog_u;
  long long* prefix;
  int32_t* counters;
};

// Units of work item `item` (KV tiles seen by its last query row; at least 1): the tensor kernels' item
// decomposition with one split (pair_item in fgw_fmha2_sm100.cu, halves_item in fgw_fmha_halves_sm100.cu).
__device__ __forceinline__ long long stream_item_units(const StreamPlanArgs& s, const int32_t* lens,
                                                       const int32_t* order, int item) {
  if (s.decode) {
    // decode_item in fgw_decode.cu with one split: heads innermost, then the query-row block
    const int rest = item / s.heads;
    const int rb = rest % s.row_blocks;
    const int len = lens[order[rest / s.row_blocks]];
    const int last = min(rb * s.rows + s.rows, s.sq) - 1;
    const int visible = s.causal ? max(len - s.sq + last + 1, 0) : len;
    return max((visible + s.tile - 1) / s.tile, 1);
  }
  const int p_rev = item % s.qblocks;
  const int b = order[(item / s.qblocks) / s.heads];
  const int q0 = (s.qblocks - 1 - p_rev) * s.block_rows;
  const int last = min(q0 + s.block_rows, s.sq) - 1;
  const int len = lens[b];
  const int visible = s.causal ? max(len - s.sq + last + 1, 0) : len;
  return max((visible + 127) / 128, 1);
}

__device__ __forceinline__ long long stream_program_start(long long total, int programs, int p) {
  return static_cast<long long>(p) * (total / programs) + min(static_cast<long long>(p), total % programs);
}

__global__ void __launch_bounds__(1024) plan_kernel(const int32_t* __restrict__ lengths, int32_t* __restrict__ lens,
                                                   int32_t* __restrict__ order, WorkspaceHeader* ws, int batch,
                                                   int capacity, StreamPlanArgs sp, int32_t* merge_counters,
                                                   int merge_groups) {
  extern __shared__ unsigned long long keys[];
  __shared__ long long chunk_sum[1024];
  grid_dependents_launch();  // the attention launch may start its set-up; it waits for this grid to finish
  if (threadIdx.x == 0) {
    ws->error = 0;
    ws->error_site = 0;
    ws->finished = 0;
    ws->next_item = 0;
  }
  // the decode kernel's fused split merge counts arrivals per row group from zero
  for (int i = threadIdx.x; i < merge_groups; i += blockDim.x) merge_counters[i] = 0;
  for (int i = threadIdx.x; i < batch; i += blockDim.x) {
    lens[i] = min(max(lengths[i], 0), capacity);
  }
  if (batch > kPlanSortMax) {
    for (int i = threadIdx.x; i < batch; i += blockDim.x) order[i] = i;
  } else {
    int n = 1;
    while (n < batch) n <<= 1;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      if (i < batch) {
        const unsigned len = static_cast<unsigned>(min(max(lengths[i], 0), capacity));
        keys[i] = (static_cast<unsigned long long>(0x7fffffffu - len) << 32) | static_cast<unsigned>(i);
      } else {
        keys[i] = ~0ull;
      }
    }
    __syncthreads();
    for (int k = 2; k <= n; k <<= 1) {
      for (int j = k >> 1; j > 0; j >>= 1) {
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
          const int ixj = i ^ j;
          if (ixj > i) {
            const bool ascending = (i & k) == 0;
            const unsigned long long x = keys[i], y = keys[ixj];
            if ((x > y) == ascending) {
              keys[i] = y;
              keys[ixj] = x;
            }
          }
        }
        __syncthreads();
      }
    }
    for (int i = threadIdx.x; i < batch; i += blockDim.x) order[i] = static_cast<int32_t>(keys[i] & 0xffffffffu);
  }
  if (!sp.enabled) return;
  __syncthreads();  // lens and order are read below by other threads of this block
  // exclusive prefix of the units of items [first, items) (indices relative to `first`): each thread sums a
  // contiguous chunk, the chunk sums are scanned
  const int n = sp.items - sp.first;
  const int per = (n + blockDim.x - 1) / blockDim.x;
  const int lo = min(n, static_cast<int>(threadIdx.x) * per);
  const int hi = min(n, lo + per);
  long long local = 0;
  for (int i = lo; i < hi; ++i) {
    local += stream_item_units(sp, lens, order, sp.first + i);
    sp.counters[sp.first + i] = 0;
  }
  chunk_sum[threadIdx.x] = local;
  __syncthreads();
  if (threadIdx.x == 0) {
    long long run = 0;
    for (int t = 0; t < static_cast<int>(blockDim.x); ++t) {
      const long long v = chunk_sum[t];
      chunk_sum[t] = run;
      run += v;
    }
    sp.prefix[n] = run;
  }
  __syncthreads();
  long long run = chunk_sum[threadIdx.x];
  for (int i = lo; i < hi; ++i) {
    sp.prefix[i] = run;
    run += stream_item_units(sp, lens, order, sp.first + i);
  }
  __syncthreads();
  // program starts: the item holding unit U_p (the last item whose first unit is <= U_p)
  const long long total = sp.prefix[n];
  for (int p = threadIdx.x; p <= sp.programs; p += blockDim.x) {
    const long long u = stream_program_start(total, sp.programs, p);
    sp.prog_u[p] = u;
    if (p == sp.programs) continue;
    int a = 0, b = n;  // prefix[a] <= u < prefix[b] (b == n when u == total)
    while (b - a > 1) {
      const int mid = (a + b) / 2;
      if (sp.prefix[mid] <= u) {
        a = mid;
      } else {
        b = mid;
      }
    }
    if (u >= total) {
      sp.prog_item[p] = sp.items;
      sp.prog_off[p] = 0;
    } else {
      sp.prog_item[p] = sp.first + a;
      sp.prog_off[p] = static_cast<int32_t>(u - sp.prefix[a]);
    }
  }
}

cudaError_t launch_plan(const LaunchDesc& d) {
  const int batch = d.p.batch;
  int n = 1;
  while (n < batch) n <<= 1;
  const size_t smem = batch <= kPlanSortMax ? n * sizeof(unsigned long long) : 0;
  if (smem > 32 * 1024) {
    cudaError_t err = prepare_kernel(reinterpret_cast<const void*>(plan_kernel), (int)smem, d.device, nullptr);
    if (err != cudaSuccess) return err;
  }
  StreamPlanArgs sp{};
  if (d.contiguous) {
    sp.enabled = 1;
    sp.items = d.items;
    sp.first = d.tail_start;
    sp.programs = d.programs;
    sp.heads = d.p.heads;
    sp.sq = d.p.q_len;
    sp.causal = d.p.causal;
    sp.block_rows = d.slot_rows;  // one work item's query rows
    sp.qblocks = (d.p.q_len + sp.block_rows - 1) / sp.block_rows;
    if (resolve_path(d.p) == FGW_PATH_DECODE) {
      sp.decode = 1;
      sp.rows = decode_rows_per_item(d.p.head_dim);
      sp.tile = decode_tile_tokens(d.p.head_dim);
      sp.row_blocks = (d.p.q_len + sp.rows - 1) / sp.rows;
    }
    sp.prog_item = d.prog_item;
    sp.prog_off = d.prog_off;
    sp.prog_u = d.prog_u;
    sp.prefix = d.prefix;
    sp.counters = d.counters;
  }
  plan_kernel<<<1, 1024, smem, d.stream>>>(d.p.cache_seqlens, d.lens, d.order, d.header, batch,
                                          d.p.table_width * d.p.page_size, sp, d.merge_counters, d.merge_groups);
  return cudaGetLastError();
}

template <typename T>
__global__ void __launch_bounds__(256) merge_kernel(const float* __restrict__ part_o,
                                                   const float* __restrict__ part_lse, T* __restrict__ out,
                                                   long long rows, int splits, int dim) {
  const long long row = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (row >= rows) return;
  constexpr int kMaxPerLane = 8;  // dim <= 256
  float acc[kMaxPerLane];
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) acc[i] = 0.f;
  float peak = kEmptyLse, total = 0.f;
  const float* lse_row = part_lse + row * splits;
  const float* o_row = part_o + row * splits * dim;
  constexpr int kChunk = 8;  // splits whose loads are in flight together
  for (int s0 = 0; s0 < splits; s0 += kChunk) {
    float lse[kChunk], o[kChunk][kMaxPerLane];
#pragma unroll
    for (int c = 0; c < kChunk; ++c) {
      if (s0 + c < splits) {
        lse[c] = lse_row[s0 + c];
        const float* src = o_row + (s0 + c) * dim;
#pragma unroll
        for (int i = 0; i < kMaxPerLane; ++i) o[c][i] = lane + 32 * i < dim ? src[lane + 32 * i] : 0.f;
      }
    }
#pragma unroll
    for (int c = 0; c < kChunk; ++c) {
      if (s0 + c < splits) {
        float w_old, w_new;
        merge_split_weights(lse[c], peak, total, w_old, w_new);
#pragma unroll
        for (int i = 0; i < kMaxPerLane; ++i) acc[i] = merge_split_accumulate(acc[i], w_old, w_new, o[c][i]);
      }
    }
  }
  T* dst = out + row * dim;
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int d = lane + 32 * i;
    if (d < dim) dst[d] = ElemTraits<T>::from_float(merge_split_finish(acc[i], total));
  }
}

cudaError_t launch_merge(const LaunchDesc& d) {
  const fgw_mha_params& p = d.p;
  const long long rows = (long long)p.batch * p.q_len * p.heads;
  const long long threads = rows * 32;
  const unsigned blocks = (unsigned)((threads + 255) / 256);
  if (blocks == 0) return cudaSuccess;
  if (p.dtype == FGW_DTYPE_BFLOAT16) {
    merge_kernel<__nv_bfloat16><<<blocks, 256, 0, d.stream>>>(d.part_o, d.part_lse,
                                                              reinterpret_cast<__nv_bfloat16*>(p.out), rows,
                                                              p.num_splits, p.head_dim);
  } else {
    merge_kernel<__half><<<blocks, 256, 0, d.stream>>>(d.part_o, d.part_lse, reinterpret_cast<__half*>(p.out), rows,
                                                       p.num_splits, p.head_dim);
  }
  return cudaGetLastError();
}

// Failure-detection self-test (fgw_mha_selftest_wait): the library's bounded wait on a phase nobody
// completes gives up after the budget and records the timeout; nothing traps or faults.
__global__ void wait_selftest_kernel(WorkspaceHeader* ws, uint64_t budget_ns, int complete) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    ws->error = 0;
    ws->error_site = 0;
    mbar_init(&bar, 1);
    fence_barrier_init();
    if (complete) mbar_arrive(&bar);
    if (!mbar_wait(&bar, 0, budget_ns)) record_error(ws, FGW_ERR_DEVICE_TIMEOUT, 99);
  }
}

cudaError_t launch_wait_selftest(WorkspaceHeader* ws, uint64_t budget_ns, int complete, cudaStream_t stream) {
  wait_selftest_kernel<<<1, 32, 0, stream>>>(ws, budget_ns, complete);
  return cudaGetLastError();
}

}  // namespace fgw
