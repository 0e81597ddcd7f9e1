// Planning and merge kernels.
//
// plan_kernel: clears the workspace error word, clamps cache lengths into [0, width * page]
//   and orders request rows by descending length, so persistent CTAs walking the work list
//   round-robin start with the longest requests (longest-processing-time-first). This is the
//   length-aware part of the reference's persistent scheduler (v7.py:112-113, 260-270), moved
//   onto the device so no length ever has to cross to the host.
// merge_kernel: LSE-weighted merge of split-KV partials, one warp per output row; replaces the
//   reference merge prim_funcs (v7.py:317-371, cube_general.py:224-279). Partials carry a base-2
//   LSE; the empty-split sentinel and validity threshold keep the reference's -1e30 / -1e29.
#include "fgw_common.cuh"
#include "fgw_kernels.h"

namespace fgw {

constexpr int kPlanSortMax = 8192;

__global__ void __launch_bounds__(1024) plan_kernel(const int32_t* __restrict__ lengths, int32_t* __restrict__ lens,
                                                   int32_t* __restrict__ order, WorkspaceHeader* ws, int batch,
                                                   int capacity) {
  extern __shared__ unsigned long long keys[];
  if (threadIdx.x == 0) {
    ws->error = 0;
    ws->error_site = 0;
  }
  for (int i = threadIdx.x; i < batch; i += blockDim.x) {
    lens[i] = min(max(lengths[i], 0), capacity);
  }
  if (batch > kPlanSortMax) {
    for (int i = threadIdx.x; i < batch; i += blockDim.x) order[i] = i;
    return;
  }
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

cudaError_t launch_plan(const LaunchDesc& d) {
  const int batch = d.p.batch;
  int n = 1;
  while (n < batch) n <<= 1;
  const size_t smem = batch <= kPlanSortMax ? n * sizeof(unsigned long long) : 0;
  if (smem > 48 * 1024) {
    cudaError_t err = cudaFuncSetAttribute(plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess) return err;
  }
  plan_kernel<<<1, 1024, smem, d.stream>>>(d.p.cache_seqlens, d.lens, d.order, d.header, batch,
                                          d.p.table_width * d.p.page_size);
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
  for (int s = 0; s < splits; ++s) {
    const float lse = lse_row[s];
    const float next = fmaxf(peak, lse);
    const float w_old = fast_exp2(peak - next);
    const float w_new = lse > kValidLse ? fast_exp2(lse - next) : 0.f;
    const float* src = o_row + s * dim;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      const int d = lane + 32 * i;
      if (d < dim) acc[i] = acc[i] * w_old + (w_new != 0.f ? src[d] * w_new : 0.f);
    }
    total = total * w_old + w_new;
    peak = next;
  }
  const float inv = 1.f / fmaxf(total, 1e-30f);
  T* dst = out + row * dim;
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int d = lane + 32 * i;
    if (d < dim) dst[d] = ElemTraits<T>::from_float(acc[i] * inv);
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

}  // namespace fgw
