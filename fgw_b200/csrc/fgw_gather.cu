// Paged-cache gather: copies the rows of a paged KV cache that the requests reach, in request order, into a
// dense buffer (fgw_paged_cache_gather in include/fgw_mha.h).
//
// Reference: the TileOPs paged-cache gather FGW pins as its pre-pass experiment
// (third_party/tileops_yyttt6/paged_cache_gather.py:108-232 `_compile`, :44-104 `_compile_generic`,
// :264-296 `forward`), driven by benchmarks/mha/external_cache_gather.py:38-58. Row r of request i
// (cu[i] <= r < cu[i+1]) receives cache row table[i, pos / page] * page + pos % page, pos = r - cu[i] + start[i];
// FP8 rows are multiplied by the scale and rounded to the output type.
//
// B200 design: the copy is HBM-bound byte moving, so it is not staged through shared memory. Consecutive
// positions inside one page are consecutive physical rows, so every (request, page) run of rows is one
// contiguous range in both the cache and the output: each CTA walks its contiguous range of output rows
// run by run and copies each run with 16-byte vector loads and stores from all of its threads, four in
// flight per thread. Lengths, page ids and offsets stay device data; nothing is copied to the host.
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include <algorithm>

#include "fgw_common.cuh"
#include "fgw_kernels.h"

namespace fgw {

struct GatherArgs {
  void* dst;
  const void* cache;
  const int32_t* table;
  const int32_t* cu;
  const int32_t* starts;
  const float* scale;
  long long total;
  int batch, num_pages, page, width, row;  // row: elements per cache row
  bool vec;                                // 16-byte vector path (row bytes and both bases 16-byte aligned)
};

constexpr int kGatherThreads = 256;
constexpr int kGatherUnroll = 4;

template <typename TOut>
__device__ __forceinline__ TOut gather_from_float(float x);
template <>
__device__ __forceinline__ __half gather_from_float<__half>(float x) {
  return __float2half_rn(x);
}
template <>
__device__ __forceinline__ __nv_bfloat16 gather_from_float<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

// Copy `n` consecutive cache rows starting at `src_row` to output rows starting at `dst_row` (src_row < 0:
// write zeros). Same element type in and out.
template <typename T>
__device__ __forceinline__ void copy_run(const GatherArgs& g, long long src_row, long long dst_row, long long n) {
  const long long elems = n * g.row;
  T* dst = reinterpret_cast<T*>(g.dst) + dst_row * g.row;
  const T* src = reinterpret_cast<const T*>(g.cache) + (src_row >= 0 ? src_row : 0) * g.row;
  if (g.vec) {
    const long long n16 = elems * static_cast<long long>(sizeof(T)) / 16;
    uint4* d = reinterpret_cast<uint4*>(dst);
    const uint4* s = reinterpret_cast<const uint4*>(src);
    const long long step = static_cast<long long>(kGatherThreads) * kGatherUnroll;
    for (long long base = threadIdx.x; base < n16; base += step) {
      uint4 v[kGatherUnroll];
#pragma unroll
      for (int u = 0; u < kGatherUnroll; ++u) {
        const long long i = base + static_cast<long long>(u) * kGatherThreads;
        v[u] = (i < n16 && src_row >= 0) ? s[i] : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < kGatherUnroll; ++u) {
        const long long i = base + static_cast<long long>(u) * kGatherThreads;
        if (i < n16) d[i] = v[u];
      }
    }
  } else {
    for (long long i = threadIdx.x; i < elems; i += kGatherThreads) {
      dst[i] = src_row >= 0 ? src[i] : T();
    }
  }
}

// FP8 (E4M3) rows: out = round(float(code) * scale) in the output type.
template <typename TOut>
__device__ __forceinline__ void copy_run_fp8(const GatherArgs& g, long long src_row, long long dst_row, long long n,
                                             float scale) {
  const long long elems = n * g.row;
  TOut* dst = reinterpret_cast<TOut*>(g.dst) + dst_row * g.row;
  const __nv_fp8_e4m3* src = reinterpret_cast<const __nv_fp8_e4m3*>(g.cache) + (src_row >= 0 ? src_row : 0) * g.row;
  if (g.vec) {
    // 16 codes in, 16 outputs (two 16-byte stores) out per thread and step
    const long long n16 = elems / 16;
    const uint4* s = reinterpret_cast<const uint4*>(src);
    uint4* d = reinterpret_cast<uint4*>(dst);
    for (long long i = threadIdx.x; i < n16; i += kGatherThreads) {
      const uint4 raw = src_row >= 0 ? s[i] : make_uint4(0, 0, 0, 0);
      const uint32_t words[4] = {raw.x, raw.y, raw.z, raw.w};
      TOut out[16];
#pragma unroll
      for (int w = 0; w < 4; ++w) {
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          __nv_fp8_e4m3 code;
          code.__x = static_cast<__nv_fp8_storage_t>((words[w] >> (8 * b)) & 0xffu);
          out[4 * w + b] = src_row >= 0 ? gather_from_float<TOut>(static_cast<float>(code) * scale)
                                        : gather_from_float<TOut>(0.f);
        }
      }
      d[2 * i] = *reinterpret_cast<const uint4*>(&out[0]);
      d[2 * i + 1] = *reinterpret_cast<const uint4*>(&out[8]);
    }
  } else {
    for (long long i = threadIdx.x; i < elems; i += kGatherThreads) {
      dst[i] = src_row >= 0 ? gather_from_float<TOut>(static_cast<float>(src[i]) * scale) : gather_from_float<TOut>(0.f);
    }
  }
}

template <typename TIn, typename TOut>
__global__ void __launch_bounds__(kGatherThreads) gather_kernel(const GatherArgs g) {
  const long long per = (g.total + gridDim.x - 1) / gridDim.x;
  long long row = static_cast<long long>(blockIdx.x) * per;
  const long long end = min(g.total, row + per);
  if (row >= end) return;
  const float scale = g.scale != nullptr ? *g.scale : 1.f;
  // the last request i in [0, batch) with cu[i] <= row (0 when row lies before cu[0])
  int lo = 0, hi = g.batch - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) / 2;
    if (g.cu[mid] <= row) {
      lo = mid;
    } else {
      hi = mid - 1;
    }
  }
  int req = lo;
  // Every thread walks the same runs (uniform scalar loop; the metadata reads are broadcasts).
  while (row < end) {
    while (req + 1 < g.batch && g.cu[req + 1] <= row) ++req;
    const long long first = g.cu[req], last = g.cu[req + 1];
    long long run_end = end;
    long long src_row = -1;  // -1: zeros
    if (row < first) {
      run_end = min(end, first);  // rows before the first request's offset
    } else if (row >= last) {
      run_end = end;              // rows past cu[batch]
    } else {
      const long long pos = row - first + (g.starts != nullptr ? g.starts[req] : 0);
      run_end = min(end, last);
      if (pos < 0) {
        run_end = min(run_end, row - pos);
      } else if (pos / g.page < g.width) {
        const long long in_page = pos % g.page;
        run_end = min(run_end, row + (g.page - in_page));
        const long long page_id = g.table[static_cast<long long>(req) * g.width + pos / g.page];
        if (page_id >= 0 && page_id < g.num_pages) src_row = page_id * g.page + in_page;
      }
      // positions past the table, and page ids outside the pool, give zero rows (never an out-of-bounds read)
    }
    if constexpr (sizeof(TIn) == 1) {
      copy_run_fp8<TOut>(g, src_row, row, run_end - row, scale);
    } else {
      copy_run<TIn>(g, src_row, row, run_end - row);
    }
    row = run_end;
  }
}

static int dtype_bytes(int dtype) {
  switch (dtype) {
    case FGW_DTYPE_FLOAT16:
    case FGW_DTYPE_BFLOAT16:
      return 2;
    case FGW_DTYPE_FLOAT8_E4M3:
      return 1;
    default:
      return 0;
  }
}

int gather_validate(const fgw_gather_params& p) {
  for (int r : p.reserved) {
    if (r != 0) return FGW_ERR_INVALID_ARGUMENT;
  }
  if (p.batch <= 0 || p.num_pages <= 0 || p.page_size <= 0 || p.table_width <= 0 || p.row_width <= 0 ||
      p.total_rows < 0) {
    return FGW_ERR_INVALID_ARGUMENT;
  }
  if (static_cast<long long>(p.page_size) * p.table_width > 0x7fffffffll) return FGW_ERR_INVALID_ARGUMENT;
  if (dtype_bytes(p.dtype) == 0 || dtype_bytes(p.out_dtype) != 2) return FGW_ERR_INVALID_ARGUMENT;
  const bool fp8 = p.dtype == FGW_DTYPE_FLOAT8_E4M3;
  if (!fp8 && p.out_dtype != p.dtype) return FGW_ERR_INVALID_ARGUMENT;  // an unquantized gather keeps the type
  if (fp8 != (p.scale != nullptr)) return FGW_ERR_INVALID_ARGUMENT;     // the scale goes with FP8 only
  if (p.total_rows > 0 && (p.dst == nullptr || p.cache == nullptr || p.block_table == nullptr ||
                           p.cu_seq_lens == nullptr)) {
    return FGW_ERR_INVALID_ARGUMENT;
  }
  return FGW_OK;
}

cudaError_t launch_gather(const fgw_gather_params& p, int sm_count, cudaStream_t stream) {
  if (p.total_rows == 0) return cudaSuccess;
  GatherArgs g;
  g.dst = p.dst;
  g.cache = p.cache;
  g.table = p.block_table;
  g.cu = p.cu_seq_lens;
  g.starts = p.seq_starts;
  g.scale = p.scale;
  g.total = p.total_rows;
  g.num_pages = p.num_pages;
  g.batch = p.batch;
  g.page = p.page_size;
  g.width = p.table_width;
  g.row = p.row_width;
  const bool fp8 = p.dtype == FGW_DTYPE_FLOAT8_E4M3;
  const uintptr_t dst_addr = reinterpret_cast<uintptr_t>(p.dst), src_addr = reinterpret_cast<uintptr_t>(p.cache);
  const long long in_row_bytes = static_cast<long long>(p.row_width) * dtype_bytes(p.dtype);
  const long long out_row_bytes = static_cast<long long>(p.row_width) * 2;
  g.vec = in_row_bytes % 16 == 0 && out_row_bytes % 16 == 0 && dst_addr % 16 == 0 && src_addr % 16 == 0;
  // about 32 KB of output per CTA, at most 8 resident CTAs per SM
  const long long bytes = p.total_rows * out_row_bytes;
  const long long grid = std::max(1ll, std::min<long long>((bytes + 32767) / 32768, 8ll * sm_count));
  const unsigned blocks = static_cast<unsigned>(std::min<long long>(grid, p.total_rows));
  if (fp8) {
    if (p.out_dtype == FGW_DTYPE_BFLOAT16) {
      gather_kernel<__nv_fp8_e4m3, __nv_bfloat16><<<blocks, kGatherThreads, 0, stream>>>(g);
    } else {
      gather_kernel<__nv_fp8_e4m3, __half><<<blocks, kGatherThreads, 0, stream>>>(g);
    }
  } else if (p.dtype == FGW_DTYPE_BFLOAT16) {
    gather_kernel<__nv_bfloat16, __nv_bfloat16><<<blocks, kGatherThreads, 0, stream>>>(g);
  } else {
    gather_kernel<__half, __half><<<blocks, kGatherThreads, 0, stream>>>(g);
  }
  return cudaGetLastError();
}

}  // namespace fgw
