// C ABI of libfgw_mha.so: argument validation, workspace carve-up, path choice and launch order.
// The host-side control flow mirrors the reference's launch callables (v7.py:471-498,
// cube_general.py:186-188, 284-288): one launch when there is one split, partial then merge
// otherwise (the decode path merges in the same launch, the CTA completing a row group's splits
// merging them), all on the caller's stream. A small planning launch precedes them and replaces the
// reference's host copy of the cache lengths (v7.py:548).
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "fgw_common.cuh"
#include "fgw_kernels.h"

namespace fgw {

static size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
  });
  return fn;
}

CUresult encode_tiled_cached(CUtensorMap* map, CUtensorMapDataType dtype, cuuint32_t rank, void* base,
                             const cuuint64_t* dims, const cuuint64_t* strides, const cuuint32_t* box,
                             const cuuint32_t* elem_strides, CUtensorMapInterleave interleave,
                             CUtensorMapSwizzle swizzle, CUtensorMapL2promotion l2, CUtensorMapFloatOOBfill fill) {
  struct Key {
    void* base;
    cuuint64_t dims[5], strides[4];
    cuuint32_t box[5], elem_strides[5];
    int dtype, rank, interleave, swizzle, l2, fill;
    bool operator==(const Key& o) const { return std::memcmp(this, &o, sizeof(Key)) == 0; }
  };
  struct Entry {
    Key key;
    CUtensorMap map;
  };
  constexpr int kEntries = 32;
  static std::mutex mu;
  static Entry cache[kEntries];
  static int used = 0, next = 0;
  if (rank < 1 || rank > 5) return CUDA_ERROR_INVALID_VALUE;
  Key k;
  std::memset(&k, 0, sizeof(k));
  k.base = base;
  for (cuuint32_t i = 0; i < rank; ++i) {
    k.dims[i] = dims[i];
    k.box[i] = box[i];
    k.elem_strides[i] = elem_strides[i];
    if (i + 1 < rank) k.strides[i] = strides[i];
  }
  k.dtype = dtype;
  k.rank = static_cast<int>(rank);
  k.interleave = interleave;
  k.swizzle = swizzle;
  k.l2 = l2;
  k.fill = fill;
  {
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < used; ++i) {
      if (cache[i].key == k) {
        *map = cache[i].map;
        return CUDA_SUCCESS;
      }
    }
  }
  const CUresult r = encode_tiled()(map, dtype, rank, base, dims, strides, box, elem_strides, interleave, swizzle,
                                    l2, fill);
  if (r != CUDA_SUCCESS) return r;
  std::lock_guard<std::mutex> lock(mu);
  cache[next].key = k;
  cache[next].map = *map;
  next = (next + 1) % kEntries;
  used = used < kEntries ? used + 1 : kEntries;
  return CUDA_SUCCESS;
}

// The tcgen05 kernel the tensor path runs for these parameters (FGW_TENSOR_KERNEL_AUTO resolved).
int resolve_tensor_kernel(const fgw_mha_params& p) {
  if (p.tensor_kernel != FGW_TENSOR_KERNEL_AUTO) return p.tensor_kernel;
  return p.head_dim <= 128 ? FGW_TENSOR_KERNEL_PAIRS : FGW_TENSOR_KERNEL_SINGLE;
}

long long pair_items(const fgw_mha_params& p) {
  return static_cast<long long>(p.batch) * p.heads * p.num_splits * ((p.q_len + kPairRows - 1) / kPairRows);
}

int stream_slot_rows(const fgw_mha_params& p) {
  if (resolve_path(p) == FGW_PATH_DECODE) return decode_rows_per_item(p.head_dim);
  return resolve_tensor_kernel(p) == FGW_TENSOR_KERNEL_HALVES ? 128 : kPairRows;
}

long long stream_items(const fgw_mha_params& p) {
  const int rows = stream_slot_rows(p);
  return static_cast<long long>(p.batch) * ((p.q_len + rows - 1) / rows) * p.heads * p.num_splits;
}

// Decode path, one split: CONTIGUOUS or TAIL when asked for; AUTO deals whole items dynamically (a counter hands
// the next item, longest request first with heads innermost, to whichever CTA asks), so the items in flight at
// once are consecutive ones (the heads of a few requests) and DRAM sees long runs of each token's rows; the
// contiguous cut gives every CTA the same number of KV stages, but its CTAs walk different requests' 256-byte
// head slices, which measured 0.75 of the HBM copy peak on config 5 against 0.99-1.03 for whole items.
// Tensor path, both tcgen05 kernels with contiguous forms (two-tile and key-halves): AUTO takes the contiguous
// schedule only when whole items would leave more than a third of the programs idle in their single wave
// (items < 2/3 of the programs). Measured on config 2 the strided schedule is faster: two-tile kernel (256
// items, two waves) 120 us strided against 174 us contiguous, key-halves kernel (512 items) 158 against 214 us,
// since cutting items adds segment starts and piece merges.
bool use_stream_schedule(const fgw_mha_params& p) {
  if (p.schedule == FGW_SCHEDULE_STRIDED || p.num_splits != 1) return false;
  if (stream_items(p) > kStreamMaxItems) return false;
  if (resolve_path(p) == FGW_PATH_DECODE) {
    return p.schedule == FGW_SCHEDULE_CONTIGUOUS || p.schedule == FGW_SCHEDULE_TAIL;
  }
  if (p.head_dim > 128) return false;
  const int kernel = resolve_tensor_kernel(p);
  if (kernel != FGW_TENSOR_KERNEL_PAIRS && kernel != FGW_TENSOR_KERNEL_HALVES) return false;
  return p.schedule == FGW_SCHEDULE_CONTIGUOUS || p.schedule == FGW_SCHEDULE_TAIL ||
         3 * stream_items(p) < 2ll * kStreamMaxPrograms;
}

namespace {
// Byte sizes of the contiguous-schedule regions, in workspace order.
struct StreamSizes {
  size_t prog_item, prog_off, prog_u, prefix, counters, slot_lse, slot_o;
  size_t total() const { return prog_item + prog_off + prog_u + prefix + counters + slot_lse + slot_o; }
};

StreamSizes stream_sizes(const fgw_mha_params& p) {
  const size_t programs = kStreamMaxPrograms;
  const size_t items = static_cast<size_t>(stream_items(p));
  const size_t rows = static_cast<size_t>(stream_slot_rows(p));
  StreamSizes z;
  z.prog_item = align256(programs * sizeof(int32_t));
  z.prog_off = align256(programs * sizeof(int32_t));
  z.prog_u = align256((programs + 1) * sizeof(long long));
  z.prefix = align256((items + 1) * sizeof(long long));
  z.counters = align256(items * sizeof(int32_t));
  z.slot_lse = align256(2 * programs * rows * sizeof(float));
  z.slot_o = align256(2 * programs * rows * static_cast<size_t>(p.head_dim) * sizeof(float));
  return z;
}
}  // namespace

// Split-KV on the decode path keeps one arrival counter per output row group (fused merge).
static bool decode_merge_counters(const fgw_mha_params& p, int path) {
  return p.num_splits > 1 && path == FGW_PATH_DECODE;
}

size_t workspace_bytes(const fgw_mha_params& p, int path) {
  size_t bytes = sizeof(WorkspaceHeader);
  bytes += align256(sizeof(int32_t) * p.batch);  // lens
  bytes += align256(sizeof(int32_t) * p.batch);  // order
  const size_t rows = static_cast<size_t>(p.batch) * p.q_len * p.heads;
  if (p.num_splits > 1) {
    bytes += align256(rows * p.num_splits * sizeof(float));
    bytes += align256(rows * p.num_splits * p.head_dim * sizeof(float));
  }
  if (use_stream_schedule(p)) bytes += stream_sizes(p).total();
  if (decode_merge_counters(p, path)) bytes += align256(rows * sizeof(int32_t));
  return bytes;
}

void carve_workspace(LaunchDesc& d, void* workspace, int path) {
  const fgw_mha_params& p = d.p;
  uint8_t* base = static_cast<uint8_t*>(workspace);
  d.header = reinterpret_cast<WorkspaceHeader*>(base);
  base += sizeof(WorkspaceHeader);
  d.lens = reinterpret_cast<int32_t*>(base);
  base += align256(sizeof(int32_t) * p.batch);
  d.order = reinterpret_cast<int32_t*>(base);
  base += align256(sizeof(int32_t) * p.batch);
  const size_t rows = static_cast<size_t>(p.batch) * p.q_len * p.heads;
  d.part_lse = reinterpret_cast<float*>(base);
  d.part_o = nullptr;
  if (p.num_splits > 1) {
    base += align256(rows * p.num_splits * sizeof(float));
    d.part_o = reinterpret_cast<float*>(base);
    base += align256(rows * p.num_splits * p.head_dim * sizeof(float));
  }
  d.contiguous = use_stream_schedule(p);
  if (d.contiguous) {
    const StreamSizes z = stream_sizes(p);
    d.items = static_cast<int>(stream_items(p));
    d.slot_rows = stream_slot_rows(p);
    d.prog_item = reinterpret_cast<int32_t*>(base);
    base += z.prog_item;
    d.prog_off = reinterpret_cast<int32_t*>(base);
    base += z.prog_off;
    d.prog_u = reinterpret_cast<long long*>(base);
    base += z.prog_u;
    d.prefix = reinterpret_cast<long long*>(base);
    base += z.prefix;
    d.counters = reinterpret_cast<int32_t*>(base);
    base += z.counters;
    d.slot_lse = reinterpret_cast<float*>(base);
    base += z.slot_lse;
    d.slot_o = reinterpret_cast<float*>(base);
    base += z.slot_o;
  }
  if (decode_merge_counters(p, path)) {
    d.merge_counters = reinterpret_cast<int32_t*>(base);
    d.merge_groups = static_cast<int>(rows);
  }
}

int resolve_path(const fgw_mha_params& p) {
  if (p.path == FGW_PATH_DECODE || p.path == FGW_PATH_TENSOR) return p.path;
  return p.q_len <= 8 ? FGW_PATH_DECODE : FGW_PATH_TENSOR;
}

static bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

static int validate(const fgw_mha_params* p) {
  if (p == nullptr) return FGW_ERR_INVALID_ARGUMENT;
  if (p->batch <= 0 || p->q_len <= 0 || p->heads <= 0 || p->head_dim <= 0) return FGW_ERR_INVALID_ARGUMENT;
  if (p->head_dim < 16 || p->head_dim > 256 || p->head_dim % 16) return FGW_ERR_INVALID_ARGUMENT;
  if (p->page_size <= 0 || p->page_size % 16) return FGW_ERR_INVALID_ARGUMENT;
  if (p->pool_rows <= 0 || p->pool_rows % p->page_size || p->pool_rows >= (1ll << 31)) {
    return FGW_ERR_INVALID_ARGUMENT;
  }
  if (p->table_width <= 0) return FGW_ERR_INVALID_ARGUMENT;
  if (static_cast<long long>(p->table_width) * p->page_size >= (1ll << 31)) return FGW_ERR_INVALID_ARGUMENT;
  if (p->dtype != FGW_DTYPE_FLOAT16 && p->dtype != FGW_DTYPE_BFLOAT16) return FGW_ERR_INVALID_ARGUMENT;
  if (p->causal != 0 && p->causal != 1) return FGW_ERR_INVALID_ARGUMENT;
  if (p->num_splits < 1 || p->num_splits > 1024) return FGW_ERR_INVALID_ARGUMENT;
  if (p->grid_cap < 0 || p->wait_budget_ms < 0) return FGW_ERR_INVALID_ARGUMENT;
  if (p->path < FGW_PATH_AUTO || p->path > FGW_PATH_TENSOR) return FGW_ERR_INVALID_ARGUMENT;
  if (p->schedule < FGW_SCHEDULE_AUTO || p->schedule > FGW_SCHEDULE_TAIL) return FGW_ERR_INVALID_ARGUMENT;
  if (p->tensor_kernel < FGW_TENSOR_KERNEL_AUTO || p->tensor_kernel > FGW_TENSOR_KERNEL_HALVES) {
    return FGW_ERR_INVALID_ARGUMENT;
  }
  for (int i = 0; i < 2; ++i) {
    if (p->reserved[i] != 0) return FGW_ERR_INVALID_ARGUMENT;
  }
  if (!p->q || !p->k_cache || !p->v_cache || !p->block_table || !p->cache_seqlens || !p->out) {
    return FGW_ERR_INVALID_ARGUMENT;
  }
  if (!aligned16(p->q) || !aligned16(p->k_cache) || !aligned16(p->v_cache) || !aligned16(p->out) ||
      (reinterpret_cast<uintptr_t>(p->block_table) & 3u) || (reinterpret_cast<uintptr_t>(p->cache_seqlens) & 3u)) {
    return FGW_ERR_INVALID_ARGUMENT;
  }
  return FGW_OK;
}

static int device_sm_count_cached(int device, int* sms) {
  static std::mutex mu;
  static int cache[64] = {0};
  if (device < 0 || device >= 64) return FGW_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[device] == 0) {
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return FGW_ERR_NO_DEVICE;
    if (prop.major != 10) return FGW_ERR_NO_DEVICE;
    cache[device] = prop.multiProcessorCount;
  }
  *sms = cache[device];
  return FGW_OK;
}

cudaError_t prepare_kernel(const void* kernel, int smem_bytes, int device, int* regs) {
  struct Prepared {
    const void* kernel;
    int device, smem_bytes, regs;
  };
  static std::mutex mu;
  static std::vector<Prepared> done;
  {
    std::lock_guard<std::mutex> lock(mu);
    for (const Prepared& k : done) {
      if (k.kernel == kernel && k.device == device && k.smem_bytes >= smem_bytes) {
        if (regs != nullptr) *regs = k.regs;
        return cudaSuccess;
      }
    }
  }
  cudaFuncAttributes attr;
  cudaError_t err = cudaFuncGetAttributes(&attr, kernel);
  if (err != cudaSuccess) return err;
  if (smem_bytes > 0) {
    err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
    if (err != cudaSuccess) return err;
  }
  std::lock_guard<std::mutex> lock(mu);
  done.push_back({kernel, device, smem_bytes, attr.numRegs});
  if (regs != nullptr) *regs = attr.numRegs;
  return cudaSuccess;
}

static int prepare(const fgw_mha_params* params, void* workspace, size_t workspace_bytes_given, void* stream,
                   LaunchDesc& d) {
  int st = validate(params);
  if (st != FGW_OK) return st;
  if (workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 255u)) return FGW_ERR_INVALID_ARGUMENT;
  std::memset(&d, 0, sizeof(d));
  d.p = *params;
  const int path = resolve_path(d.p);
  if (workspace_bytes_given < workspace_bytes(d.p, path)) return FGW_ERR_WORKSPACE_TOO_SMALL;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return FGW_ERR_NO_DEVICE;
  d.device = device;
  st = device_sm_count_cached(device, &d.sm_count);
  if (st != FGW_OK) return st;
  if (encode_tiled() == nullptr) return FGW_ERR_CUDA;
  carve_workspace(d, workspace, path);
  const int budget_ms = d.p.wait_budget_ms > 0 ? d.p.wait_budget_ms : 2000;
  d.budget_ns = static_cast<uint64_t>(budget_ms) * 1000000ull;
  d.stream = static_cast<cudaStream_t>(stream);
  d.tensor_kernel = resolve_tensor_kernel(d.p);
  if (d.contiguous) {
    const int cap = d.p.grid_cap > 0 ? d.p.grid_cap : d.sm_count;
    d.programs = std::min(std::min(cap, d.sm_count), kStreamMaxPrograms);
    // TAIL: whole items for the full waves, cut only the last partial wave's items
    d.tail_start = d.p.schedule == FGW_SCHEDULE_TAIL ? (d.items / d.programs) * d.programs : 0;
  }
  return FGW_OK;
}

static int launch_main(const LaunchDesc& d, bool partials, bool fused_merge = false) {
  const int path = resolve_path(d.p);
  cudaError_t err =
      path == FGW_PATH_TENSOR ? launch_tensor(d, partials) : launch_decode(d, partials, partials && fused_merge);
  if (err == cudaErrorNotSupported) return FGW_ERR_UNSUPPORTED;
  return err == cudaSuccess ? FGW_OK : FGW_ERR_CUDA;
}

}  // namespace fgw

using namespace fgw;

extern "C" {

int fgw_mha_abi_version(void) { return FGW_MHA_ABI_VERSION; }

const char* fgw_mha_status_string(int status) {
  switch (status) {
    case FGW_OK:
      return "ok";
    case FGW_ERR_INVALID_ARGUMENT:
      return "invalid argument";
    case FGW_ERR_UNSUPPORTED:
      return "unsupported configuration";
    case FGW_ERR_WORKSPACE_TOO_SMALL:
      return "workspace too small";
    case FGW_ERR_CUDA:
      return "CUDA error";
    case FGW_ERR_DEVICE_TIMEOUT:
      return "device-side wait timed out";
    case FGW_ERR_NO_DEVICE:
      return "no sm_100 device";
    default:
      return "unknown status";
  }
}

int fgw_mha_device_sm_count(int device, int* sm_count) {
  if (sm_count == nullptr) return FGW_ERR_INVALID_ARGUMENT;
  return device_sm_count_cached(device, sm_count);
}

int fgw_mha_resolve_path(const fgw_mha_params* params, int* path) {
  if (params == nullptr || path == nullptr) return FGW_ERR_INVALID_ARGUMENT;
  *path = resolve_path(*params);
  return FGW_OK;
}

int fgw_mha_resolve_schedule(const fgw_mha_params* params, int* schedule) {
  if (params == nullptr || schedule == nullptr) return FGW_ERR_INVALID_ARGUMENT;
  if (!use_stream_schedule(*params)) {
    *schedule = FGW_SCHEDULE_STRIDED;
  } else {
    *schedule = params->schedule == FGW_SCHEDULE_TAIL ? FGW_SCHEDULE_TAIL : FGW_SCHEDULE_CONTIGUOUS;
  }
  return FGW_OK;
}

int fgw_mha_workspace_size(const fgw_mha_params* params, size_t* bytes) {
  if (params == nullptr || bytes == nullptr) return FGW_ERR_INVALID_ARGUMENT;
  fgw_mha_params p = *params;
  if (p.batch <= 0 || p.q_len <= 0 || p.heads <= 0 || p.head_dim <= 0 || p.num_splits < 1) {
    return FGW_ERR_INVALID_ARGUMENT;
  }
  *bytes = workspace_bytes(p, resolve_path(p));
  return FGW_OK;
}

int fgw_mha_paged_fwd(const fgw_mha_params* params, void* workspace, size_t workspace_bytes_given, void* stream) {
  LaunchDesc d;
  int st = prepare(params, workspace, workspace_bytes_given, stream, d);
  if (st != FGW_OK) return st;
  if (launch_plan(d) != cudaSuccess) return FGW_ERR_CUDA;
  const bool split = d.p.num_splits > 1;
  // split-KV on the decode path merges in place (the CTA completing a row group's splits), no merge launch
  const bool fused = d.merge_counters != nullptr;
  st = launch_main(d, split, fused);
  if (st != FGW_OK) return st;
  if (split && !fused && launch_merge(d) != cudaSuccess) return FGW_ERR_CUDA;
  return FGW_OK;
}

int fgw_mha_plan(const fgw_mha_params* params, void* workspace, size_t workspace_bytes_given, void* stream) {
  LaunchDesc d;
  int st = prepare(params, workspace, workspace_bytes_given, stream, d);
  if (st != FGW_OK) return st;
  return launch_plan(d) == cudaSuccess ? FGW_OK : FGW_ERR_CUDA;
}

int fgw_mha_attend(const fgw_mha_params* params, void* workspace, size_t workspace_bytes_given, void* stream) {
  LaunchDesc d;
  int st = prepare(params, workspace, workspace_bytes_given, stream, d);
  if (st != FGW_OK) return st;
  return launch_main(d, d.p.num_splits > 1);
}

int fgw_mha_partial(const fgw_mha_params* params, void* workspace, size_t workspace_bytes_given, void* stream) {
  LaunchDesc d;
  int st = prepare(params, workspace, workspace_bytes_given, stream, d);
  if (st != FGW_OK) return st;
  if (d.p.num_splits < 2) return FGW_ERR_INVALID_ARGUMENT;
  if (launch_plan(d) != cudaSuccess) return FGW_ERR_CUDA;
  return launch_main(d, true);
}

int fgw_mha_merge(const fgw_mha_params* params, void* workspace, size_t workspace_bytes_given, void* stream) {
  LaunchDesc d;
  int st = prepare(params, workspace, workspace_bytes_given, stream, d);
  if (st != FGW_OK) return st;
  return launch_merge(d) == cudaSuccess ? FGW_OK : FGW_ERR_CUDA;
}

int fgw_mha_selftest_wait(void* workspace, size_t workspace_bytes, int budget_ms, int complete, void* stream) {
  if (workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 255u) ||
      workspace_bytes < sizeof(WorkspaceHeader) || budget_ms <= 0) {
    return FGW_ERR_INVALID_ARGUMENT;
  }
  int device = 0, sms = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return FGW_ERR_NO_DEVICE;
  const int st = device_sm_count_cached(device, &sms);
  if (st != FGW_OK) return st;
  const cudaError_t err = launch_wait_selftest(static_cast<WorkspaceHeader*>(workspace),
                                               static_cast<uint64_t>(budget_ms) * 1000000ull, complete,
                                               static_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? FGW_OK : FGW_ERR_CUDA;
}

int fgw_paged_cache_gather(const fgw_gather_params* params, void* stream) {
  if (params == nullptr) return FGW_ERR_INVALID_ARGUMENT;
  int st = gather_validate(*params);
  if (st != FGW_OK || params->total_rows == 0) return st;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return FGW_ERR_NO_DEVICE;
  int sms = 0;
  st = device_sm_count_cached(device, &sms);
  if (st != FGW_OK) return st;
  return launch_gather(*params, sms, static_cast<cudaStream_t>(stream)) == cudaSuccess ? FGW_OK : FGW_ERR_CUDA;
}

int fgw_mha_read_error(const void* workspace, void* stream, int* device_status, int* site) {
  if (workspace == nullptr || device_status == nullptr) return FGW_ERR_INVALID_ARGUMENT;
  if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess) return FGW_ERR_CUDA;
  int32_t words[2] = {0, 0};
  if (cudaMemcpy(words, workspace, sizeof(words), cudaMemcpyDeviceToHost) != cudaSuccess) return FGW_ERR_CUDA;
  *device_status = words[0];
  if (site != nullptr) *site = words[1];
  return FGW_OK;
}

}  // extern "C"
