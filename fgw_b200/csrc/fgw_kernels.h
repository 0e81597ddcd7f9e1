// Internal launch interface between the C ABI (fgw_api.cu) and the kernel translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "fgw_mha.h"

namespace fgw {

struct WorkspaceHeader;

// Contiguous schedule (fgw_schedule CONTIGUOUS): at most this many programs (persistent CTAs), and at
// most this many work items to lay end to end (the plan launch scans them in one CTA).
constexpr int kStreamMaxPrograms = 148;
constexpr int kStreamMaxItems = 65536;
// rows of one work item of the two-tile kernel (two 128-row query tiles)
constexpr int kPairRows = 256;

// Resolved launch description shared by every kernel family.
struct LaunchDesc {
  fgw_mha_params p;
  int device;         // the current CUDA device of the call
  // workspace carve-up (device pointers)
  WorkspaceHeader* header;
  int32_t* lens;      // [batch] cache lengths clamped into [0, table_width * page_size]
  int32_t* order;     // [batch] batch rows by descending cache length
  float* part_o;      // [batch*q_len*heads, splits, head_dim] FP32 normalised partial outputs
  float* part_lse;    // [batch*q_len*heads, splits] base-2 LSE per partial
  // contiguous schedule (contiguous == true): per-program start item / offset (in KV tiles) / first unit,
  // prog_u[programs] = total units; per-item arrival counters; two partial slots per program
  bool contiguous;
  int programs;
  int items;
  int tail_start;      // first item of the cut range: 0 (CONTIGUOUS) or the items of the full waves (TAIL)
  int32_t* prog_item;  // [programs]
  int32_t* prog_off;   // [programs]
  long long* prog_u;   // [programs + 1]
  long long* prefix;   // [items + 1] plan scratch: first unit of every item
  int32_t* counters;   // [items]
  int slot_rows;       // query rows per slot (stream_slot_rows)
  float* slot_lse;     // [2 * programs, slot_rows] base-2 LSE of each piece row
  float* slot_o;       // [2 * programs, slot_rows, head_dim] FP32 normalised piece outputs
  // split-KV on the decode path: one arrival counter per (request, row block, head) group, so the CTA that
  // completes a group's split set merges it in the same launch (zeroed by plan_kernel)
  int32_t* merge_counters;  // [batch * q_len * heads] (an upper bound on the groups)
  int merge_groups;         // 0 when there is nothing to zero
  uint64_t budget_ns;
  int sm_count;
  int tensor_kernel;  // fgw_tensor_kernel the tensor path runs (resolve_tensor_kernel)
  cudaStream_t stream;
};

// Work items of the two-tile tensor kernel: batch x heads x splits x ceil(q_len / 256).
long long pair_items(const fgw_mha_params& p);
// Query rows of one decode work item, and tokens of one decode pipeline stage (fgw_decode.cu).
int decode_rows_per_item(int head_dim);

// Once per kernel, device and shared-memory size instead of on every call: opts the kernel into
// `smem_bytes` of dynamic shared memory (an attribute of the function in the device's context) and reports the
// registers per thread the build gave it (`regs` may be null).
cudaError_t prepare_kernel(const void* kernel, int smem_bytes, int device, int* regs);

// Launch of a kernel that follows the plan kernel on the stream, as a programmatic dependent launch (it may start
// while the plan finishes; it calls grid_dependency_wait() before reading the plan's results).
template <typename... KernelArgs, typename... Args>
cudaError_t launch_after_plan(void (*kernel)(KernelArgs...), unsigned grid, unsigned block, size_t smem,
                              cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
int decode_tile_tokens(int head_dim);
// Work items the contiguous schedule lays end to end: the two-tile kernel's on the tensor path, the decode
// kernel's (request, query-row block, head) on the decode path.
long long stream_items(const fgw_mha_params& p);
// Query rows of one partial slot of the contiguous schedule: one two-tile item, or one decode item.
int stream_slot_rows(const fgw_mha_params& p);
// Whether the main launch runs the contiguous schedule (fused piece merge): the two-tile tensor kernel, or
// the decode kernel, with one split.
bool use_stream_schedule(const fgw_mha_params& p);

// Workspace layout: header | lens | order | part_lse | part_o | (contiguous schedule: prog_item | prog_off |
// prog_u | prefix | counters | slot_lse | slot_o) | (split decode: merge_counters), each 256-byte aligned.
size_t workspace_bytes(const fgw_mha_params& p, int path);
void carve_workspace(LaunchDesc& d, void* workspace, int path);

// Kernel launchers (return a cudaError_t from the launch).
// Paged-cache gather (fgw_gather.cu): argument check (an fgw_status) and launch.
int gather_validate(const fgw_gather_params& p);
cudaError_t launch_gather(const fgw_gather_params& p, int sm_count, cudaStream_t stream);
cudaError_t launch_plan(const LaunchDesc& d);
// fused_merge (with write_partials): the CTA completing a group's split set merges it into the output.
cudaError_t launch_decode(const LaunchDesc& d, bool write_partials, bool fused_merge);
cudaError_t launch_merge(const LaunchDesc& d);
cudaError_t launch_wait_selftest(WorkspaceHeader* ws, uint64_t budget_ns, int complete, cudaStream_t stream);
cudaError_t launch_tensor(const LaunchDesc& d, bool write_partials);
// Two-query-tile tensor kernel (head_dim <= 128); called by launch_tensor with its tensor maps.
cudaError_t launch_tensor_pairs(const LaunchDesc& d, bool write_partials, const CUtensorMap& qmap,
                                const CUtensorMap& kmap, const CUtensorMap& vmap, int box_rows);
// Key-halves tensor kernel (head_dim <= 128, opt-in); called by launch_tensor with its tensor maps.
cudaError_t launch_tensor_halves(const LaunchDesc& d, bool write_partials, const CUtensorMap& kmap,
                                 const CUtensorMap& vmap, int box_rows);

// Which path AUTO picks, and which tcgen05 kernel the tensor path runs.
int resolve_path(const fgw_mha_params& p);
int resolve_tensor_kernel(const fgw_mha_params& p);

// Tensor-map encoder from the driver (resolved once through the runtime).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled();
// cuTensorMapEncodeTiled through a small cache of recent descriptors: a serving loop encodes the same K/V pool
// maps every call, and a descriptor depends only on these arguments (no device state), so a hit skips the
// driver call.
CUresult encode_tiled_cached(CUtensorMap* map, CUtensorMapDataType dtype, cuuint32_t rank, void* base,
                             const cuuint64_t* dims, const cuuint64_t* strides, const cuuint32_t* box,
                             const cuuint32_t* elem_strides, CUtensorMapInterleave interleave,
                             CUtensorMapSwizzle swizzle, CUtensorMapL2promotion l2, CUtensorMapFloatOOBfill fill);

}  // namespace fgw
