// Allocation-free variant of fgw_mha_paged_fwd.
//
// Some callers cannot call cudaMalloc at the point where they run attention: code running inside a
// custom allocator or memory-pool callback, real-time serving loops that forbid allocator traffic
// (and the device-wide synchronisation cudaFree implies), and plugins whose host framework owns all
// device memory and hands out only input and output buffers. For them this entry point runs the same
// plan / attention / merge kernels as fgw_mha_paged_fwd, but its scratch (workspace header, clamped
// lengths, request order and split-KV partials) lives in one file-scope __device__ array of
// FGW_MHA_STATIC_WORKSPACE_BYTES that every GPU loading the library holds until the process exits.
//
// The array's name is only a host-side stand-in in host code; its device address is looked up once
// per device with cudaGetSymbolAddress (with that device current) on the first call made on that device,
// and cached for the process (a cudaDeviceReset, which reloads the module, would leave it stale; the
// header says not to call after one). Nothing here allocates.
#include <mutex>

#include "fgw_mha.h"

#include <cuda_runtime.h>

namespace {

static __device__ __align__(256) unsigned char g_static_workspace[FGW_MHA_STATIC_WORKSPACE_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mutex;
void* g_device_ptr[kMaxDevices] = {nullptr};

// Device address of g_static_workspace on the current device (looked up on first use).
int static_workspace_ptr(void** ptr) {
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) return FGW_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_device_ptr[device] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_static_workspace) != cudaSuccess || p == nullptr) return FGW_ERR_CUDA;
    g_device_ptr[device] = p;
  }
  *ptr = g_device_ptr[device];
  return FGW_OK;
}

}  // namespace

// Status of the last fgw_mha_paged_fwd_static_ws call on the current device: the workspace header lives in the
// library's array, so the caller (who never sees its address) reads it here. Copies the header's two words out
// of the array by symbol; allocates nothing.
extern "C" int fgw_mha_static_ws_read_error(void* stream, int* device_status, int* site) {
  if (device_status == nullptr) return FGW_ERR_INVALID_ARGUMENT;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return FGW_ERR_NO_DEVICE;
  if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess) return FGW_ERR_CUDA;
  int32_t words[2] = {0, 0};
  if (cudaMemcpyFromSymbol(words, g_static_workspace, sizeof(words), 0, cudaMemcpyDeviceToHost) != cudaSuccess) {
    return FGW_ERR_CUDA;
  }
  *device_status = words[0];
  if (site != nullptr) *site = words[1];
  return FGW_OK;
}

extern "C" int fgw_mha_paged_fwd_static_ws(const fgw_mha_params* params, void* stream) {
  if (params == nullptr) return FGW_ERR_INVALID_ARGUMENT;
  fgw_mha_params p = *params;
  size_t needed = 0;
  int st = fgw_mha_workspace_size(&p, &needed);
  if (st != FGW_OK) return st;
  if (needed > static_cast<size_t>(FGW_MHA_STATIC_WORKSPACE_BYTES) && p.schedule == FGW_SCHEDULE_AUTO) {
    // The contiguous schedule's partial slots do not fit: the strided schedule needs no slots.
    p.schedule = FGW_SCHEDULE_STRIDED;
    st = fgw_mha_workspace_size(&p, &needed);
    if (st != FGW_OK) return st;
  }
  if (needed > static_cast<size_t>(FGW_MHA_STATIC_WORKSPACE_BYTES)) return FGW_ERR_WORKSPACE_TOO_SMALL;
  void* ws = nullptr;
  st = static_workspace_ptr(&ws);
  if (st != FGW_OK) return st;
  // What must start at zero is zeroed on the device by the plan kernel that starts every forward: the
  // error word and the per-item arrival counters the contiguous and tail schedules' piece merges count
  // on. Every other byte of scratch the kernels read (lengths, order, partials) is written earlier in
  // the same call, so the previous call's leftovers never reach an output.
  return fgw_mha_paged_fwd(&p, ws, FGW_MHA_STATIC_WORKSPACE_BYTES, stream);
}
