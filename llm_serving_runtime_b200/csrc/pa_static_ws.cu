// pa_static_ws.cu — paged decode for callers that cannot allocate device memory.
//
// pa_decode needs a scratch workspace (device error word, merge counters and
// the partial (m, l, acc) slots of rows split between warps).  Some callers
// cannot provide one: a plugin host that hands its kernels only their inputs
// and outputs, a serving loop that has given all free HBM to the KV pool and
// may not allocate afterwards, or code on a path where cudaMalloc's implicit
// device synchronisation is not acceptable.  pa_decode_static_workspace serves
// them from a fixed scratch array that lives inside this library.
//
// The array is a file-scope __device__ variable of PA_STATIC_WORKSPACE_BYTES
// (16 MiB).  The CUDA runtime loads a library's device code lazily by default,
// so the array is created in a device's memory by the first call on that device
// (the address lookup below) and then stays there until the process exits.
// Host code cannot use the array's name as a device address (there it is only a
// host-side stand-in), so that first call looks the device address up with
// cudaGetSymbolAddress, with the device current, and caches it.  Make the first
// call on each device before handing the rest of its free memory to the KV pool,
// and before any stream capture; later calls need no free device memory.  Every
// call shares the one array and it keeps the previous call's contents: each
// call clears the part that must start at zero (error word and merge counters)
// on its stream, and calls whose kernels overlap on the GPU (other streams)
// race on it.  Nothing here allocates: no cudaMalloc, cudaFree or allocating
// library routine is called.
#include <stdio.h>

#include <mutex>

#include "pa_common.cuh"
#include "pa_internal.h"

namespace {

__device__ __align__(256) unsigned char g_static_workspace[PA_STATIC_WORKSPACE_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_static_mu;
void* g_static_addr[kMaxDevices] = {nullptr};

// Device address of g_static_workspace on `dev` (the current device).
int static_workspace_address(int dev, void** out) {
  if (dev < 0 || dev >= kMaxDevices)
    return pa::set_last_error(PA_ERR_INVALID_ARGUMENT, "device index out of range");
  std::lock_guard<std::mutex> lk(g_static_mu);
  if (g_static_addr[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_static_workspace);
    if (e != cudaSuccess || p == nullptr) {
      char msg[256];
      snprintf(msg, sizeof(msg), "cudaGetSymbolAddress(static workspace): %s", cudaGetErrorString(e));
      return pa::set_last_error(PA_ERR_CUDA, msg);
    }
    g_static_addr[dev] = p;
  }
  *out = g_static_addr[dev];
  return PA_OK;
}

}  // namespace

extern "C" PA_API int pa_decode_static_workspace(const pa_decode_args* args, void* stream) {
  if (args == nullptr) return pa::set_last_error(PA_ERR_INVALID_ARGUMENT, "null args");
  if (args->batch == 0) return pa_decode(args, stream);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return pa::set_last_error(PA_ERR_CUDA, "cudaGetDevice failed");
  int num_sms = 0;
  e = cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof(msg), "cudaDeviceGetAttribute(SM count): %s", cudaGetErrorString(e));
    return pa::set_last_error(PA_ERR_CUDA, msg);
  }
  void* ws = nullptr;
  int st = static_workspace_address(dev, &ws);
  if (st != PA_OK) return st;

  if (args->num_q_heads <= 0 || args->num_kv_heads <= 0 || args->q_len <= 0 || args->head_dim <= 0 ||
      args->batch < 0 || args->num_q_heads % args->num_kv_heads != 0)
    return pa_decode(args, stream);  // pa_decode reports the shape error itself
  const size_t need = pa_decode_workspace_bytes(args->batch, args->num_q_heads, args->num_kv_heads,
                                                args->q_len, args->head_dim, args->dtype, dev);
  if (need == 0) {
    // the shape is valid, so the sizing failed on a device query
    char msg[256];
    snprintf(msg, sizeof(msg), "sizing the decode scratch on device %d failed: %s", dev, pa_last_error());
    return pa::set_last_error(PA_ERR_CUDA, msg);
  }
  if (need > PA_STATIC_WORKSPACE_BYTES) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "this shape needs %zu bytes of decode scratch; the static workspace holds %u bytes "
             "(use pa_decode with a caller workspace)",
             need, (unsigned)PA_STATIC_WORKSPACE_BYTES);
    return pa::set_last_error(PA_ERR_WORKSPACE, msg);
  }

  // Error word, slot claims and merge counters must start at zero.
  const size_t zero_bytes = pa::kWsFixedBytes + pa::ws_counter_bytes(num_sms * pa::kDecodeWarps);
  e = cudaMemsetAsync(ws, 0, zero_bytes, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return pa::set_last_error(PA_ERR_CUDA, "cudaMemsetAsync(static workspace) failed");

  pa_decode_args a = *args;
  a.workspace = ws;
  a.workspace_bytes = PA_STATIC_WORKSPACE_BYTES;
  a.allow_overlap_with_previous = 0;  // the memset above now precedes the decode launch
  return pa_decode(&a, stream);
}
