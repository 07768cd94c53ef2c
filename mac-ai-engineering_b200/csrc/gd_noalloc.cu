// gd_forward_noalloc: the forward of gd_forward for callers that cannot allocate device memory themselves.
//
// Who needs it: a host program that embeds this library but hands all device memory to another allocator (a serving
// engine's pre-reserved pool, a framework that owns the whole GPU), so a cudaMalloc of its own would fail or take memory
// the pool counts on; and latency-bound callers that may not call cudaMalloc / cudaFree at all, because those calls
// can synchronise the device. Such a caller cannot provide the workspace gd_forward needs.
//
// What it does instead: the workspace lives in one fixed device array of kScratchBytes (64 MiB), declared below. Host
// code cannot pass the array's name to a kernel (in host code that name is a host-side stand-in, not a device
// address), so the first call on each device, with that device current, asks the runtime for the array's device address
// with cudaGetSymbolAddress and keeps it; that first call should therefore come before any stream capture. Every later
// call on the device reuses the address as long as the device's CUDA context is the one it was looked up in: after a
// cudaDeviceReset (or any other end of the primary context) the module is loaded again and the array may sit elsewhere,
// so a call that finds a new context looks the address up again (that call, too, should come before any capture).
// The array is shared by every call on the device and keeps the last call's contents: the only part that must start at
// zero, the error word, is cleared by each call on its own stream; calls whose work overlaps on the GPU (two streams, or
// two threads) race on the array and must be serialised by the caller. The array stays allocated until the process
// exits on every GPU whose copy of this code has been loaded. The stored-states training forward (GD_STORE_STATES) is
// refused: its workspace must survive until the backward, which a shared array cannot promise.
#include <cuda_runtime.h>

#include <mutex>

#include "gated_delta_b200.h"
#include "gd_common.cuh"
#include "gd_layout.cuh"

namespace {

// the fixed workspace: about 510 chunks of 64 tokens x one value head (e.g. 16 value heads x 1,984 tokens)
constexpr size_t kScratchBytes = size_t(64) << 20;

static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

std::mutex g_setup_mutex;
unsigned char* g_scratch_addr[gd::kMaxDevices] = {};  // the array's device address, per device
CUcontext g_scratch_ctx[gd::kMaxDevices] = {};        // the context that address belongs to

// cuCtxGetCurrent from the driver (the library links only the runtime)
using CtxGetCurrent = CUresult (*)(CUcontext*);
CtxGetCurrent ctx_get_current() {
  static CtxGetCurrent fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult res{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &res) != cudaSuccess ||
        res != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<CtxGetCurrent>(p);
  }();
  return fn;
}

int scratch_address(unsigned char** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return GD_ERR_DEVICE;
  if (dev < 0 || dev >= gd::kMaxDevices) return GD_ERR_DEVICE;
  // before the first runtime call that needs it the primary context may not exist yet (ctx null): then the address
  // is looked up (which creates the context) and the context read again
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  CtxGetCurrent get = ctx_get_current();
  CUcontext ctx = nullptr;
  if (get == nullptr || get(&ctx) != CUDA_SUCCESS) return GD_ERR_DEVICE;
  if (g_scratch_addr[dev] == nullptr || ctx == nullptr || ctx != g_scratch_ctx[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_scratch) != cudaSuccess || p == nullptr) return GD_ERR_DEVICE;
    if (get(&ctx) != CUDA_SUCCESS || ctx == nullptr) return GD_ERR_DEVICE;
    g_scratch_addr[dev] = static_cast<unsigned char*>(p);
    g_scratch_ctx[dev] = ctx;
  }
  *out = g_scratch_addr[dev];
  return GD_OK;
}

}  // namespace

extern "C" int gd_forward_noalloc(const void* q, const void* k, const void* v, const float* g, const float* beta,
                                  const float* s0, void* o, float* sT, int dtype, int B, int T, int H, int HK, int DK,
                                  int DV, int flags, void* stream, int* device_status) {
  // the stored-states forward keeps its workspace for the backward: not with a shared array
  if (flags & GD_STORE_STATES) return GD_ERR_ARG;
  // sizes first: a request beyond the fixed array is refused before any device call
  const size_t need = gd_workspace_bytes(B, T, H, HK, DK, DV, 0);
  if (need == 0) return GD_ERR_SHAPE;
  if (need > kScratchBytes) return GD_ERR_SCRATCH;
  unsigned char* ws = nullptr;
  int s = scratch_address(&ws);
  if (s) return s;
  // exactly the forward layout's size, so that gd_prep lays the array out for the forward alone
  s = gd_forward(q, k, v, g, beta, s0, o, sT, dtype, B, T, H, HK, DK, DV, flags, ws, need, stream);
  if (s) return s;
  if (device_status != nullptr) *device_status = gd_read_error(ws, stream, nullptr);
  return GD_OK;
}
