// The C ABI (include/gated_delta_b200.h): argument checks, dispatch on dtype and head widths, kernel sequencing.
// No entry point allocates, synchronises (except gd_read_error) or aborts.
#include <atomic>
#include <cstdint>
#include <cuda_runtime.h>

#include "gd_common.cuh"
#include "gd_layout.cuh"

namespace gd {
template <typename T, int DK, int DV>
cudaError_t launch_prep(const void*, const void*, const void*, const float*, const float*, const Layout&, int,
                        unsigned char*, cudaStream_t);
template <typename T, int DK, int DV>
cudaError_t launch_state(const float*, void*, float*, const Layout&, int, unsigned char*, cudaStream_t);
template <typename T, int DK, int DV>
cudaError_t launch_bwd_state(const void*, const float*, float*, const Layout&, int, unsigned char*, cudaStream_t);
template <typename T, int DK, int DV>
cudaError_t launch_bwd_chunk(const void*, const void*, const void*, const float*, const void*, void*, void*, void*,
                             float*, float*, const Layout&, int, unsigned char*, cudaStream_t);
cudaError_t launch_chunk_table(const int*, const Layout&, unsigned char*, cudaStream_t);
cudaError_t launch_scatter(const void*, void*, int, const Layout&, const unsigned char*, cudaStream_t);
}  // namespace gd

namespace {

using gd::Layout;

bool aligned16(const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_dims(int B, int T, int H, int HK, int DK, int DV, int dtype) {
  if (B <= 0 || T <= 0 || H <= 0 || HK <= 0) return GD_ERR_SHAPE;
  if (H % HK != 0) return GD_ERR_SHAPE;
  if (DK != 128 || DV != 128) return GD_ERR_SHAPE;
  if (dtype != GD_FLOAT32 && dtype != GD_FLOAT16 && dtype != GD_BFLOAT16) return GD_ERR_ARG;
  if ((long long)B * H * ((T + 63) / 64) > (1ll << 31) - 1) return GD_ERR_SHAPE;
  if (H > 65535 || B > 65535) return GD_ERR_SHAPE;
  return GD_OK;
}

// The current device must be sm_100 (the kernels are built for sm_100a only). The answer is kept per device index
// (-1 = not yet asked), so a process that drives several GPUs gets each device's own answer; concurrent first calls
// on one device store the same value.
std::atomic<int> g_device_ok[gd::kMaxDevices];  // zero-initialised: 0 = not asked, 1 = sm_100, 2 = other

int check_device() {
  int dev = 0, major = 0, minor = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return GD_ERR_DEVICE;
  const bool cacheable = dev >= 0 && dev < gd::kMaxDevices;
  if (cacheable) {
    const int known = g_device_ok[dev].load(std::memory_order_relaxed);
    if (known != 0) return known == 1 ? GD_OK : GD_ERR_DEVICE;
  }
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return GD_ERR_DEVICE;
  if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) return GD_ERR_DEVICE;
  const bool ok = major == 10 && minor == 0;
  if (cacheable) g_device_ok[dev].store(ok ? 1 : 2, std::memory_order_relaxed);
  return ok ? GD_OK : GD_ERR_DEVICE;
}

int launched(cudaError_t e) { return e == cudaSuccess ? GD_OK : GD_ERR_LAUNCH; }

// packed rows: N sequences, T rows in all (one batch row); the state passes' grid rows are the sequences
int check_packed(int N, int T, int H, int HK, int DK, int DV, int dtype) {
  if (N <= 0 || N > 65535) return GD_ERR_SHAPE;
  int s = check_dims(1, T, H, HK, DK, DV, dtype);
  if (s) return s;
  if ((long long)H * (T / 64 + N) > (1ll << 31) - 1) return GD_ERR_SHAPE;
  return GD_OK;
}

int elem_bytes(int dtype) { return dtype == GD_FLOAT32 ? 4 : 2; }

int prep(const void* q, const void* k, const void* v, const float* g, const float* beta, int dtype, const Layout& L,
         int flags, void* ws, cudaStream_t st) {
  auto w = static_cast<unsigned char*>(ws);
  switch (dtype) {
    case GD_BFLOAT16: return launched(gd::launch_prep<__nv_bfloat16, 128, 128>(q, k, v, g, beta, L, flags, w, st));
    case GD_FLOAT16: return launched(gd::launch_prep<__half, 128, 128>(q, k, v, g, beta, L, flags, w, st));
    default: return launched(gd::launch_prep<float, 128, 128>(q, k, v, g, beta, L, flags, w, st));
  }
}

int fwd_state(const float* s0, void* o, float* sT, int dtype, const Layout& L, int flags, void* ws, cudaStream_t st) {
  auto w = static_cast<unsigned char*>(ws);
  switch (dtype) {
    case GD_BFLOAT16: return launched(gd::launch_state<__nv_bfloat16, 128, 128>(s0, o, sT, L, flags, w, st));
    case GD_FLOAT16: return launched(gd::launch_state<__half, 128, 128>(s0, o, sT, L, flags, w, st));
    default: return launched(gd::launch_state<float, 128, 128>(s0, o, sT, L, flags, w, st));
  }
}

int bwd_state(const void* d_o, const float* dsT, float* ds0, int dtype, const Layout& L, int flags, void* ws,
              cudaStream_t st) {
  auto w = static_cast<unsigned char*>(ws);
  switch (dtype) {
    case GD_BFLOAT16: return launched(gd::launch_bwd_state<__nv_bfloat16, 128, 128>(d_o, dsT, ds0, L, flags, w, st));
    case GD_FLOAT16: return launched(gd::launch_bwd_state<__half, 128, 128>(d_o, dsT, ds0, L, flags, w, st));
    default: return launched(gd::launch_bwd_state<float, 128, 128>(d_o, dsT, ds0, L, flags, w, st));
  }
}

int bwd_chunk(const void* q, const void* k, const void* v, const float* beta, const void* d_o, void* dq, void* dk,
              void* dv, float* dg, float* dbeta, int dtype, const Layout& L, int flags, void* ws, cudaStream_t st) {
  auto w = static_cast<unsigned char*>(ws);
  switch (dtype) {
    case GD_BFLOAT16:
      return launched(gd::launch_bwd_chunk<__nv_bfloat16, 128, 128>(q, k, v, beta, d_o, dq, dk, dv, dg, dbeta, L,
                                                                     flags, w, st));
    case GD_FLOAT16:
      return launched(
          gd::launch_bwd_chunk<__half, 128, 128>(q, k, v, beta, d_o, dq, dk, dv, dg, dbeta, L, flags, w, st));
    default:
      return launched(
          gd::launch_bwd_chunk<float, 128, 128>(q, k, v, beta, d_o, dq, dk, dv, dg, dbeta, L, flags, w, st));
  }
}

}  // namespace

extern "C" {

const char* gd_status_string(int status) {
  switch (status) {
    case GD_OK: return "ok";
    case GD_ERR_ARG: return "invalid argument (null pointer, dtype or flag)";
    case GD_ERR_SHAPE: return "unsupported sizes (head widths must be 128; value heads a multiple of key heads)";
    case GD_ERR_ALIGN: return "a pointer is not 16-byte aligned";
    case GD_ERR_WORKSPACE: return "workspace smaller than gd_workspace_bytes()";
    case GD_ERR_LAUNCH: return "CUDA kernel launch failed";
    case GD_ERR_TIMEOUT: return "a device-side wait gave up (kernel stage recorded in the error word)";
    case GD_ERR_DEVICE: return "the current CUDA device is not sm_100 (B200)";
    case GD_ERR_SCRATCH: return "sizes need more than gd_forward_noalloc's fixed 64 MiB scratch array";
    default: return "unknown status";
  }
}

size_t gd_workspace_bytes(int B, int T, int H, int HK, int DK, int DV, int for_backward) {
  if (check_dims(B, T, H, HK, DK, DV, GD_BFLOAT16) != GD_OK) return 0;
  return Layout::make(B, T, H, HK, DK, DV, for_backward != 0).total;
}

int gd_prep(const void* q, const void* k, const void* v, const float* g, const float* beta, int dtype, int B, int T,
            int H, int HK, int DK, int DV, int flags, void* workspace, size_t workspace_bytes, void* stream) {
  int s = check_dims(B, T, H, HK, DK, DV, dtype);
  if (s) return s;
  if (!q || !k || !v || !g || !beta || !workspace) return GD_ERR_ARG;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(workspace)) return GD_ERR_ALIGN;
  if ((s = check_device())) return s;
  // the layout kind (forward-only or backward) follows the workspace size the caller provides
  Layout L = Layout::make(B, T, H, HK, DK, DV, true);
  if (workspace_bytes < L.total) L = Layout::make(B, T, H, HK, DK, DV, false);
  if (workspace_bytes < L.total) return GD_ERR_WORKSPACE;
  // every call sequence starts here: clear the error word (stream-ordered, no allocation)
  if (cudaMemsetAsync(workspace, 0, sizeof(gd::ErrorWord), static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return GD_ERR_LAUNCH;
  return prep(q, k, v, g, beta, dtype, L, flags, workspace, static_cast<cudaStream_t>(stream));
}

int gd_fwd_state(const float* s0, void* o, float* sT, int dtype, int B, int T, int H, int HK, int DK, int DV,
                 int flags, void* workspace, size_t workspace_bytes, void* stream) {
  int s = check_dims(B, T, H, HK, DK, DV, dtype);
  if (s) return s;
  if (!workspace) return GD_ERR_ARG;
  if (!aligned16(workspace)) return GD_ERR_ALIGN;
  if ((s = check_device())) return s;
  Layout L = Layout::make(B, T, H, HK, DK, DV, true);
  if (workspace_bytes < L.total) {
    if (flags & GD_STORE_STATES) return GD_ERR_WORKSPACE;
    L = Layout::make(B, T, H, HK, DK, DV, false);
  }
  if (workspace_bytes < L.total) return GD_ERR_WORKSPACE;
  return fwd_state(s0, o, sT, dtype, L, flags, workspace, static_cast<cudaStream_t>(stream));
}

int gd_bwd_state(const void* d_o, const float* dsT, float* ds0, int dtype, int B, int T, int H, int HK, int DK, int DV,
                 int flags, void* workspace, size_t workspace_bytes, void* stream) {
  int s = check_dims(B, T, H, HK, DK, DV, dtype);
  if (s) return s;
  if (!workspace) return GD_ERR_ARG;
  if (!aligned16(workspace) || !aligned16(d_o)) return GD_ERR_ALIGN;
  if ((s = check_device())) return s;
  Layout L = Layout::make(B, T, H, HK, DK, DV, true);
  if (workspace_bytes < L.total) return GD_ERR_WORKSPACE;
  return bwd_state(d_o, dsT, ds0, dtype, L, flags, workspace, static_cast<cudaStream_t>(stream));
}

int gd_bwd_chunk(const void* q, const void* k, const void* v, const float* beta, const void* d_o, void* dq, void* dk,
                 void* dv, float* dg, float* dbeta, int dtype, int B, int T, int H, int HK, int DK, int DV, int flags,
                 void* workspace, size_t workspace_bytes, void* stream) {
  int s = check_dims(B, T, H, HK, DK, DV, dtype);
  if (s) return s;
  if (!q || !k || !v || !beta || !dq || !dk || !dv || !dg || !dbeta || !workspace) return GD_ERR_ARG;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(d_o) || !aligned16(dq) || !aligned16(dk) ||
      !aligned16(dv) || !aligned16(workspace))
    return GD_ERR_ALIGN;
  if ((s = check_device())) return s;
  Layout L = Layout::make(B, T, H, HK, DK, DV, true);
  if (workspace_bytes < L.total) return GD_ERR_WORKSPACE;
  return bwd_chunk(q, k, v, beta, d_o, dq, dk, dv, dg, dbeta, dtype, L, flags, workspace,
                   static_cast<cudaStream_t>(stream));
}

int gd_forward(const void* q, const void* k, const void* v, const float* g, const float* beta, const float* s0,
               void* o, float* sT, int dtype, int B, int T, int H, int HK, int DK, int DV, int flags, void* workspace,
               size_t workspace_bytes, void* stream) {
  int s = check_dims(B, T, H, HK, DK, DV, dtype);
  if (s) return s;
  // GD_STORE_STATES: the backward layout, every image the backward reads written here (the stored-states training
  // forward); otherwise the forward-only layout in any workspace at least that large (prep skips the extra images)
  const bool keep = (flags & GD_STORE_STATES) != 0;
  const size_t bytes = Layout::make(B, T, H, HK, DK, DV, keep).total;
  if (workspace_bytes < bytes) return GD_ERR_WORKSPACE;
  if (!o) return GD_ERR_ARG;
  if (!aligned16(o)) return GD_ERR_ALIGN;
  const int f = flags & (GD_L2NORM | GD_SCALE_Q | GD_KEY_WIDTH_MASK);
  s = gd_prep(q, k, v, g, beta, dtype, B, T, H, HK, DK, DV, f, workspace, bytes, stream);
  if (s) return s;
  return gd_fwd_state(s0, o, sT, dtype, B, T, H, HK, DK, DV,
                      f | (keep ? GD_STORE_STATES : 0) | (flags & GD_WIDE_STATE_PASS), workspace, bytes, stream);
}

int gd_backward(const void* q, const void* k, const void* v, const float* g, const float* beta, const float* s0,
                const void* d_o, const float* dsT, void* dq, void* dk, void* dv, float* dg, float* dbeta, float* ds0,
                int dtype, int B, int T, int H, int HK, int DK, int DV, int flags, void* workspace,
                size_t workspace_bytes, void* stream) {
  int s = check_dims(B, T, H, HK, DK, DV, dtype);
  if (s) return s;
  if (!workspace) return GD_ERR_ARG;
  if (!aligned16(workspace)) return GD_ERR_ALIGN;
  if (workspace_bytes < Layout::make(B, T, H, HK, DK, DV, true).total) return GD_ERR_WORKSPACE;
  const int f = flags & (GD_L2NORM | GD_SCALE_Q | GD_KEY_WIDTH_MASK);
  if (flags & GD_STATES_STORED) {
    // the workspace holds what gd_forward(GD_STORE_STATES) wrote for these inputs: no recompute; the error word is
    // cleared here as gd_prep would
    if ((s = check_device())) return s;
    if (cudaMemsetAsync(workspace, 0, sizeof(gd::ErrorWord), static_cast<cudaStream_t>(stream)) != cudaSuccess)
      return GD_ERR_LAUNCH;
  } else {
    if ((s = gd_prep(q, k, v, g, beta, dtype, B, T, H, HK, DK, DV, f, workspace, workspace_bytes, stream))) return s;
    if ((s = gd_fwd_state(s0, nullptr, nullptr, dtype, B, T, H, HK, DK, DV, f | GD_STORE_STATES, workspace,
                          workspace_bytes, stream)))
      return s;
  }
  if ((s = gd_bwd_state(d_o, dsT, ds0, dtype, B, T, H, HK, DK, DV, f, workspace, workspace_bytes, stream))) return s;
  return gd_bwd_chunk(q, k, v, beta, d_o, dq, dk, dv, dg, dbeta, dtype, B, T, H, HK, DK, DV, f, workspace,
                      workspace_bytes, stream);
}

size_t gd_workspace_bytes_packed(int N, int T, int H, int HK, int DK, int DV, int for_backward) {
  if (check_packed(N, T, H, HK, DK, DV, GD_BFLOAT16) != GD_OK) return 0;
  return Layout::make(1, T, H, HK, DK, DV, for_backward != 0, N).total;
}

int gd_forward_packed(const void* q, const void* k, const void* v, const float* g, const float* beta,
                      const float* s0, void* o, float* sT, const int* cu_seqlens, int N, int dtype, int T, int H,
                      int HK, int DK, int DV, int flags, void* workspace, size_t workspace_bytes, void* stream) {
  int s = check_packed(N, T, H, HK, DK, DV, dtype);
  if (s) return s;
  const bool keep = (flags & GD_STORE_STATES) != 0;
  const Layout L = Layout::make(1, T, H, HK, DK, DV, keep, N);
  if (!q || !k || !v || !g || !beta || !o || !cu_seqlens || !workspace) return GD_ERR_ARG;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o) || !aligned16(workspace)) return GD_ERR_ALIGN;
  if (workspace_bytes < L.total) return GD_ERR_WORKSPACE;
  if ((s = check_device())) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto ws = static_cast<unsigned char*>(workspace);
  if (cudaMemsetAsync(workspace, 0, sizeof(gd::ErrorWord), st) != cudaSuccess) return GD_ERR_LAUNCH;
  if ((s = launched(gd::launch_chunk_table(cu_seqlens, L, ws, st)))) return s;
  const int f = flags & (GD_L2NORM | GD_SCALE_Q | GD_KEY_WIDTH_MASK);
  if ((s = prep(q, k, v, g, beta, dtype, L, f, workspace, st))) return s;
  const int fs = f | (keep ? GD_STORE_STATES : 0) | (flags & GD_WIDE_STATE_PASS);
  if ((s = fwd_state(s0, ws + L.opad, sT, dtype, L, fs, workspace, st))) return s;
  return launched(gd::launch_scatter(ws + L.opad, o, H * DV * elem_bytes(dtype), L, ws, st));
}

int gd_backward_packed(const void* q, const void* k, const void* v, const float* g, const float* beta,
                       const float* s0, const void* d_o, const float* dsT, void* dq, void* dk, void* dv, float* dg,
                       float* dbeta, float* ds0, const int* cu_seqlens, int N, int dtype, int T, int H, int HK, int DK,
                       int DV, int flags, void* workspace, size_t workspace_bytes, void* stream) {
  int s = check_packed(N, T, H, HK, DK, DV, dtype);
  if (s) return s;
  const Layout L = Layout::make(1, T, H, HK, DK, DV, true, N);
  if (!q || !k || !v || !beta || !dq || !dk || !dv || !dg || !dbeta || !cu_seqlens || !workspace) return GD_ERR_ARG;
  if (!(flags & GD_STATES_STORED) && !g) return GD_ERR_ARG;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(d_o) || !aligned16(dq) || !aligned16(dk) ||
      !aligned16(dv) || !aligned16(workspace))
    return GD_ERR_ALIGN;
  if (workspace_bytes < L.total) return GD_ERR_WORKSPACE;
  if ((s = check_device())) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto ws = static_cast<unsigned char*>(workspace);
  if (cudaMemsetAsync(workspace, 0, sizeof(gd::ErrorWord), st) != cudaSuccess) return GD_ERR_LAUNCH;
  if ((s = launched(gd::launch_chunk_table(cu_seqlens, L, ws, st)))) return s;
  const int f = flags & (GD_L2NORM | GD_SCALE_Q | GD_KEY_WIDTH_MASK);
  if (!(flags & GD_STATES_STORED)) {  // recompute the chunk states from the inputs
    if ((s = prep(q, k, v, g, beta, dtype, L, f, workspace, st))) return s;
    if ((s = fwd_state(s0, nullptr, nullptr, dtype, L, f | GD_STORE_STATES, workspace, st))) return s;
  }
  if ((s = bwd_state(d_o, dsT, ds0, dtype, L, f, workspace, st))) return s;
  if ((s = bwd_chunk(q, k, v, beta, d_o, ws + L.dqpad, ws + L.dkpad, ws + L.dvpad, dg, dbeta, dtype, L, f, workspace,
                     st)))
    return s;
  const int eb = elem_bytes(dtype);
  if ((s = launched(gd::launch_scatter(ws + L.dqpad, dq, HK * DK * eb, L, ws, st)))) return s;
  if ((s = launched(gd::launch_scatter(ws + L.dkpad, dk, HK * DK * eb, L, ws, st)))) return s;
  return launched(gd::launch_scatter(ws + L.dvpad, dv, H * DV * eb, L, ws, st));
}

int gd_read_error(void* workspace, void* stream, int* where) {
  if (!workspace) return GD_ERR_ARG;
  gd::ErrorWord w{};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(&w, workspace, sizeof(w), cudaMemcpyDeviceToHost, st) != cudaSuccess) return GD_ERR_LAUNCH;
  if (cudaStreamSynchronize(st) != cudaSuccess) return GD_ERR_LAUNCH;
  if (w.code != 0) {
    gd::ErrorWord zero{};
    cudaMemcpyAsync(workspace, &zero, sizeof(zero), cudaMemcpyHostToDevice, st);
    cudaStreamSynchronize(st);
  }
  if (where) *where = w.where;
  return w.code;
}

}  // extern "C"
