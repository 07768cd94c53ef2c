// Backward kernels (reverse state pass, per-chunk gradients). Placeholder launchers until the kernels land.
#include "gd_common.cuh"
#include "gd_layout.cuh"

namespace gd {
template <typename T, int DK, int DV>
cudaError_t launch_bwd_state(const void*, const float*, float*, const Layout&, int, unsigned char*, cudaStream_t) {
  return cudaErrorNotSupported;
}
template <typename T, int DK, int DV>
cudaError_t launch_bwd_chunk(const void*, const void*, const void*, const float*, const void*, void*, void*, void*,
                             float*, float*, const Layout&, int, unsigned char*, cudaStream_t) {
  return cudaErrorNotSupported;
}
#define INST(T)                                                                                                    \
  template cudaError_t launch_bwd_state<T, 128, 128>(const void*, const float*, float*, const Layout&, int,         \
                                                     unsigned char*, cudaStream_t);                                 \
  template cudaError_t launch_bwd_chunk<T, 128, 128>(const void*, const void*, const void*, const float*,           \
                                                     const void*, void*, void*, void*, float*, float*, const Layout&, \
                                                     int, unsigned char*, cudaStream_t);
INST(__nv_bfloat16)
INST(__half)
INST(float)
}  // namespace gd
