// Packed rows (cu_seqlens): N sequences concatenated along the token axis of one batch row. Each sequence starts a
// new chunk, so every chunk belongs to one sequence and the chunk kernels run unchanged; the state passes walk each
// sequence's chunks with its own initial and final state. Two small kernels serve the entry points:
//   chunk_table_kernel  cu_seqlens [N + 1] -> the workspace's chunk table (each chunk's first row in the caller's
//                       arrays and its sequence's end) and each sequence's first chunk (one CTA, a block scan of the
//                       per-sequence chunk counts; no host synchronisation, so the calls stay graph-capturable)
//   scatter_kernel      the chunk-aligned rows the kernels wrote (o, dq, dk, dv in the workspace) -> the caller's
//                       packed rows (16-byte copies; rows past a sequence's end are not copied)
#include <cuda_runtime.h>

#include <cstdint>

#include "gd_layout.cuh"

namespace gd {
namespace {

constexpr int kScanThreads = 1024;

__device__ __forceinline__ int clampi(int x, int lo, int hi) { return x < lo ? lo : (x > hi ? hi : x); }

// Sequence n covers rows [cu[n], cu[n + 1]) (clamped into [0, Tin] and to a non-negative length, so that any input
// stays in bounds; the caller checks the boundaries themselves); its chunks are numbered from seg[n]. Chunk entries
// past the last sequence's, and any beyond NT, are (0, 0) / not written.
__global__ void __launch_bounds__(kScanThreads) chunk_table_kernel(const int* __restrict__ cu, int N, int Tin, int NT,
                                                                   int2* __restrict__ ctab, int* __restrict__ seg) {
  __shared__ int warp_tot[kScanThreads / 32];
  __shared__ int carry, next_carry;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) carry = 0;
  __syncthreads();
  for (int base = 0; base < N; base += kScanThreads) {
    const int n = base + tid;
    int start = 0, end = 0, cnt = 0;
    if (n < N) {
      start = clampi(cu[n], 0, Tin);
      end = clampi(cu[n + 1], start, Tin);
      cnt = (end - start + 63) / 64;
    }
    // inclusive scan of cnt over the block: within warps, then over the warp totals
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int w = warp_tot[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      warp_tot[lane] = w;  // inclusive over warps 0 .. lane
    }
    __syncthreads();
    if (warp > 0) incl += warp_tot[warp - 1];
    const int first = carry + incl - cnt;
    if (n < N) {
      seg[n] = first < NT ? first : NT;
      for (int j = 0; j < cnt && first + j < NT; ++j) ctab[first + j] = make_int2(start + 64 * j, end);
    }
    if (tid == kScanThreads - 1) next_carry = carry + incl;
    __syncthreads();
    if (tid == 0) carry = next_carry;
    __syncthreads();
  }
  const int used = carry < NT ? carry : NT;
  if (tid == 0) seg[N] = used;
  for (int c = used + tid; c < NT; c += kScanThreads) ctab[c] = make_int2(0, 0);
}

// grid: one CTA per chunk. Row r of chunk c (padded row c * 64 + r) goes to row ctab[c].x + r of the caller's array
// when that is below ctab[c].y. row_bytes: one row's bytes (heads x D x element size, a multiple of 16).
__global__ void __launch_bounds__(256) scatter_kernel(const unsigned char* __restrict__ src, unsigned char* __restrict__ dst,
                                                      const int2* __restrict__ ctab, int row_bytes) {
  const int c = blockIdx.x;
  const int2 e = ctab[c];
  const int rows = e.y - e.x < 64 ? e.y - e.x : 64;
  if (rows <= 0) return;
  const int per_row = row_bytes / 16;
  const uint4* s = reinterpret_cast<const uint4*>(src + (size_t)c * 64 * row_bytes);
  uint4* d = reinterpret_cast<uint4*>(dst + (size_t)e.x * row_bytes);
  const int total = rows * per_row;  // the chunk's valid rows are contiguous on both sides
  for (int i = threadIdx.x; i < total; i += blockDim.x) d[i] = s[i];
}

}  // namespace

cudaError_t launch_chunk_table(const int* cu_seqlens, const Layout& lay, unsigned char* ws, cudaStream_t st) {
  chunk_table_kernel<<<1, kScanThreads, 0, st>>>(cu_seqlens, lay.N, lay.Tin, lay.NT,
                                                 reinterpret_cast<int2*>(ws + lay.ctab),
                                                 reinterpret_cast<int*>(ws + lay.seg));
  return cudaGetLastError();
}

cudaError_t launch_scatter(const void* src, void* dst, int row_bytes, const Layout& lay, const unsigned char* ws,
                           cudaStream_t st) {
  scatter_kernel<<<lay.NT, 256, 0, st>>>(static_cast<const unsigned char*>(src), static_cast<unsigned char*>(dst),
                                         reinterpret_cast<const int2*>(ws + lay.ctab), row_bytes);
  return cudaGetLastError();
}

}  // namespace gd
