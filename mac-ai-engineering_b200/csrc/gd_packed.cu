// Packed rows (cu_seqlens): N sequences concatenated along the token axis of one batch row. Each sequence starts a
// new chunk, so every chunk belongs to one sequence and the chunk kernels run unchanged; the state passes walk each
// sequence's chunks with its own initial and final state. Two small kernels serve the entry points:
//   chunk_table_kernel  cu_seqlens [N + 1] -> the workspace's chunk table (each chunk's first row in the caller's
//                       arrays and its sequence's end), each sequence's first chunk (one CTA, a block scan of the
//                       per-sequence chunk counts; no host synchronisation, so the calls stay graph-capturable) and
//                       the sequences in descending chunk count (a counting sort over 1024 buckets), the order in
//                       which the state passes start them
//   scatter_kernel      the chunk-aligned rows the kernels wrote (o, dq, dk, dv in the workspace) -> the caller's
//                       packed rows (16-byte copies over the whole GPU; rows past a sequence's end are not copied)
#include <cuda_runtime.h>

#include <cstdint>

#include "gd_layout.cuh"

namespace gd {
namespace {

constexpr int kScanThreads = 1024;
constexpr int kMaxDevicesPacked = 64;
constexpr int kBuckets = 1024;  // chunk counts for the state passes' start order (longer sequences share the last)

__device__ __forceinline__ int clampi(int x, int lo, int hi) { return x < lo ? lo : (x > hi ? hi : x); }

// Sequence n covers rows [cu[n], cu[n + 1]) (clamped into [0, Tin] and to a non-negative length, so that any input
// stays in bounds; the caller checks the boundaries themselves); its chunks are numbered from seg[n]. Chunk entries
// past the last sequence's, and any beyond NT, are (0, 0) / not written.
__global__ void __launch_bounds__(kScanThreads) chunk_table_kernel(const int* __restrict__ cu, int N, int Tin, int NT,
                                                                   int2* __restrict__ ctab, int* __restrict__ seg,
                                                                   int* __restrict__ ord) {
  __shared__ int warp_tot[kScanThreads / 32];
  __shared__ int carry, next_carry;
  __shared__ int bucket[kBuckets];
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

  // the order: bucket = chunk count (capped); buckets laid out from the largest down; within a bucket any order
  // (only which CTA starts when depends on it, not any result)
  for (int i = tid; i < kBuckets; i += kScanThreads) bucket[i] = 0;
  __syncthreads();  // also publishes seg (global writes of this CTA, read back below)
  for (int n = tid; n < N; n += kScanThreads) {
    const int cnt = seg[n + 1] - seg[n];
    atomicAdd(&bucket[cnt < kBuckets - 1 ? cnt : kBuckets - 1], 1);
  }
  __syncthreads();
  {  // exclusive offsets, largest bucket first: thread i scans bucket kBuckets - 1 - i (block scan as above)
    static_assert(kBuckets == kScanThreads, "one bucket a thread");
    const int mine = bucket[kBuckets - 1 - tid];
    int incl = mine;
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
      warp_tot[lane] = w;
    }
    __syncthreads();
    if (warp > 0) incl += warp_tot[warp - 1];
    bucket[kBuckets - 1 - tid] = incl - mine;
  }
  __syncthreads();
  for (int n = tid; n < N; n += kScanThreads) {
    const int cnt = seg[n + 1] - seg[n];
    ord[atomicAdd(&bucket[cnt < kBuckets - 1 ? cnt : kBuckets - 1], 1)] = n;
  }
}

// Row r of chunk c (padded row c * 64 + r) goes to row ctab[c].x + r of the caller's array when that is below
// ctab[c].y. row_bytes: one row's bytes (heads x D x element size, a multiple of 16). A grid-stride walk over the
// padded rows' 16-byte units, kUnroll of them in flight a thread.
constexpr int kUnroll = 4;
__global__ void __launch_bounds__(256) scatter_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                                      const int2* __restrict__ ctab, int per_row, long long units) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i0 = (long long)blockIdx.x * blockDim.x + threadIdx.x; i0 < units; i0 += stride * kUnroll) {
    uint4 v[kUnroll];
    long long to[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const long long i = i0 + u * stride;
      to[u] = -1;
      if (i < units) {
        const long long p = i / per_row;  // padded row
        const int2 e = __ldg(ctab + (p >> 6));
        const int t = e.x + (int)(p & 63);
        if (t < e.y) {
          to[u] = (long long)t * per_row + (i - p * per_row);
          v[u] = __ldg(src + i);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
      if (to[u] >= 0) dst[to[u]] = v[u];
  }
}

}  // namespace

cudaError_t launch_chunk_table(const int* cu_seqlens, const Layout& lay, unsigned char* ws, cudaStream_t st) {
  chunk_table_kernel<<<1, kScanThreads, 0, st>>>(cu_seqlens, lay.N, lay.Tin, lay.NT,
                                                 reinterpret_cast<int2*>(ws + lay.ctab),
                                                 reinterpret_cast<int*>(ws + lay.seg),
                                                 reinterpret_cast<int*>(ws + lay.ord));
  return cudaGetLastError();
}

cudaError_t launch_scatter(const void* src, void* dst, int row_bytes, const Layout& lay, const unsigned char* ws,
                           cudaStream_t st) {
  static int sms[kMaxDevicesPacked] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevicesPacked) return cudaErrorInvalidDevice;
  if (sms[dev] == 0 && (e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
    return e;
  const int per_row = row_bytes / 16;
  const long long units = (long long)lay.NT * 64 * per_row;
  const long long want = (units + 256LL * kUnroll - 1) / (256LL * kUnroll);
  const int grid = (int)(want < 8LL * sms[dev] ? (want > 0 ? want : 1) : 8LL * sms[dev]);
  scatter_kernel<<<grid, 256, 0, st>>>(static_cast<const uint4*>(src), static_cast<uint4*>(dst),
                                       reinterpret_cast<const int2*>(ws + lay.ctab), per_row, units);
  return cudaGetLastError();
}

}  // namespace gd
