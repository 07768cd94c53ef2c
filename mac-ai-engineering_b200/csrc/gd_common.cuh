// Shared device helpers for the chunked gated delta rule kernels (sm_100a only).
//
// - tcgen05 tensor-core primitives: TMEM allocation, bf16 x bf16 -> fp32 MMA from shared-memory descriptors, commit to an
//   mbarrier, TMEM -> register loads. Encodings follow the PTX ISA (tcgen05 instruction and shared-memory matrix
//   descriptors, the SWIZZLE_NONE canonical layouts).
// - bounded mbarrier waits: every wait gives up after a fixed number of SM clocks, records GD_ERR_TIMEOUT in the call's error
//   word and lets the kernel fall through to its clean-up (TMEM is always freed); no kernel traps or spins forever.
// - the "blocked" bf16 tile layout used for every MMA operand: a [R x C] matrix (R, C multiples of 8) is stored as 8 x 8
//   core matrices of 128 contiguous bytes (8 rows of 16 bytes), core (rb, cb) at byte ((rb * C/8) + cb) * 128. The same
//   bytes serve as a K-major operand (rows = M or N, cols = K) or an MN-major one (rows = K, cols = M or N); only the
//   descriptor's two strides differ.
#pragma once

#include <cstdint>
#include <type_traits>
#include <cuda.h>  // CUtensorMap (the descriptor type only; the encoder is fetched at run time)
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "gated_delta_b200.h"

namespace gd {

constexpr int C = 64;                      // chunk length (tokens); every chunk matrix is C x C
constexpr long long kWaitCycles = 4000000000ll;  // SM clocks a wait may take before it gives up (~2 s at 1.9 GHz)

// ------------------------------------------------------------------------------------------------------------------
// error word: the first 64 bytes of every workspace; kernels set the first failure code and the place it happened

struct ErrorWord {
  int code;
  int where;
  int block;
  int pad[13];
};

// Phase tracing for builds with -DGD_TRACE (profiling only; a normal build compiles it away): thread 0 of each
// 128-thread group of CTA (0, 0, 0) stores clock64() into the trace area of the workspace at (group, slot).
#ifdef GD_TRACE
#define GD_TRACE_AT(ws, lay, slot)                                                                        \
  do {                                                                                                    \
    if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && (threadIdx.x & 127) == 0 && (slot) < 4096) \
      reinterpret_cast<long long*>((ws) + (lay).trace)[(threadIdx.x >> 7) * 4096 + (slot)] = clock64();   \
  } while (0)
// the same from a single calling thread (an issuer lane), into group 0's row
#define GD_TRACE_ONE(ws, lay, slot)                                                              \
  do {                                                                                           \
    if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && (slot) < 4096)                  \
      reinterpret_cast<long long*>((ws) + (lay).trace)[(slot)] = clock64();                      \
  } while (0)
// lane 0 of every warp of CTA (0, 0, 0): slot (< 16) of its warp in row 3 from index 2048
#define GD_TRACE_WARP(ws, lay, slot)                                                                    \
  do {                                                                                                  \
    if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && (threadIdx.x & 31) == 0 && (slot) < 16)  \
      reinterpret_cast<long long*>((ws) + (lay).trace)[3 * 4096 + 2048 + (threadIdx.x >> 5) * 16 + (slot)] = \
          clock64();                                                                                    \
  } while (0)
// per CTA (up to 4096 of them): SM id, then globaltimer (ns) at entry (which 0) and exit (which 1), in rows 1-3
#define GD_TRACE_CTA(ws, lay, which)                                                                    \
  do {                                                                                                  \
    const unsigned int cta_ = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);           \
    if (threadIdx.x == 0 && cta_ < 4096) {                                                              \
      unsigned long long t_;                                                                            \
      unsigned int sm_;                                                                                 \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                                            \
      asm volatile("mov.u32 %0, %%smid;" : "=r"(sm_));                                                  \
      long long* tr_ = reinterpret_cast<long long*>((ws) + (lay).trace);                                \
      tr_[4096 + cta_] = sm_;                                                                           \
      tr_[4096 * (2 + (which)) + cta_] = (long long)t_;                                                 \
    }                                                                                                   \
  } while (0)
#else
#define GD_TRACE_CTA(ws, lay, which) \
  do {                               \
  } while (0)
#define GD_TRACE_AT(ws, lay, slot) \
  do {                             \
  } while (0)
#define GD_TRACE_ONE(ws, lay, slot) \
  do {                              \
  } while (0)
#define GD_TRACE_WARP(ws, lay, slot) \
  do {                               \
  } while (0)
#endif

__device__ __forceinline__ void report(ErrorWord* err, int code, int where) {
  if (err != nullptr && atomicCAS(&err->code, 0, code) == 0) {
    err->where = where;
    err->block = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  }
}

// ------------------------------------------------------------------------------------------------------------------
// host: the dynamic shared-memory opt-in of a kernel, set once per device (the first call of an entry point on a
// device must therefore come before any stream capture that records it)

constexpr int kMaxDevices = 64;

template <typename K>
inline cudaError_t set_smem_once(K kern, size_t bytes, bool (&done)[kMaxDevices]) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < kMaxDevices && done[dev]) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e == cudaSuccess && dev >= 0 && dev < kMaxDevices) done[dev] = true;
  return e;
}

// The query scale of GD_SCALE_Q: (key head width)^-1/2, the width from the flags' GD_KEY_WIDTH bits when the caller
// zero-padded narrower heads to DK, else DK; 1 without GD_SCALE_Q.
__device__ __forceinline__ float q_scale(int flags, int DK) {
  if (!(flags & GD_SCALE_Q)) return 1.f;
  const int w = (flags & GD_KEY_WIDTH_MASK) >> 16;
  return rsqrtf((float)(w ? w : DK));
}

// ------------------------------------------------------------------------------------------------------------------
// shared memory, fences, mbarriers, bulk copies

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking test of the phase with this parity (for threads that poll several barriers in turn: try_wait may
// suspend the thread on one barrier while another becomes ready).
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase with this parity to complete. Returns false (and records a timeout) if it does not within the
// poll limit; callers then skip their remaining work and go to clean-up.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, ErrorWord* err, int where) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitCycles) {
      report(err, GD_ERR_TIMEOUT, where);
      return false;
    }
  }
  return true;
}

// The same with a caller-chosen budget (SM clocks).
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, ErrorWord* err, int where,
                                              long long budget) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > budget) {
      report(err, GD_ERR_TIMEOUT, where);
      return false;
    }
  }
  return true;
}

// Budget of the test-only wait that GD_TEST_WAIT_EXPIRES adds (~1 ms at 1.9 GHz).
constexpr long long kTestWaitCycles = 2000000ll;

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// One arrival per warp after the whole warp got here (lane 0 arrives; the barrier counts warps).
__device__ __forceinline__ void mbar_arrive_warp(uint64_t* bar) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// 1-D bulk copy (TMA engine) global -> shared, completion counted on the mbarrier in bytes. Both addresses 16-byte
// aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---- host: TMA tensor maps over [B, T, heads, D] 16-bit rows (D innermost); box = one head's D columns x 64 tokens
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled from the driver (a host-only function: no device work, usable during stream capture)
inline EncodeTiled encode_tiled() {
  static EncodeTiled fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult res{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &res) != cudaSuccess ||
        res != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<EncodeTiled>(p);
  }();
  return fn;
}

// loads past T read zeros; stores past T are not written. box_d: the box's columns (default all D)
inline bool rows_map(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int B, int T, int heads, int D,
                     int box_d = 0) {
  EncodeTiled enc = encode_tiled();
  if (enc == nullptr) return false;
  const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)heads, (cuuint64_t)T, (cuuint64_t)B};
  const cuuint64_t strides[3] = {(cuuint64_t)D * 2, (cuuint64_t)heads * D * 2, (cuuint64_t)T * heads * D * 2};
  const cuuint32_t box[4] = {(cuuint32_t)(box_d > 0 ? box_d : D), 1, 64, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return enc(m, dt, 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename T>
constexpr CUtensorMapDataType map_dtype() {
  return std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
}

// The reverse: a 4-D tiled tensor copy shared -> global (TMA engine), in the issuing thread's bulk async-group;
// elements outside the tensor are not written. c0 is the innermost coordinate.
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, int c0, int c1, int c2, int c3, const void* src) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%1, %2, %3, %4}], [%5];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(src))
               : "memory");
}

// A 4-D tiled tensor copy global -> shared (TMA engine, no multicast) completing on an mbarrier (transaction bytes =
// the whole box; out-of-range elements arrive as zeros). c0 is the innermost coordinate.
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

// 1-D bulk copy shared -> global (TMA engine), tracked by the issuing thread's bulk async-group.
__device__ __forceinline__ void bulk_s2g(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem_u32(src)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// generic-proxy shared-memory writes -> visible to the async proxy (tensor core, bulk copies)
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ------------------------------------------------------------------------------------------------------------------
// tcgen05

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {  // one full warp
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {  // one full warp
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Instruction descriptor, kind::f16 with bf16 A and B, fp32 accumulator. a_mn / b_mn: operand is MN-major.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4)                          // D format: f32
         | (1u << 7)                        // A format: bf16
         | (1u << 10)                       // B format: bf16
         | ((a_mn ? 1u : 0u) << 15)         // A major
         | ((b_mn ? 1u : 0u) << 16)         // B major
         | ((uint32_t)(N >> 3) << 17)       // N / 8
         | ((uint32_t)(M >> 4) << 24);      // M / 16
}

// Shared-memory matrix descriptor, SWIZZLE_NONE. lbo: byte stride between 8-element groups along K;
// sbo: byte stride between 8-row groups along M (or N).
__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// A bf16 tile in the blocked layout: smem byte address and its column count (the row-block stride is cols/8 * 128 B).
struct Tile {
  uint32_t addr;
  uint32_t cols;
  __device__ __forceinline__ uint32_t rowblk_bytes() const { return (cols / 8) * 128; }
};

// D[M x N] (+)= X[M x K] . Y[K x N], every operand a blocked tile.
//   x_rows_m: X's tile rows index M (K-major A); otherwise the tile is X^T (rows index K: MN-major A).
//   y_rows_k: Y's tile rows index K (MN-major B); otherwise the tile is Y^T (rows index N: K-major B).
// (m0, n0, k0) select a sub-block of the tiles (multiples of 8, 8, 16). Issued by one thread.
// negate_x: D (+)= -X . Y (the instruction descriptor's negate-A bit).
__device__ __forceinline__ void mma_tiles(uint32_t d_tmem, int M, int N, int K, Tile x, bool x_rows_m, int m0, int k0,
                                          Tile y, bool y_rows_k, int n0, bool accumulate, bool negate_x = false) {
  const uint32_t idesc = idesc_bf16(M, N, !x_rows_m, y_rows_k) | (negate_x ? (1u << 13) : 0u);
  uint32_t xa, x_lbo, x_sbo, x_step, ya, y_lbo, y_sbo, y_step;
  if (x_rows_m) {  // K-major: K groups adjacent (128 B), M groups one row block apart
    xa = x.addr + (m0 / 8) * x.rowblk_bytes() + (k0 / 8) * 128;
    x_lbo = 128;
    x_sbo = x.rowblk_bytes();
    x_step = 256;
  } else {  // MN-major: M groups adjacent, K groups one row block apart
    xa = x.addr + (k0 / 8) * x.rowblk_bytes() + (m0 / 8) * 128;
    x_lbo = x.rowblk_bytes();
    x_sbo = 128;
    x_step = 2 * x.rowblk_bytes();
  }
  if (y_rows_k) {  // MN-major B
    ya = y.addr + (k0 / 8) * y.rowblk_bytes() + (n0 / 8) * 128;
    y_lbo = y.rowblk_bytes();
    y_sbo = 128;
    y_step = 2 * y.rowblk_bytes();
  } else {  // K-major B
    ya = y.addr + (n0 / 8) * y.rowblk_bytes() + (k0 / 8) * 128;
    y_lbo = 128;
    y_sbo = y.rowblk_bytes();
    y_step = 256;
  }
  // the descriptors once; each K step moves only the 14-bit start-address field (shared addresses < 2^18, so the
  // field never carries into the strides)
  const uint64_t dx = sdesc(xa, x_lbo, x_sbo), dy = sdesc(ya, y_lbo, y_sbo);
  const uint64_t sx = x_step >> 4, sy = y_step >> 4;
  mma_bf16(d_tmem, dx, dy, idesc, accumulate ? 1u : 0u);
#pragma unroll 8
  for (int kk = 1; kk < K / 16; ++kk) mma_bf16(d_tmem, dx + kk * sx, dy + kk * sy, idesc, 1u);
}

// TMEM -> registers: this warp's 32 lanes, 32 consecutive fp32 columns each (thread t gets lane (lane_base + t)).
// The load and its wait are one asm statement, so no use of the registers can be scheduled before the wait.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// TMEM -> registers: this warp's 32 lanes, 16 consecutive fp32 columns each.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 8 consecutive 32-bit columns of the thread's own lane (shape 32x32b: M = 128 accumulators, row = lane).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// Two such loads in flight under one wait.
__device__ __forceinline__ void tmem_ld16x2(uint32_t a0, float (&v0)[16], uint32_t a1, float (&v1)[16]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%32];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%33];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(a0), "r"(a1)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    v0[i] = __uint_as_float(r[i]);
    v1[i] = __uint_as_float(r[16 + i]);
  }
}

// An M = 64 accumulator (rows in lanes 0-15 of each 32-lane quadrant) read by a whole warp: shape 16x32bx2, thread
// t < 16 gets row (quadrant base + t), columns [col, col + 8); thread t >= 16 the same row t - 16, columns
// [col + 8, col + 16). taddr carries the quadrant's lane base and col.
__device__ __forceinline__ void tmem_ld8h(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.16x32bx2.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8], 8;\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// The same with 4 columns a half-warp: thread t < 16 gets row (quadrant base + t), columns [col, col + 4); thread
// t >= 16 the same row t - 16, columns [col + 4, col + 8). Two loads under one wait.
__device__ __forceinline__ void tmem_ld4hx2(uint32_t a0, float (&v0)[4], uint32_t a1, float (&v1)[4]) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.16x32bx2.x4.b32 {%0,%1,%2,%3}, [%8], 4;\n\t"
      "tcgen05.ld.sync.aligned.16x32bx2.x4.b32 {%4,%5,%6,%7}, [%9], 4;\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
      : "r"(a0), "r"(a1)
      : "memory");
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v0[i] = __uint_as_float(r[i]);
    v1[i] = __uint_as_float(r[4 + i]);
  }
}

__device__ __forceinline__ void tmem_ld4h(uint32_t taddr, float (&v)[4]) {
  uint32_t r[4];
  asm volatile(
      "tcgen05.ld.sync.aligned.16x32bx2.x4.b32 {%0,%1,%2,%3}, [%4], 4;\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(r[i]);
}

// Two such loads under one wait.
__device__ __forceinline__ void tmem_ld8hx2(uint32_t a0, float (&v0)[8], uint32_t a1, float (&v1)[8]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.16x32bx2.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%16], 8;\n\t"
      "tcgen05.ld.sync.aligned.16x32bx2.x8.b32 {%8,%9,%10,%11,%12,%13,%14,%15}, [%17], 8;\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(a0), "r"(a1)
      : "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v0[i] = __uint_as_float(r[i]);
    v1[i] = __uint_as_float(r[8 + i]);
  }
}

// Three such loads under one wait.
__device__ __forceinline__ void tmem_ld8hx3(uint32_t a0, float (&v0)[8], uint32_t a1, float (&v1)[8], uint32_t a2,
                                            float (&v2)[8]) {
  uint32_t r[24];
  asm volatile(
      "tcgen05.ld.sync.aligned.16x32bx2.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%24], 8;\n\t"
      "tcgen05.ld.sync.aligned.16x32bx2.x8.b32 {%8,%9,%10,%11,%12,%13,%14,%15}, [%25], 8;\n\t"
      "tcgen05.ld.sync.aligned.16x32bx2.x8.b32 {%16,%17,%18,%19,%20,%21,%22,%23}, [%26], 8;\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23])
      : "r"(a0), "r"(a1), "r"(a2)
      : "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v0[i] = __uint_as_float(r[i]);
    v1[i] = __uint_as_float(r[8 + i]);
    v2[i] = __uint_as_float(r[16 + i]);
  }
}

// The same shape with 16 columns per half: thread t < 16 gets row (base + t), columns [col, col + 16); thread t >= 16
// row t - 16, columns [col + 16, col + 32).
__device__ __forceinline__ void tmem_ld16h(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.16x32bx2.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16], 16;\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Reduce-scatter inside each 16-lane half of a warp: lane l gets the sum over its half's 16 lanes of v[l % 8]
// (lanes l and l ^ 8 hold the same sum).
__device__ __forceinline__ float halfwarp_reduce_scatter8(float (&v)[8]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int s = 4; s >= 1; s >>= 1) {
    const bool upper = (lane & s) != 0;
#pragma unroll
    for (int k = 0; k < s; ++k) {
      const float send = upper ? v[k] : v[k + s];
      const float keep = upper ? v[k + s] : v[k];
      v[k] = keep + __shfl_xor_sync(0xffffffffu, send, s);
    }
  }
  return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 8);
}

// TMEM address of column `col` in the lane quadrant of this warp (warps w, w+4, w+8, ... share a quadrant).
__device__ __forceinline__ uint32_t tmem_lane_addr(uint32_t base, int warp, int col) {
  return base + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)col;
}

// The accumulator row a thread owns after a tcgen05.ld 32x32b: M = 128 -> row = lane; M = 64 -> rows live in lanes
// 0-15 of each quadrant (row = 16 * quadrant + lane), lanes 16-31 hold nothing.
__device__ __forceinline__ int acc_row(int M, int warp, int lane) {
  return M == 128 ? 32 * (warp & 3) + lane : (lane < 16 ? 16 * (warp & 3) + lane : -1);
}

// ------------------------------------------------------------------------------------------------------------------
// blocked-tile element addressing and conversions

__host__ __device__ constexpr uint32_t blk_off(int r, int c, int cols) {  // byte offset of bf16 element (r, c)
  return (uint32_t)((((r >> 3) * (cols >> 3) + (c >> 3)) << 7) + ((r & 7) << 4) + ((c & 7) << 1));
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Split x into hi + lo, both bf16: hi = bf16(x), lo = bf16(x - hi). hi + lo carries ~16 significant bits.
__device__ __forceinline__ void split_bf16(float x, float& hi, float& lo) {
  hi = __bfloat162float(__float2bfloat16_rn(x));
  lo = x - hi;
}

// 8 consecutive floats of one tile row -> one 16-byte blocked-row segment (bf16)
__device__ __forceinline__ void store8_bf16(unsigned char* tile, int r, int c0, int cols, const float* v) {
  uint4 u;
  u.x = pack_bf16(v[0], v[1]);
  u.y = pack_bf16(v[2], v[3]);
  u.z = pack_bf16(v[4], v[5]);
  u.w = pack_bf16(v[6], v[7]);
  *reinterpret_cast<uint4*>(tile + blk_off(r, c0, cols)) = u;
}

// Four bf16 (8 bytes) at (r, c0 .. c0 + 3) of a blocked tile, c0 % 4 == 0; and the same with a hi / lo split
__device__ __forceinline__ void store4_bf16(unsigned char* tile, int r, int c0, int cols, const float* v) {
  *reinterpret_cast<uint2*>(tile + blk_off(r, c0, cols)) = make_uint2(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]));
}
// (a, b) -> their bf16 high halves packed (low 16 bits: a) and the packed bf16 remainders a - hi(a), b - hi(b): the
// values of split_bf16, with one paired conversion for the high halves (read back by shift and mask)
__device__ __forceinline__ void split_pack_bf16(float a, float b, uint32_t& hi, uint32_t& lo) {
  hi = pack_bf16(a, b);
  lo = pack_bf16(a - __uint_as_float(hi << 16), b - __uint_as_float(hi & 0xffff0000u));
}
__device__ __forceinline__ void store4_split(unsigned char* hi_tile, unsigned char* lo_tile, int r, int c0, int cols,
                                             const float* v) {
  uint2 h, l;
  split_pack_bf16(v[0], v[1], h.x, l.x);
  split_pack_bf16(v[2], v[3], h.y, l.y);
  *reinterpret_cast<uint2*>(hi_tile + blk_off(r, c0, cols)) = h;
  *reinterpret_cast<uint2*>(lo_tile + blk_off(r, c0, cols)) = l;
}

// the same with a hi / lo split into two tiles
// 8 floats -> their packed bf16 high halves and remainders (split_bf16's values), for storing more than once
__device__ __forceinline__ void split8_bf16(const float* v, uint4& h, uint4& l) {
  split_pack_bf16(v[0], v[1], h.x, l.x);
  split_pack_bf16(v[2], v[3], h.y, l.y);
  split_pack_bf16(v[4], v[5], h.z, l.z);
  split_pack_bf16(v[6], v[7], h.w, l.w);
}
__device__ __forceinline__ void store8_pair(unsigned char* hi_tile, unsigned char* lo_tile, int r, int c0, int cols,
                                            const uint4& h, const uint4& l) {
  *reinterpret_cast<uint4*>(hi_tile + blk_off(r, c0, cols)) = h;
  *reinterpret_cast<uint4*>(lo_tile + blk_off(r, c0, cols)) = l;
}
__device__ __forceinline__ void store8_split(unsigned char* hi_tile, unsigned char* lo_tile, int r, int c0, int cols,
                                             const float* v) {
  uint4 h, l;
  split8_bf16(v, h, l);
  store8_pair(hi_tile, lo_tile, r, c0, cols, h, l);
}

// A blocked [R x Cc] bf16 tile in shared memory -> its transpose, a blocked [Cc x R] image in global memory. Each warp
// moves four 8 x 8 core matrices per step: ldmatrix.trans hands lane l the transposed core's row l / 4, elements
// 2 (l % 4) and 2 (l % 4) + 1, which is the 4-byte word l of that 128-byte core (so a warp's stores are contiguous).
template <int R, int Cc, int NWARPS>
__device__ __forceinline__ void store_tile_transposed(const unsigned char* src, unsigned char* dst) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int NCORE = (R / 8) * (Cc / 8);
  static_assert(NCORE % 4 == 0, "whole groups of four core matrices");
  for (int gidx = warp; gidx < NCORE / 4; gidx += NWARPS) {
    const uint32_t addr = smem_u32(src + (4 * gidx + (lane >> 3)) * 128 + (lane & 7) * 16);
    uint32_t r[4];
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int cs = 4 * gidx + i, rb = cs / (Cc / 8), cb = cs % (Cc / 8);  // source core (rb, cb) -> (cb, rb)
      reinterpret_cast<uint32_t*>(dst + ((size_t)cb * (R / 8) + rb) * 128)[lane] = r[i];
    }
  }
}

template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

// Load 8 consecutive elements (16-byte aligned for 16-bit types, 32-byte for fp32) as floats.
template <typename T>
__device__ __forceinline__ void load8(const T* p, float* v);
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float* v) {
  uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void load8<__half>(const __half* p, float* v) {
  uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void load8<float>(const float* p, float* v) {
  float4 a = __ldg(reinterpret_cast<const float4*>(p));
  float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// x where c holds, else +0, as a bit AND (x may be inf or NaN where c fails). A select of an expensive expression
// (x * exp(..)) is compiled into per-element branches that serialise otherwise independent chains.
__device__ __forceinline__ float keep_if(float x, bool c) {
  return __uint_as_float(__float_as_uint(x) & (0u - (unsigned)c));
}

// one output element, rounded as store8 rounds
template <typename T>
__device__ __forceinline__ T cvt_out(float x);
template <>
__device__ __forceinline__ __nv_bfloat16 cvt_out<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ __half cvt_out<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ float cvt_out<float>(float x) { return x; }

template <typename T>
__device__ __forceinline__ void store8(T* p, const float* v);
template <>
__device__ __forceinline__ void store8<__nv_bfloat16>(__nv_bfloat16* p, const float* v) {
  uint4 u;
  u.x = pack_bf16(v[0], v[1]);
  u.y = pack_bf16(v[2], v[3]);
  u.z = pack_bf16(v[4], v[5]);
  u.w = pack_bf16(v[6], v[7]);
  *reinterpret_cast<uint4*>(p) = u;
}
template <>
__device__ __forceinline__ void store8<__half>(__half* p, const float* v) {
  uint4 u;
  __half2 h[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
  u = *reinterpret_cast<uint4*>(h);
  *reinterpret_cast<uint4*>(p) = u;
}
template <>
__device__ __forceinline__ void store8<float>(float* p, const float* v) {
  reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}

// v[16]: this lane's values at head-dimension index d0 + lane % 8 (d0: its 8-lane group's first index) for tokens
// tok + 0 .. 15. An 8 x 8 transpose inside each 8-lane group (three shuffle rounds) leaves lane L with tokens tok + L
// and tok + 8 + L at the group's 8 consecutive indices, each stored as one 8-element row segment (16 bytes for
// 16-bit T) at out + t * tok_stride + d0; tokens t >= T_ are skipped.
template <typename T>
__device__ __forceinline__ void store_token_rows(float (&v)[16], T* out, size_t tok_stride, int tok, int T_, int d0) {
  const int L = threadIdx.x & 7;
#pragma unroll
  for (int s = 4; s >= 1; s >>= 1) {
    const bool upper = (L & s) != 0;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      if ((e & s) == 0) {  // the pair (e, e + s) inside one 8-block
        const float send = upper ? v[e] : v[e + s];
        const float recv = __shfl_xor_sync(0xffffffffu, send, s);
        if (upper) {
          v[e] = recv;
        } else {
          v[e + s] = recv;
        }
      }
    }
  }
#pragma unroll
  for (int blk = 0; blk < 2; ++blk) {
    const int t = tok + 8 * blk + L;
    if (t < T_) store8<T>(out + (size_t)t * tok_stride + d0, v + 8 * blk);
  }
}

// One 8 x 8 block of the above: v[8] at head-dimension index d0 + lane % 8 for tokens tok .. tok + 7; after the
// transpose lane L stores token tok + L (if below T_) at d0 .. d0 + 7.
template <typename T>
__device__ __forceinline__ void store_token_rows8(float (&v)[8], T* out, size_t tok_stride, int tok, int T_, int d0) {
  const int L = threadIdx.x & 7;
#pragma unroll
  for (int s = 4; s >= 1; s >>= 1) {
    const bool upper = (L & s) != 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      if ((e & s) == 0) {
        const float send = upper ? v[e] : v[e + s];
        const float recv = __shfl_xor_sync(0xffffffffu, send, s);
        if (upper) {
          v[e] = recv;
        } else {
          v[e + s] = recv;
        }
      }
    }
  }
  const int t = tok + L;
  if (t < T_) store8<T>(out + (size_t)t * tok_stride + d0, v);
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}


// 64 rows x D of a [B, T, heads, D] tensor -> a blocked bf16 tile, in two steps so that several tensors' loads are in
// flight at once: rows_issue starts the global loads into registers, rows_finish (after any other work) converts.
// With norm, each row is scaled by rsqrt(sum x^2 + eps) * scale (the l2 prologue of src/macai/gated_delta/_norm.py:27-43),
// else by `scale`. Rows past T, and every row when x is null, are zero. With lo_tile, the rounding remainder goes
// there (hi + lo). NWARPS warps share the 64 rows; each warp stores 8 rows x 32 columns per instruction (512
// contiguous bytes: no bank conflict).
template <typename T>
struct Piece {  // 8 consecutive elements, raw
  uint4 u;
  __device__ __forceinline__ void load(const T* p) { u = __ldg(reinterpret_cast<const uint4*>(p)); }
  __device__ __forceinline__ void load_shared(const unsigned char* p) { u = *reinterpret_cast<const uint4*>(p); }
  __device__ __forceinline__ void zero() { u = make_uint4(0, 0, 0, 0); }
  __device__ __forceinline__ void to_f32(float* v) const;
};
template <>
__device__ __forceinline__ void Piece<__nv_bfloat16>::to_f32(float* v) const {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void Piece<__half>::to_f32(float* v) const {
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
template <>
struct Piece<float> {
  float4 a, b;
  __device__ __forceinline__ void load(const float* p) {
    a = __ldg(reinterpret_cast<const float4*>(p));
    b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  }
  __device__ __forceinline__ void zero() { a = b = make_float4(0.f, 0.f, 0.f, 0.f); }
  __device__ __forceinline__ void to_f32(float* v) const {
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
};

// ROT: lane (r = lane % 8, g = lane / 8) holds the 8-column groups (r + 4 g + j) mod 16 of its row instead of g + 4 j,
// so that 8 rows 256 bytes apart in shared memory (a row-major staging of 16-bit rows, D = 128) are read by a
// quarter warp without bank conflicts.
template <typename T, int D, int NWARPS = 4, bool ROT = false>
struct Rows {
  static constexpr int J = D / 32;              // 8-column groups per lane
  static constexpr int RB = 64 / (8 * NWARPS);  // row blocks per warp
  static_assert(!ROT || (D == 128 && sizeof(T) == 2), "the rotated mapping covers 16 groups of 16 bytes a row");
  Piece<T> p[RB][J];
  __device__ __forceinline__ static int row(int rbi) {
    return 8 * (RB * (int)(threadIdx.x >> 5) + rbi) + (int)(threadIdx.x & 7);
  }
  __device__ __forceinline__ static int col(int j) {
    const int g = (int)((threadIdx.x & 31) >> 3);
    return ROT ? 8 * (((int)(threadIdx.x & 7) + 4 * g + j) & 15) : 8 * (g + 4 * j);
  }

  // the same pieces from row-major rows already in shared memory (row r at raw + r * D * sizeof(T)); rows past T_ zero
  __device__ __forceinline__ void issue_staged(const unsigned char* raw, int t0, int T_) {
#pragma unroll
    for (int rbi = 0; rbi < RB; ++rbi) {
      const int r = row(rbi);
      const bool valid = t0 + r < T_;
#pragma unroll
      for (int j = 0; j < J; ++j) {
        if (valid) {
          p[rbi][j].load_shared(raw + ((size_t)r * D + col(j)) * sizeof(T));
        } else {
          p[rbi][j].zero();
        }
      }
    }
  }

  // rows t0 + r of batch row b of x [B][rows][heads][D]; rows at or past `end` zero
  __device__ __forceinline__ void issue(const T* x, int b, int t0, int rows, int end, int heads, int hh) {
#pragma unroll
    for (int rbi = 0; rbi < RB; ++rbi) {
      const int t = t0 + row(rbi);
      const bool valid = x != nullptr && t < end;
      const T* rp = x + (((size_t)b * rows + (valid ? t : 0)) * heads + hh) * D;
#pragma unroll
      for (int j = 0; j < J; ++j) {
        if (valid) {
          p[rbi][j].load(rp + col(j));
        } else {
          p[rbi][j].zero();
        }
      }
    }
  }

  __device__ __forceinline__ void finish(int t0, int T_, bool norm, float scale, unsigned char* tile, float* rsq_out,
                                         unsigned char* lo_tile) const {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int rbi = 0; rbi < RB; ++rbi) {
      const int r = row(rbi), t = t0 + r;
      float vals[J][8];
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < J; ++j) {
        p[rbi][j].to_f32(vals[j]);
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = fmaf(vals[j][e], vals[j][e], ss);
      }
      float f = scale;
      if (norm) {
        ss += __shfl_xor_sync(0xffffffffu, ss, 8);
        ss += __shfl_xor_sync(0xffffffffu, ss, 16);
        const float rs = rsqrtf(ss + 1e-6f);
        f = rs * scale;
        if (rsq_out != nullptr && t < T_ && lane < 8) rsq_out[r] = rs;  // the chunk's 64 slots
      }
#pragma unroll
      for (int j = 0; j < J; ++j) {
#pragma unroll
        for (int e = 0; e < 8; ++e) vals[j][e] *= f;
        if (lo_tile != nullptr) {
          store8_split(tile, lo_tile, r, col(j), D, vals[j]);
        } else {
          store8_bf16(tile, r, col(j), D, vals[j]);
        }
      }
    }
  }
};

// Reduce-scatter across a warp: each lane holds v[0..31]; returns, in lane l, the sum over the warp's lanes of v[l]
// (31 shuffles instead of 32 x 5).
__device__ __forceinline__ float warp_reduce_scatter32(float (&v)[32]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) {
    const bool upper = (lane & s) != 0;
#pragma unroll
    for (int k = 0; k < s; ++k) {
      const float send = upper ? v[k] : v[k + s];
      const float keep = upper ? v[k + s] : v[k];
      v[k] = keep + __shfl_xor_sync(0xffffffffu, send, s);
    }
  }
  return v[0];
}

// Reduce-scatter of 16 values across a warp whose two half-warps hold different partial terms of the same 16 sums:
// returns, in lane l, the sum over all 32 lanes of v[l & 15] (31 shuffles).
__device__ __forceinline__ float warp_reduce_scatter16(float (&v)[16]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < 16; ++k) v[k] += __shfl_xor_sync(0xffffffffu, v[k], 16);
#pragma unroll
  for (int s = 8; s >= 1; s >>= 1) {
    const bool upper = (lane & s) != 0;
#pragma unroll
    for (int k = 0; k < s; ++k) {
      const float send = upper ? v[k] : v[k + s];
      const float keep = upper ? v[k + s] : v[k];
      v[k] = keep + __shfl_xor_sync(0xffffffffu, send, s);
    }
  }
  return v[0];
}

// bf16 element (r, c) of a blocked tile, as float
__device__ __forceinline__ float tile_at(const unsigned char* tile, int r, int c, int cols) {
  return __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(tile + blk_off(r, c, cols)));
}

// [64][64] fp32 C x C scratch, columns XOR-swizzled by row so that both row-wise and column-wise thread patterns are
// free of bank conflicts.
__device__ __forceinline__ int cc_idx(int i, int j) { return i * 64 + (j ^ (i & 31)); }

}  // namespace gd
