// Backward kernels of the chunked gated delta rule on B200 (sm_100a):
//   bwd_state_kernel  one CTA per (value head, batch row): the reverse sequential pass carrying dS = dLoss/dS in fp32
//                     registers, chunks last to first; keeps dS_{c+1} and dVn per chunk for the per-chunk kernel;
//   bwd_chunk_kernel  one CTA per (chunk, key head, batch row): every gradient of the chunk, all independent, no atomics.
// Equations (tools/check_chunk_equations.py:49-76 and src/macai/gated_delta/_chunked.py:20-34 of the reference):
//   dVn = M^T dO + diag(e) K dS_{c+1}
//   dS_c = exp(G_last) dS_{c+1} + (diag(gamma) Q)^T dO - W^T dVn
//   dM = Gamma * (dO Vn^T) (lower), dQ = diag(gamma) dO S_c^T + dM K, dKs = diag(e) Vn dS_{c+1}^T
//   dW = -dVn S_c^T, X = A^T dW, Y = A^T dVn, dV = diag(beta) Y
//   dA = strict_lower(dW (diag(beta gamma) K)^T + dVn (diag(beta) V)^T), dL = -A^T dA A^T (strictly lower)
//   P = dL * Gamma, dK = dM^T Q + dKs + diag(beta gamma) X + diag(beta) P K + P^T diag(beta) K
//   dbeta = gamma (k . X) + (v . Y) + rowsum(P * (K K^T)); dg without cancellation (see dg_chunk below).
// Precision (bf16 operands, fp32 accumulation): dS, gamma Q, dM, Vn (with dS), dVn (in A^T dVn) are split into bf16
// hi + lo pairs; every other operand is one bf16. The choice keeps every gradient within the parity bar with margin.
#include "gd_common.cuh"
#include "gd_layout.cuh"

namespace gd {

// ------------------------------------------------------------------------------------------------------------------
// reverse state pass

template <int DK, int DV>
struct BwdStateSmem {
  static constexpr size_t dth = 0;                       // [DV x DK] dS^T hi (rows v, cols dk)
  static constexpr size_t dtl = dth + DV * DK * 2;       //           lo
  static constexpr size_t qk = dtl + DV * DK * 2;        // stage: [2][64 x DK] q, k images (hi)
  static constexpr size_t qkl = qk + 2 * 64 * DK * 2;    // stage: [2][64 x DK] their low halves
  static constexpr size_t wt = qkl + 2 * 64 * DK * 2;    // stage: [DK x 64] W^T image
  static constexpr size_t m = wt + DK * 64 * 2;          // stage: [64 x 64] M image
  static constexpr size_t g = m + 64 * 64 * 2;           // stage: [64] G
  static constexpr size_t dO = g + 64 * 4;               // [64 x DV] dO tile
  static constexpr size_t gqh = dO + 64 * DV * 2;        // [64 x DK] (gamma Q) hi
  static constexpr size_t gql = gqh + 64 * DK * 2;       //                      lo
  static constexpr size_t dvt = gql + 64 * DK * 2;       // [DV x 64] dVn^T
  static constexpr size_t bar = dvt + DV * 64 * 2;       // 2 mbarriers: mma, inputs
  static constexpr size_t tmem = bar + 2 * 8;
  static constexpr size_t total = tmem + 8;
  static constexpr uint32_t stage_bytes = 4 * 64 * DK * 2 + DK * 64 * 2 + 64 * 64 * 2 + 64 * 4;
};

template <int DK, int DV, typename S>
__device__ __forceinline__ void issue_bwd_stage(unsigned char* smem, const unsigned char* ws, const Layout& lay,
                                                size_t cidx, uint64_t* bar) {
  mbar_arrive_expect_tx(bar, S::stage_bytes);
  bulk_g2s(smem + S::qk, ws + lay.qk + cidx * lay.qk_bytes(), (uint32_t)lay.qk_bytes(), bar);
  bulk_g2s(smem + S::qkl, ws + lay.qkl + cidx * lay.qk_bytes(), (uint32_t)lay.qk_bytes(), bar);
  bulk_g2s(smem + S::wt, ws + lay.wt + cidx * lay.wt_bytes(), (uint32_t)lay.wt_bytes(), bar);
  bulk_g2s(smem + S::m, ws + lay.m + cidx * lay.m_bytes(), (uint32_t)lay.m_bytes(), bar);
  bulk_g2s(smem + S::g, ws + lay.gc + cidx * lay.gc_bytes(), (uint32_t)lay.gc_bytes(), bar);
}

template <typename T, int DK, int DV>
__global__ void __launch_bounds__(128) bwd_state_kernel(const T* __restrict__ d_o, const float* __restrict__ dsT,
                                                        float* __restrict__ ds0, Layout lay, int flags,
                                                        unsigned char* __restrict__ ws) {
  static_assert(DV == 128, "the reverse pass maps one thread to each of 128 value columns");
  using S = BwdStateSmem<DK, DV>;
  extern __shared__ __align__(1024) unsigned char smem[];
  ErrorWord* err = reinterpret_cast<ErrorWord*>(ws + lay.err);
  const int h = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int vcol = tid;
  uint64_t* bar_mma = reinterpret_cast<uint64_t*>(smem + S::bar);
  uint64_t* bar_in = bar_mma + 1;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + S::tmem);
  const float* sG = reinterpret_cast<const float*>(smem + S::g);
  const size_t row0 = ((size_t)b * lay.H + h) * lay.NT;

  if (warp == 0) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(bar_mma, 1);
    mbar_init(bar_in, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) issue_bwd_stage<DK, DV, S>(smem, ws, lay, row0 + lay.NT - 1, bar_in);

  float dS[DK];  // column vcol of dLoss/dS (all key rows), fp32
  {
    const float* p = dsT ? dsT + ((size_t)b * lay.H + h) * DK * DV : nullptr;
#pragma unroll
    for (int d = 0; d < DK; ++d) dS[d] = p ? p[(size_t)d * DV + vcol] : 0.f;
#pragma unroll
    for (int d8 = 0; d8 < DK / 8; ++d8) store8_split(smem + S::dth, smem + S::dtl, vcol, 8 * d8, DK, dS + 8 * d8);
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = *tslot;
  const uint32_t tA = tm + 0, tB = tm + 64, tC = tm + 128, tD = tm + 256;

  uint32_t ph_mma = 0, ph_in = 0;
  bool ok = true;
  for (int c = lay.NT - 1; c >= 0 && ok; --c) {
    const size_t cidx = row0 + c;
    const int t0 = c * C;
    // dS_{c+1} for the per-chunk kernel, then this chunk's dO tile
    {
      float* dsn = reinterpret_cast<float*>(ws + lay.dsn + cidx * lay.s_bytes());
#pragma unroll
      for (int d = 0; d < DK; ++d) dsn[(size_t)d * DV + vcol] = dS[d];
    }
    load_rows<T, DV>(d_o, b, t0, lay.T, lay.H, h, false, 1.f, smem + S::dO, nullptr);
    ok = mbar_wait(bar_in, ph_in, err, 30);
    ph_in ^= 1;
    ok = __syncthreads_and(ok);
    if (!ok) break;
    // (gamma Q) hi / lo from the q image's hi + lo halves
    for (int idx = tid; idx < 64 * DK / 8; idx += 128) {
      const int rl = idx & 7, cb = (idx >> 3) % (DK / 8), rb = idx / (8 * (DK / 8));
      const int r = 8 * rb + rl;
      const uint4 u = *reinterpret_cast<const uint4*>(smem + S::qk + blk_off(r, 8 * cb, DK));
      const uint4 ul = *reinterpret_cast<const uint4*>(smem + S::qkl + blk_off(r, 8 * cb, DK));
      const __nv_bfloat162* hq = reinterpret_cast<const __nv_bfloat162*>(&u);
      const __nv_bfloat162* lq = reinterpret_cast<const __nv_bfloat162*>(&ul);
      const float gr = __expf(sG[r]);
      float v[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(hq[e]);
        const float2 fl = __bfloat1622float2(lq[e]);
        v[2 * e] = gr * (f.x + fl.x);
        v[2 * e + 1] = gr * (f.y + fl.y);
      }
      store8_split(smem + S::gqh, smem + S::gql, r, 8 * cb, DK, v);
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const Tile tdo{smem_u32(smem + S::dO), DV};
      // (M^T dO)^T = dO^T M  [DV x 64]
      mma_tiles(tA, DV, 64, 64, tdo, false, 0, 0, Tile{smem_u32(smem + S::m), 64}, true, 0, false);
      // (K dS)^T = dS^T K^T  [DV x 64], dS and K split (hi hi + hi lo + lo hi)
      const Tile tk{smem_u32(smem + S::qk + 64 * DK * 2), DK}, tkl{smem_u32(smem + S::qkl + 64 * DK * 2), DK};
      mma_tiles(tB, DV, 64, DK, Tile{smem_u32(smem + S::dth), DK}, true, 0, 0, tk, false, 0, false);
      mma_tiles(tB, DV, 64, DK, Tile{smem_u32(smem + S::dth), DK}, true, 0, 0, tkl, false, 0, true);
      mma_tiles(tB, DV, 64, DK, Tile{smem_u32(smem + S::dtl), DK}, true, 0, 0, tk, false, 0, true);
      // ((gamma Q)^T dO)^T = dO^T (gamma Q)  [DV x DK], gamma Q split
      mma_tiles(tC, DV, DK, 64, tdo, false, 0, 0, Tile{smem_u32(smem + S::gqh), DK}, true, 0, false);
      mma_tiles(tC, DV, DK, 64, tdo, false, 0, 0, Tile{smem_u32(smem + S::gql), DK}, true, 0, true);
      mma_commit(bar_mma);
    }
    ok = mbar_wait(bar_mma, ph_mma, err, 31);
    ph_mma ^= 1;
    ok = __syncthreads_and(ok);
    if (!ok) break;
    tc_fence_after();
    const float Glast = sG[63];
    {
      float a[32], bb[32], dvn[32];
      float* dvn_out = reinterpret_cast<float*>(ws + lay.dvn + cidx * lay.u_bytes());
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        tmem_ld32(tmem_lane_addr(tA, warp, 32 * half), a);
        tmem_ld32(tmem_lane_addr(tB, warp, 32 * half), bb);
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          const int i = 32 * half + jj;
          dvn[jj] = fmaf(__expf(Glast - sG[i]), bb[jj], a[jj]);
          dvn_out[i * DV + vcol] = dvn[jj];
        }
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) store8_bf16(smem + S::dvt, vcol, 32 * half + 8 * q8, 64, dvn + 8 * q8);
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      // (W^T dVn)^T = dVn^T W  [DV x DK]
      mma_tiles(tD, DV, DK, 64, Tile{smem_u32(smem + S::dvt), 64}, true, 0, 0, Tile{smem_u32(smem + S::wt), 64},
                false, 0, false);
      mma_commit(bar_mma);
    }
    ok = mbar_wait(bar_mma, ph_mma, err, 32);
    ph_mma ^= 1;
    ok = __syncthreads_and(ok);
    if (!ok) break;
    tc_fence_after();
    {
      const float gl = __expf(Glast);
      float cc[32], dd[32];
#pragma unroll
      for (int q4 = 0; q4 < DK / 32; ++q4) {
        tmem_ld32(tmem_lane_addr(tC, warp, 32 * q4), cc);
        tmem_ld32(tmem_lane_addr(tD, warp, 32 * q4), dd);
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) dS[32 * q4 + jj] = fmaf(gl, dS[32 * q4 + jj], cc[jj] - dd[jj]);
      }
#pragma unroll
      for (int d8 = 0; d8 < DK / 8; ++d8) store8_split(smem + S::dth, smem + S::dtl, vcol, 8 * d8, DK, dS + 8 * d8);
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0 && c > 0) issue_bwd_stage<DK, DV, S>(smem, ws, lay, cidx - 1, bar_in);
  }
  if (ok && ds0 != nullptr) {
    float* p = ds0 + ((size_t)b * lay.H + h) * DK * DV;
#pragma unroll
    for (int d = 0; d < DK; ++d) p[(size_t)d * DV + vcol] = dS[d];
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tm, 512);
  }
}

template <typename T, int DK, int DV>
cudaError_t launch_bwd_state(const void* d_o, const float* dsT, float* ds0, const Layout& lay, int flags,
                             unsigned char* ws, cudaStream_t st) {
  using S = BwdStateSmem<DK, DV>;
  auto kern = bwd_state_kernel<T, DK, DV>;
  static bool attr_done[kMaxDevices] = {};  // once per device: no attribute call inside a graph capture
  cudaError_t e = set_smem_once(kern, S::total, attr_done);
  if (e != cudaSuccess) return e;
  dim3 grid(lay.H, lay.B);
  kern<<<grid, 128, S::total, st>>>(static_cast<const T*>(d_o), dsT, ds0, lay, flags, ws);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------------------------
// per-chunk gradients (in gd_bwd_chunk.cu)

#define INST(T)                                                                                                    \
  template cudaError_t launch_bwd_state<T, 128, 128>(const void*, const float*, float*, const Layout&, int,         \
                                                     unsigned char*, cudaStream_t);
INST(__nv_bfloat16)
INST(__half)
INST(float)
#undef INST

}  // namespace gd
