// Per-chunk gradients of the chunked gated delta rule on B200 (sm_100a): one CTA of 256 threads per (chunk, key head,
// batch row), all CTAs independent, one writer per gradient element (no atomics; bitwise reproducible).
//
// Inputs per value head, all bf16 images from the workspace copied whole by the bulk-copy engine: the q / k images,
// A = (I + L)^-1 and V (prep), S_c^T and Vn^T (the forward state pass with GD_STORE_STATES), dS_{c+1}^T, dVn^T and dO
// (the reverse pass); G, M and K K^T in fp32 (prep), the partial sums of <S_c, dS_{c+1}> (reverse pass); from the
// caller: v, beta and, for the l2 prologue's backward, q and k.
//
// Products, all tcgen05 from blocked shared-memory tiles into TMEM (transposed "[D x 64]" accumulators put the head
// dimension on TMEM lanes; C x C ones use M = 64; an image with rows along a product's K dimension is its MN-major
// operand):
//   group 1:  dO Vn^T, (dO S_c^T)^T, (dVn S_c^T)^T, (A^T dVn)^T, dVn V^T
//   group 2:  (Vn dS^T)^T                      (Vn and dS split: three products)
//   group 3:  (dM K)^T, (dM^T Q)^T, (A^T dW)^T, dW K^T      (dM, q and k split: three products each)
// M (with its decay mask) and K K^T come in fp32 from the prep kernel; q and k as bf16 hi + lo images.
//   group 4:  T1 = dA A^T;  group 5: dL = -A^T T1;  group 6: (K^T Z)^T with Z = P_beta + P_beta^T, P_beta = diag(beta) P
// Equations: tools/check_chunk_equations.py:49-76 and src/macai/gated_delta/_chunked.py:20-34 of the reference; dg is
// summed without cancellation (the regrouping of _chunked.py:1138-1142, extended to the decay-mask terms):
//   dg_t = sum_{s>=t} (a_s + w_s) + gamma_last <S_c, dS_{c+1}> + sum_{r<t} E_r + sum_{i>=t>j} R_ij
//   a_s = gamma_s q_s . (dO S_c^T)_s, w_s = beta_s gamma_s k_s . X_s, E_r = e_r k_r . (Vn dS^T)_r,
//   R_ij = dM_ij (Q K^T)_ij + dL_ij L_ij.
#include "gd_common.cuh"
#include "gd_layout.cuh"

namespace gd {

template <int DK, int DV>
struct ChunkSmem {
  // bf16 tiles
  static constexpr size_t qk = 0;                        // [128 x DK]: q image (rows 0-63), k image (rows 64-127)
  static constexpr size_t qkl = qk + 2 * 64 * DK * 2;    // [128 x DK]: their low halves
  static constexpr size_t a = qkl + 2 * 64 * DK * 2;     // [64 x 64] A
  static constexpr size_t big = a + 64 * 64 * 2;         // 64 KB, reused by phase (see the kernel)
  static constexpr size_t sc = big;                      //   phase 1: [DV x DK] S_c^T
  static constexpr size_t dO = big + DK * DV * 2;        //            [64 x DV] dO
  static constexpr size_t v = dO + 64 * DV * 2;          //            [64 x DV] V
  static constexpr size_t dsh = big;                     //   phase 2: [DV x DK] dS^T hi
  static constexpr size_t dsl = big + DK * DV * 2;       //            [DV x DK] dS^T lo
  static constexpr size_t da = big;                      //   phase 3: [64 x 64] dA
  static constexpr size_t t1 = big + 8192;               //            [64 x 64] T1
  static constexpr size_t z = big + 16384;               //            [64 x 64] Z
  static constexpr size_t vn = big + 65536;              // 32 KB: [DV x 64] Vn^T hi, lo; later fp32 [64][64] P_beta, R
  static constexpr size_t vnl = vn + DV * 64 * 2;
  static constexpr size_t pb = vn;                       //   fp32 [64][64] P_beta (swizzled)
  static constexpr size_t r = vn + 16384;                //   fp32 [64][64] R (swizzled)
  static constexpr size_t dvn = vn + 32768;              // 32 KB: [DV x 64] dVn^T hi, lo; later dM hi, lo and dW^T
  static constexpr size_t dvnl = dvn + DV * 64 * 2;
  static constexpr size_t dmh = dvn;                     //   [64 x 64] dM hi
  static constexpr size_t dml = dvn + 8192;              //   [64 x 64] dM lo
  static constexpr size_t dwt = dvn + 16384;             //   [DK x 64] dW^T
  // fp32
  static constexpr size_t g = dvn + 32768;               // [64] G
  static constexpr size_t beta = g + 256;                // [64]
  static constexpr size_t part = beta + 256;             // [5][4][64] quadrant partial dots: a, kX, vY, E, xq/xk
  static constexpr size_t pk = part + 5 * 4 * 64 * 4;    // [2][64] row halves of sum_j P_ij KG_ij
  static constexpr size_t red = pk + 2 * 64 * 4;         // [16] partial sums of <S_c, dS_{c+1}>
  static constexpr size_t bar = red + 64;                // 5 mbarriers: mma, q/k images, group 2, phase-1 and dS images
  static constexpr size_t tmem = bar + 40;
  static constexpr size_t total = tmem + 16;
};

__device__ __forceinline__ void block_sync_ok(bool& ok) { ok = __syncthreads_and(ok); }

template <typename T, int DK, int DV>
__global__ void __launch_bounds__(256) bwd_chunk_kernel(const T* __restrict__ qraw, const T* __restrict__ kraw,
                                                        const T* __restrict__ vraw, const float* __restrict__ beta,
                                                        const T* __restrict__ d_o, T* __restrict__ dq,
                                                        T* __restrict__ dk, T* __restrict__ dv,
                                                        float* __restrict__ dg, float* __restrict__ dbeta, Layout lay,
                                                        int flags, unsigned char* __restrict__ ws) {
  static_assert(DK == 128 && DV == 128, "the per-chunk kernel maps the head dimension onto the 128 TMEM lanes");
  using S = ChunkSmem<DK, DV>;
  extern __shared__ __align__(1024) unsigned char smem[];
  ErrorWord* err = reinterpret_cast<ErrorWord*>(ws + lay.err);
  const int c = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qd = warp & 3, half = warp >> 2;
  const int dcol = 32 * qd + lane;   // head-dimension index this thread owns in [D x 64] accumulators
  const int tok0 = 32 * half;        // its 32 tokens
  const int rrow = 16 * qd + lane;   // its row in M = 64 accumulators (lane < 16)
  const bool rowthr = lane < 16;
  const int t0 = c * C;
  float* sR = reinterpret_cast<float*>(smem + S::r);
  float* sG = reinterpret_cast<float*>(smem + S::g);
  float* sB = reinterpret_cast<float*>(smem + S::beta);
  float* sPart = reinterpret_cast<float*>(smem + S::part);
  float* sPk = reinterpret_cast<float*>(smem + S::pk);
  float* sRed = reinterpret_cast<float*>(smem + S::red);
  uint64_t* bar_mma = reinterpret_cast<uint64_t*>(smem + S::bar);
  uint64_t* bar_qk = bar_mma + 1;
  uint64_t* bar_g2 = bar_mma + 2;  // group 2 completes on its own barrier: its wait follows group 3's commit
  uint64_t* bar_in = bar_mma + 3;  // phase-1 images of one value head
  uint64_t* bar_ds = bar_mma + 4;  // dS images of one value head
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + S::tmem);
  const bool norm = (flags & GD_L2NORM) != 0;
  const float qscale = (flags & GD_SCALE_Q) ? rsqrtf((float)DK) : 1.f;

  if (warp == 0) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(bar_mma, 1);
    mbar_init(bar_qk, 1);
    mbar_init(bar_g2, 1);
    mbar_init(bar_in, 1);
    mbar_init(bar_ds, 1);
    fence_mbar_init();
  }
  __syncthreads();
  const size_t cidx0 = ((size_t)b * lay.H + (size_t)hk * lay.rep) * lay.NT + c;
  if (tid == 0) {  // the q / k images are the same for every value head of this key head
    mbar_arrive_expect_tx(bar_qk, 2 * (uint32_t)lay.qk_bytes());
    bulk_g2s(smem + S::qk, ws + lay.qk + cidx0 * lay.qk_bytes(), (uint32_t)lay.qk_bytes(), bar_qk);
    bulk_g2s(smem + S::qkl, ws + lay.qkl + cidx0 * lay.qk_bytes(), (uint32_t)lay.qk_bytes(), bar_qk);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = *tslot;
  // TMEM columns (each block 64 wide; reused once its reader is done)
  const uint32_t T_DAK = tm + 0, T_DL = tm + 0;
  const uint32_t T_DM = tm + 64;
  const uint32_t T_DQA = tm + 128;
  const uint32_t T_DW = tm + 192, T_X = tm + 192;
  const uint32_t T_Y = tm + 256, T_DKA = tm + 256;
  const uint32_t T_DAV = tm + 320, T_T1 = tm + 320, T_DKC = tm + 320;
  const uint32_t T_DKS = tm + 384;
  const uint32_t T_DQ = tm + 448;

  // q / k images are transposed ([DK x 64], rows d): the K-major operand wherever d is a product's M or N
  const Tile tQ{smem_u32(smem + S::qk), 64};
  const Tile tK{smem_u32(smem + S::qk + 64 * DK * 2), 64};
  const Tile tQl{smem_u32(smem + S::qkl), 64};
  const Tile tKl{smem_u32(smem + S::qkl + 64 * DK * 2), 64};
  // fp32 normalised q / k element (i, d) from the hi + lo images
  auto qhat = [&](int i, int d) {
    const int r = (i & 64) ? DK + d : d, cc = i & 63;  // token i of q (i < 64) or of k (i - 64)
    return __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(smem + S::qk + blk_off(r, cc, 64))) +
           __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(smem + S::qkl + blk_off(r, cc, 64)));
  };
  const Tile tA{smem_u32(smem + S::a), 64};

  float dQacc[32], dKacc[32];  // d(normalised q / k)[token tok0 + j][dcol], summed over the value heads
#pragma unroll
  for (int j = 0; j < 32; ++j) dQacc[j] = dKacc[j] = 0.f;

  uint32_t ph = 0;
  GD_TRACE_AT(ws, lay, 0);
  bool ok = mbar_wait(bar_qk, 0, err, 40);
  block_sync_ok(ok);

  for (int r = 0; r < lay.rep && ok; ++r) {
    const int h = hk * lay.rep + r;
    const size_t cidx = ((size_t)b * lay.H + h) * lay.NT + c;
    // ---------------- phase 1: operand images (bulk copies; the previous value head's readers are done)
    if (tid == 0) {
      const uint32_t bytes = (uint32_t)(lay.m_bytes() + lay.si_bytes() + 2 * lay.vi_bytes() + 2 * lay.vn_bytes());
      mbar_arrive_expect_tx(bar_in, bytes);
      bulk_g2s(smem + S::a, ws + lay.ai + cidx * lay.m_bytes(), (uint32_t)lay.m_bytes(), bar_in);
      bulk_g2s(smem + S::sc, ws + lay.sci + cidx * lay.si_bytes(), (uint32_t)lay.si_bytes(), bar_in);
      bulk_g2s(smem + S::dO, ws + lay.doi + cidx * lay.vi_bytes(), (uint32_t)lay.vi_bytes(), bar_in);
      bulk_g2s(smem + S::v, ws + lay.vi + cidx * lay.vi_bytes(), (uint32_t)lay.vi_bytes(), bar_in);
      bulk_g2s(smem + S::vn, ws + lay.vni + cidx * lay.vn_bytes(), (uint32_t)lay.vn_bytes(), bar_in);
      bulk_g2s(smem + S::dvn, ws + lay.dvni + cidx * lay.vn_bytes(), (uint32_t)lay.vn_bytes(), bar_in);
    }
    if (tid < 64) {
      sG[tid] = reinterpret_cast<const float*>(ws + lay.gc + cidx * lay.gc_bytes())[tid];
      const int t = t0 + tid;
      sB[tid] = (t < lay.T) ? beta[((size_t)b * lay.T + t) * lay.H + h] : 0.f;
    }
    if (tid < 16) sRed[tid] = reinterpret_cast<const float*>(ws + lay.sl + cidx * 64)[tid];
    ok = mbar_wait(bar_in, r & 1, err, 47);
    block_sync_ok(ok);
    if (!ok) break;
    if (tid == 0) {
      tc_fence_after();
      const Tile tSc{smem_u32(smem + S::sc), DK}, tDO{smem_u32(smem + S::dO), DV}, tV{smem_u32(smem + S::v), 64};
      const Tile tVn{smem_u32(smem + S::vn), 64}, tDVh{smem_u32(smem + S::dvn), 64}, tDVl{smem_u32(smem + S::dvnl), 64};
      mma_tiles(T_DM, 64, 64, DV, tDO, true, 0, 0, tVn, true, 0, false);          // dO Vn^T
      mma_tiles(T_DQA, DK, 64, DV, tSc, false, 0, 0, tDO, false, 0, false);       // S_c dO^T
      mma_tiles(T_DW, DK, 64, DV, tSc, false, 0, 0, tDVh, true, 0, false);        // S_c dVn^T
      mma_tiles(T_Y, DV, 64, 64, tDVh, true, 0, 0, tA, true, 0, false);           // dVn^T A (dVn split)
      mma_tiles(T_Y, DV, 64, 64, tDVl, true, 0, 0, tA, true, 0, true);
      mma_tiles(T_DAV, 64, 64, DV, tDVh, false, 0, 0, tV, true, 0, false);        // dVn V^T
      mma_commit(bar_mma);
    }
    GD_TRACE_AT(ws, lay, 2);
    ok = mbar_wait(bar_mma, ph, err, 41);
    ph ^= 1;
    block_sync_ok(ok);
    if (!ok) break;
    tc_fence_after();
    GD_TRACE_AT(ws, lay, 3);
    // ---------------- phase 2: dS^T images (over S_c / dO / V, whose readers are done), then (Vn dS^T)^T
    if (tid == 0) {
      mbar_arrive_expect_tx(bar_ds, 2 * (uint32_t)lay.si_bytes());
      bulk_g2s(smem + S::dsh, ws + lay.dsi + cidx * 2 * lay.si_bytes(), 2 * (uint32_t)lay.si_bytes(), bar_ds);
      if (mbar_wait(bar_ds, r & 1, err, 48)) {
        const Tile tDh{smem_u32(smem + S::dsh), DK}, tDl{smem_u32(smem + S::dsl), DK};
        const Tile tVh{smem_u32(smem + S::vn), 64}, tVl{smem_u32(smem + S::vnl), 64};
        mma_tiles(T_DKS, DK, 64, DV, tDh, false, 0, 0, tVh, true, 0, false);
        mma_tiles(T_DKS, DK, 64, DV, tDh, false, 0, 0, tVl, true, 0, true);
        mma_tiles(T_DKS, DK, 64, DV, tDl, false, 0, 0, tVh, true, 0, true);
      }
      mma_commit(bar_g2);  // completes after a failed wait too; the error word is already set
    }
    GD_TRACE_AT(ws, lay, 4);
    // epilogue of group 1 while group 2 runs
    float s_last = 0.f;
#pragma unroll
    for (int w = 0; w < 16; ++w) s_last += sRed[w];
    s_last *= __expf(sG[63]);
    {
      float acc[32];
      // dW^T tile (rows dk, cols tokens), dW = -(S_c dVn^T)^T
      tmem_ld32(tmem_lane_addr(T_DW, warp, tok0), acc);
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) acc[jj] = -acc[jj];
#pragma unroll
      for (int q8 = 0; q8 < 4; ++q8) store8_bf16(smem + S::dwt, dcol, tok0 + 8 * q8, 64, acc + 8 * q8);
      // a_t partial: gamma_t q_t . (dO S_c^T)_t over this thread's dk
      tmem_ld32(tmem_lane_addr(T_DQA, warp, tok0), acc);
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) {
        const int i = tok0 + jj;
        acc[jj] *= qhat(i, dcol);
      }
      sPart[(0 * 4 + qd) * 64 + tok0 + lane] = warp_reduce_scatter32(acc);
      // Y = A^T dVn: dV = beta Y (written now) and the (v . Y) partial
      tmem_ld32(tmem_lane_addr(T_Y, warp, tok0), acc);
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) {
        const int i = tok0 + jj, t = t0 + i;
        float vv = 0.f;
        if (t < lay.T) {
          const size_t o = (((size_t)b * lay.T + t) * lay.H + h) * DV + dcol;
          vv = to_f32<T>(vraw[o]);
          dv[o] = from_f32<T>(sB[i] * acc[jj]);
        }
        acc[jj] *= vv;
      }
      sPart[(2 * 4 + qd) * 64 + tok0 + lane] = warp_reduce_scatter32(acc);
    }
    {
      // dM = Gamma * (dO Vn^T) (lower with the diagonal) -> hi / lo tiles
      float acc[32];
      tmem_ld32(tmem_lane_addr(T_DM, warp, tok0), acc);
      if (rowthr) {
        const int i = rrow;
        const float Gi = sG[i];
        float dm[32];
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          const int j = tok0 + jj;
          dm[jj] = (j <= i) ? acc[jj] * __expf(Gi - sG[j]) : 0.f;
        }
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) store8_split(smem + S::dmh, smem + S::dml, i, tok0 + 8 * q8, 64, dm + 8 * q8);
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const Tile tDMh{smem_u32(smem + S::dmh), 64}, tDMl{smem_u32(smem + S::dml), 64}, tDW{smem_u32(smem + S::dwt), 64};
      mma_tiles(T_DQ, DK, 64, 64, tK, true, 0, 0, tDMh, false, 0, false);       // (dM K)^T = K^T dM^T
      mma_tiles(T_DQ, DK, 64, 64, tKl, true, 0, 0, tDMh, false, 0, true);
      mma_tiles(T_DQ, DK, 64, 64, tK, true, 0, 0, tDMl, false, 0, true);
      mma_tiles(T_DKA, DK, 64, 64, tQ, true, 0, 0, tDMh, true, 0, false);       // (dM^T Q)^T = Q^T dM
      mma_tiles(T_DKA, DK, 64, 64, tQl, true, 0, 0, tDMh, true, 0, true);
      mma_tiles(T_DKA, DK, 64, 64, tQ, true, 0, 0, tDMl, true, 0, true);
      mma_tiles(T_X, DK, 64, 64, tDW, true, 0, 0, tA, true, 0, false);          // (A^T dW)^T = dW^T A
      mma_tiles(T_DAK, 64, 64, DK, tDW, false, 0, 0, tK, true, 0, false);       // dW K^T
      mma_commit(bar_mma);
    }
    GD_TRACE_AT(ws, lay, 5);
    ok = mbar_wait(bar_g2, r & 1, err, 42);  // group 2 (one phase per value head)
    if (ok) ok = mbar_wait(bar_mma, ph, err, 43);  // group 3
    ph ^= 1;
    block_sync_ok(ok);
    if (!ok) break;
    tc_fence_after();
    GD_TRACE_AT(ws, lay, 6);
    // ---------------- phase 3: E, k.X partials; dA
    {
      float acc[32], kx[32];
      tmem_ld32(tmem_lane_addr(T_DKS, warp, tok0), acc);
      tmem_ld32(tmem_lane_addr(T_X, warp, tok0), kx);
      const float Glast = sG[63];
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) {
        const int i = tok0 + jj;
        const float kv = qhat(64 + i, dcol);
        acc[jj] *= __expf(Glast - sG[i]) * kv;
        kx[jj] *= kv;
      }
      sPart[(3 * 4 + qd) * 64 + tok0 + lane] = warp_reduce_scatter32(acc);
      sPart[(1 * 4 + qd) * 64 + tok0 + lane] = warp_reduce_scatter32(kx);
      // R = dM * (Q K^T) = (dO Vn^T) * M, strictly lower (M from the prep kernel, fp32, mask included)
      tmem_ld32(tmem_lane_addr(T_DM, warp, tok0), acc);
      if (rowthr) {
        const int i = rrow;
        const float* mrow = reinterpret_cast<const float*>(ws + lay.mf + cidx * lay.cc_bytes()) + i * 64 + tok0;
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          const int j = tok0 + jj;
          sR[cc_idx(i, j)] = (j < i) ? acc[jj] * mrow[jj] : 0.f;
        }
      }
      // dA = strict_lower(beta_j gamma_j (dW K^T) + beta_j (dVn V^T)) -> bf16 tile
      float ak[32], av[32];
      tmem_ld32(tmem_lane_addr(T_DAK, warp, tok0), ak);
      tmem_ld32(tmem_lane_addr(T_DAV, warp, tok0), av);
      if (rowthr) {
        const int i = rrow;
        float da[32];
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          const int j = tok0 + jj;
          da[jj] = (j < i) ? sB[j] * fmaf(__expf(sG[j]), ak[jj], av[jj]) : 0.f;
        }
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) store8_bf16(smem + S::da, i, tok0 + 8 * q8, 64, da + 8 * q8);
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      mma_tiles(T_T1, 64, 64, 64, Tile{smem_u32(smem + S::da), 64}, true, 0, 0, tA, false, 0, false);  // dA A^T
      mma_commit(bar_mma);
    }
    GD_TRACE_AT(ws, lay, 7);
    ok = mbar_wait(bar_mma, ph, err, 44);
    ph ^= 1;
    block_sync_ok(ok);
    if (!ok) break;
    tc_fence_after();
    {
      float acc[32];
      tmem_ld32(tmem_lane_addr(T_T1, warp, tok0), acc);
      if (rowthr) {
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) store8_bf16(smem + S::t1, rrow, tok0 + 8 * q8, 64, acc + 8 * q8);
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      mma_tiles(T_DL, 64, 64, 64, tA, false, 0, 0, Tile{smem_u32(smem + S::t1), 64}, true, 0, false);  // A^T T1
      mma_commit(bar_mma);
    }
    GD_TRACE_AT(ws, lay, 8);
    ok = mbar_wait(bar_mma, ph, err, 45);
    ph ^= 1;
    block_sync_ok(ok);
    if (!ok) break;
    tc_fence_after();
    {
      // dL = -(A^T T1), strictly lower; L = beta_i KG_ij Gamma_ij; R += dL L; P = dL Gamma; P_beta = beta_i P
      float acc[32];
      float* sPB = reinterpret_cast<float*>(smem + S::pb);
      tmem_ld32(tmem_lane_addr(T_DL, warp, tok0), acc);
      if (rowthr) {
        const int i = rrow;
        const float Gi = sG[i], bi = sB[i];
        const float* kgrow = reinterpret_cast<const float*>(ws + lay.kg + cidx * lay.cc_bytes()) + i * 64 + tok0;
        float pk = 0.f;
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          const int j = tok0 + jj;
          const int ci = cc_idx(i, j);
          float pb = 0.f;
          if (j < i) {
            const float dl = -acc[jj];
            const float gam = __expf(Gi - sG[j]);
            const float kg = kgrow[jj];
            const float P = dl * gam;
            sR[ci] += dl * bi * kg * gam;
            pk = fmaf(P, kg, pk);
            pb = bi * P;
          }
          sPB[ci] = pb;
        }
        sPk[half * 64 + i] = pk;
      }
    }
    __syncthreads();
    {
      // Z = P_beta + P_beta^T -> bf16 tile (rows i, cols j)
      const float* sPB = reinterpret_cast<const float*>(smem + S::pb);
      for (int idx = tid; idx < 64 * 8; idx += 256) {
        const int rl = idx & 7, cb = (idx >> 3) & 7, rb = idx >> 6;
        const int i = 8 * rb + rl;
        float zz[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int j = 8 * cb + e;
          zz[e] = sPB[cc_idx(i, j)] + sPB[cc_idx(j, i)];
        }
        store8_bf16(smem + S::z, i, 8 * cb, 64, zz);
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      mma_tiles(T_DKC, DK, 64, 64, tK, true, 0, 0, Tile{smem_u32(smem + S::z), 64}, false, 0, false);  // K^T Z^T
      mma_commit(bar_mma);
    }
    GD_TRACE_AT(ws, lay, 9);
    // rect_t = sum_{i >= t} sum_{j < t} R_ij while the tensor core works: row prefixes in place, then column suffixes
    if (tid < 64) {
      const int i = tid;
      float run = 0.f;
      for (int j = 0; j < 64; ++j) {
        const int ci = cc_idx(i, j);
        const float x = sR[ci];
        sR[ci] = run;  // sum_{j' < j} R_ij'
        run += x;
      }
    }
    ok = mbar_wait(bar_mma, ph, err, 46);
    ph ^= 1;
    block_sync_ok(ok);
    if (!ok) break;
    tc_fence_after();
    GD_TRACE_AT(ws, lay, 10);
    // ---------------- phase 4: dQ, dK of this value head; dg and dbeta
    {
      float a[32], bq[32];
      tmem_ld32(tmem_lane_addr(T_DQA, warp, tok0), a);
      tmem_ld32(tmem_lane_addr(T_DQ, warp, tok0), bq);
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) dQacc[jj] += fmaf(__expf(sG[tok0 + jj]), a[jj], bq[jj]);
      float ka[32], ks[32];
      tmem_ld32(tmem_lane_addr(T_DKA, warp, tok0), ka);
      tmem_ld32(tmem_lane_addr(T_DKS, warp, tok0), ks);
      const float Glast = sG[63];
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) dKacc[jj] += fmaf(__expf(Glast - sG[tok0 + jj]), ks[jj], ka[jj]);
      tmem_ld32(tmem_lane_addr(T_X, warp, tok0), ka);
      tmem_ld32(tmem_lane_addr(T_DKC, warp, tok0), ks);
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) {
        const int i = tok0 + jj;
        dKacc[jj] += fmaf(sB[i] * __expf(sG[i]), ka[jj], ks[jj]);
      }
    }
    if (tid < 64) {
      const int t = tid;
      float rect = 0.f;
      for (int i = t; i < 64; ++i) rect += sR[cc_idx(i, t)];
      const float a = __expf(sG[t]) * (sPart[(0 * 4 + 0) * 64 + t] + sPart[(0 * 4 + 1) * 64 + t] +
                                        sPart[(0 * 4 + 2) * 64 + t] + sPart[(0 * 4 + 3) * 64 + t]);
      const float kx = sPart[(1 * 4 + 0) * 64 + t] + sPart[(1 * 4 + 1) * 64 + t] + sPart[(1 * 4 + 2) * 64 + t] +
                       sPart[(1 * 4 + 3) * 64 + t];
      const float vy = sPart[(2 * 4 + 0) * 64 + t] + sPart[(2 * 4 + 1) * 64 + t] + sPart[(2 * 4 + 2) * 64 + t] +
                       sPart[(2 * 4 + 3) * 64 + t];
      const float E = sPart[(3 * 4 + 0) * 64 + t] + sPart[(3 * 4 + 1) * 64 + t] + sPart[(3 * 4 + 2) * 64 + t] +
                      sPart[(3 * 4 + 3) * 64 + t];
      const float gt = __expf(sG[t]);
      const float w = sB[t] * gt * kx;
      const float db = gt * kx + vy + sPk[t] + sPk[64 + t];
      // suffix sum of (a + w) over the chunk (64 tokens in two warps), exclusive prefix of E
      float aw = a + w;
      float suf = aw, pre = E;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_down_sync(0xffffffffu, suf, o);
        if (lane + o < 32) suf += y;
        const float z = __shfl_up_sync(0xffffffffu, pre, o);
        if (lane >= o) pre += z;
      }
      // combine the two warps: warp 0 adds warp 1's total suffix; warp 1 adds warp 0's total prefix. The exclusive
      // prefix is the inclusive one shifted by a lane (never inclusive minus E: that would cancel)
      if (lane == 0 && warp == 1) sPart[4 * 4 * 64 + 0] = suf;   // warp 1's full sum of (a + w)
      if (lane == 31 && warp == 0) sPart[4 * 4 * 64 + 1] = pre;  // warp 0's full sum of E
      float pre_excl = __shfl_up_sync(0xffffffffu, pre, 1);
      if (lane == 0) pre_excl = 0.f;
      asm volatile("bar.sync 1, 64;" ::: "memory");
      if (warp == 0) suf += sPart[4 * 4 * 64 + 0];
      if (warp == 1) pre_excl += sPart[4 * 4 * 64 + 1];
      const float dgt = suf + s_last + pre_excl + rect;
      const int tt = t0 + t;
      if (tt < lay.T) {
        dg[((size_t)b * lay.T + tt) * lay.H + h] = dgt;
        dbeta[((size_t)b * lay.T + tt) * lay.H + h] = db;
      }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }
  if (ok) {
    // l2 prologue backward (src/macai/gated_delta/_norm.py:6-9): dx = scale r (dy - x_hat (x_hat . dy))
    float xq[32], xk[32], pq[32], pk_[32];
    float rq[32], rk[32];
#pragma unroll
    for (int jj = 0; jj < 32; ++jj) {
      const int t = t0 + tok0 + jj;
      const bool valid = t < lay.T;
      const size_t o = (((size_t)b * lay.T + (valid ? t : 0)) * lay.HK + hk) * DK + dcol;
      const size_t ro = ((size_t)b * lay.T + (valid ? t : 0)) * lay.HK + hk;
      rq[jj] = (norm && valid) ? reinterpret_cast<const float*>(ws + lay.rq)[ro] : 1.f;
      rk[jj] = (norm && valid) ? reinterpret_cast<const float*>(ws + lay.rk)[ro] : 1.f;
      xq[jj] = valid ? to_f32<T>(qraw[o]) * rq[jj] : 0.f;
      xk[jj] = valid ? to_f32<T>(kraw[o]) * rk[jj] : 0.f;
      pq[jj] = xq[jj] * dQacc[jj];
      pk_[jj] = xk[jj] * dKacc[jj];
    }
    float* sDot = sPart;  // reuse: [2][4][64]
    __syncthreads();
    sDot[(0 * 4 + qd) * 64 + tok0 + lane] = warp_reduce_scatter32(pq);
    sDot[(1 * 4 + qd) * 64 + tok0 + lane] = warp_reduce_scatter32(pk_);
    __syncthreads();
#pragma unroll
    for (int jj = 0; jj < 32; ++jj) {
      const int i = tok0 + jj, t = t0 + i;
      if (t < lay.T) {
        const size_t o = (((size_t)b * lay.T + t) * lay.HK + hk) * DK + dcol;
        float gq, gk;
        if (norm) {
          const float dotq = sDot[0 * 64 + i] + sDot[1 * 64 + i] + sDot[2 * 64 + i] + sDot[3 * 64 + i];
          const float dotk = sDot[4 * 64 + i] + sDot[5 * 64 + i] + sDot[6 * 64 + i] + sDot[7 * 64 + i];
          gq = qscale * rq[jj] * (dQacc[jj] - xq[jj] * dotq);
          gk = rk[jj] * (dKacc[jj] - xk[jj] * dotk);
        } else {
          gq = qscale * dQacc[jj];
          gk = dKacc[jj];
        }
        dq[o] = from_f32<T>(gq);
        dk[o] = from_f32<T>(gk);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tm, 512);
  }
}

template <typename T, int DK, int DV>
cudaError_t launch_bwd_chunk(const void* q, const void* k, const void* v, const float* beta, const void* d_o, void* dq,
                             void* dk, void* dv, float* dg, float* dbeta, const Layout& lay, int flags,
                             unsigned char* ws, cudaStream_t st) {
  using S = ChunkSmem<DK, DV>;
  auto kern = bwd_chunk_kernel<T, DK, DV>;
  static bool attr_done[kMaxDevices] = {};  // once per device: no attribute call inside a graph capture
  cudaError_t e = set_smem_once(kern, S::total, attr_done);
  if (e != cudaSuccess) return e;
  dim3 grid(lay.NT, lay.HK, lay.B);
  kern<<<grid, 256, S::total, st>>>(static_cast<const T*>(q), static_cast<const T*>(k), static_cast<const T*>(v), beta,
                                    static_cast<const T*>(d_o), static_cast<T*>(dq), static_cast<T*>(dk),
                                    static_cast<T*>(dv), dg, dbeta, lay, flags, ws);
  return cudaGetLastError();
}

#define INST(T)                                                                                                     \
  template cudaError_t launch_bwd_chunk<T, 128, 128>(const void*, const void*, const void*, const float*,          \
                                                     const void*, void*, void*, void*, float*, float*, const Layout&, \
                                                     int, unsigned char*, cudaStream_t);
INST(__nv_bfloat16)
INST(__half)
INST(float)
#undef INST

}  // namespace gd
