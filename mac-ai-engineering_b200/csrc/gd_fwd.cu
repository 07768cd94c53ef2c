// Forward kernels of the chunked gated delta rule on B200 (sm_100a):
//   prep_kernel   one CTA per (chunk, value head, batch row): l2 prologue, cumulative decay, the chunk's C x C products
//                 on tcgen05, the unit-lower-triangular inverse, W and U;
//   state_kernel  one CTA per (value head, batch row): the sequential chunk pass with the state in registers (fp32) and
//                 every product on tcgen05 from shared memory, chunk inputs streamed in by the bulk-copy engine.
// Equations (per chunk; src/macai/gated_delta/_chunked.py:1-35, tools/check_chunk_equations.py:29-46 of the reference):
//   G = cumsum(g), gamma = exp(G), e = exp(G_last - G)
//   L = diag(beta) (K K^T) * exp(G_i - G_j) (i > j),  M = (Q K^T) * exp(G_i - G_j) (i >= j),  A = (I + L)^-1
//   W = A diag(beta gamma) K,  U = A diag(beta) V
//   Vn = U - W S,  O = diag(gamma) Q S + M Vn,  S <- exp(G_last) S + K^T diag(e) Vn
// Precision: bf16 operands with fp32 accumulation; A diag(beta) (in U), Vn (in M Vn) and e * Vn (in the state update)
// are split into bf16 hi + lo pairs (two MMAs into one accumulator), the state is carried in fp32.
#include "gd_common.cuh"
#include "gd_layout.cuh"

namespace gd {

// ------------------------------------------------------------------------------------------------------------------
// prep

template <int DK, int DV>
struct PrepSmem {
  static constexpr size_t q = 0;                          // [64 x DK] bf16 blocked, normalised q (scaled)
  static constexpr size_t k = q + 64 * DK * 2;            // [64 x DK], directly after q: [Q; K] is one [128 x DK] tile
  static constexpr size_t v = k + 64 * DK * 2;            // [64 x DV]
  static constexpr size_t a1 = v + 64 * DV * 2;           // [64 x 64] A diag(beta gamma)
  static constexpr size_t a2h = a1 + 64 * 64 * 2;         // [64 x 64] A diag(beta), hi
  static constexpr size_t a2l = a2h + 64 * 64 * 2;        //                           lo
  static constexpr size_t L = a2l + 64 * 64 * 2;          // [64][65] fp32, L (strictly lower)
  static constexpr size_t Ai = L + 64 * 65 * 4;           // [64][65] fp32, A
  static constexpr size_t ql = L;                         // [64 x DK] low half of q, then k: live only until the
  static constexpr size_t kl = ql + 64 * DK * 2;          //   Q K^T / K K^T product is done (L and A reuse them)
  static_assert(2 * 64 * DK * 2 <= 2 * 64 * 65 * 4, "the q / k low halves must fit in the L and A buffers");
  static constexpr size_t T3 = Ai + 64 * 65 * 4;          // [3][16][17] fp32 block products of the inverse
  static constexpr size_t G = T3 + 3 * 16 * 17 * 4;       // [64] cumulative log decay
  static constexpr size_t beta = G + 64 * 4;              // [64]
  static constexpr size_t scan = beta + 64 * 4;           // [2] warp totals of the scan
  static constexpr size_t bar = (scan + 16 + 7) & ~size_t(7);
  static constexpr size_t tmem = bar + 8;
  static constexpr size_t total = tmem + 16;
};

// A = (I + L)^-1 for the 64 x 64 strictly lower L (fp32, row stride 65), by substitution inside the four 16 x 16
// diagonal blocks and block merges below them, A_IJ = -A_II sum_{m=J}^{I-1} L_Im A_mJ (one block distance at a time),
// as in the reference's gdc_prep (src/macai/gated_delta/_chunked.py:282-311) with 16-row blocks. 128 threads.
__device__ __forceinline__ void unit_lower_inverse(const float* L, float* A, float* T3) {
  const int tid = threadIdx.x;
  // zero the strictly upper blocks (and everything, so the blocks below are written over a clean slate)
  for (int idx = tid; idx < 64 * 64; idx += 128) {
    const int i = idx >> 6, j = idx & 63;
    if ((i >> 4) < (j >> 4)) A[i * 65 + j] = 0.f;
  }
  if (tid < 64) {
    const int blk = tid >> 4, col = tid & 15, o = 16 * blk;
    float x[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      float s = (r == col) ? 1.f : 0.f;
      if (r > col) {
#pragma unroll
        for (int m = 0; m < 16; ++m)
          if (m >= col && m < r) s = fmaf(-L[(o + r) * 65 + o + m], x[m], s);
      }
      x[r] = s;
    }
#pragma unroll
    for (int r = 0; r < 16; ++r) A[(o + r) * 65 + o + col] = x[r];
  }
  __syncthreads();
  for (int d = 1; d < 4; ++d) {
    const int npairs = 4 - d;  // pairs (I, J) = (J + d, J), J = 0 .. npairs-1
    // T_IJ = sum_{m=J}^{I-1} L_Im A_mJ
    for (int idx = tid; idx < npairs * 256; idx += 128) {
      const int p = idx >> 8, r = (idx >> 4) & 15, s = idx & 15;
      const int J = p, I = p + d;
      float acc = 0.f;
      for (int m = J; m < I; ++m) {
#pragma unroll
        for (int u = 0; u < 16; ++u) acc = fmaf(L[(16 * I + r) * 65 + 16 * m + u], A[(16 * m + u) * 65 + 16 * J + s], acc);
      }
      T3[p * 16 * 17 + r * 17 + s] = acc;
    }
    __syncthreads();
    // A_IJ = -A_II T_IJ (A_II unit lower)
    for (int idx = tid; idx < npairs * 256; idx += 128) {
      const int p = idx >> 8, r = (idx >> 4) & 15, s = idx & 15;
      const int J = p, I = p + d;
      float acc = T3[p * 16 * 17 + r * 17 + s];
      for (int u = 0; u < r; ++u) acc = fmaf(A[(16 * I + r) * 65 + 16 * I + u], T3[p * 16 * 17 + u * 17 + s], acc);
      A[(16 * I + r) * 65 + 16 * J + s] = -acc;
    }
    __syncthreads();
  }
}

template <typename T, int DK, int DV>
__global__ void __launch_bounds__(128) prep_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                   const T* __restrict__ v, const float* __restrict__ g,
                                                   const float* __restrict__ beta, Layout lay, int flags,
                                                   unsigned char* __restrict__ ws) {
  using S = PrepSmem<DK, DV>;
  extern __shared__ __align__(1024) unsigned char smem[];
  ErrorWord* err = reinterpret_cast<ErrorWord*>(ws + lay.err);
  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / lay.rep;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = c * C;
  const size_t cidx = ((size_t)b * lay.H + h) * lay.NT + c;
  float* sL = reinterpret_cast<float*>(smem + S::L);
  float* sAi = reinterpret_cast<float*>(smem + S::Ai);
  float* sG = reinterpret_cast<float*>(smem + S::G);
  float* sB = reinterpret_cast<float*>(smem + S::beta);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + S::bar);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + S::tmem);

  if (warp == 0) {
    tmem_alloc(tslot, 256);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }

  // l2 prologue and operand tiles
  const bool norm = (flags & GD_L2NORM) != 0;
  const bool bwd = lay.backward() && (h % lay.rep == 0);
  float* rq = bwd ? reinterpret_cast<float*>(ws + lay.rq) : nullptr;
  float* rk = bwd ? reinterpret_cast<float*>(ws + lay.rk) : nullptr;
  const float qscale = (flags & GD_SCALE_Q) ? rsqrtf((float)DK) : 1.f;
  load_rows<T, DK>(q, b, t0, lay.T, lay.HK, hk, norm, qscale, smem + S::q, rq, smem + S::ql);
  load_rows<T, DK>(k, b, t0, lay.T, lay.HK, hk, norm, 1.f, smem + S::k, rk, smem + S::kl);
  load_rows<T, DV>(v, b, t0, lay.T, lay.H, h, false, 1.f, smem + S::v, nullptr);

  // cumulative log decay (padding rows: g = 0, beta = 0, which leaves G constant past the last token)
  if (tid < 64) {
    const int t = t0 + tid;
    float gi = 0.f, bi = 0.f;
    if (t < lay.T) {
      gi = g[((size_t)b * lay.T + t) * lay.H + h];
      bi = beta[((size_t)b * lay.T + t) * lay.H + h];
    }
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, gi, o);
      if (lane >= o) gi += y;
    }
    float* scan = reinterpret_cast<float*>(smem + S::scan);
    if (lane == 31) scan[warp] = gi;
    sB[tid] = bi;
    sG[tid] = gi;  // warp 1 adds warp 0's total below
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  if (tid >= 32 && tid < 64) sG[tid] += reinterpret_cast<float*>(smem + S::scan)[0];
  tc_fence_after();
  const uint32_t tm = *tslot;

  // [Q; K] K^T with q and k carried as bf16 hi + lo (three products): lanes 0-63 hold Q K^T rows, 64-127 K K^T rows
  if (tid == 0) {
    const Tile qkh{smem_u32(smem + S::q), DK}, qkl{smem_u32(smem + S::ql), DK};
    const Tile kh{smem_u32(smem + S::k), DK}, kl{smem_u32(smem + S::kl), DK};
    mma_tiles(tm, 128, 64, DK, qkh, true, 0, 0, kh, false, 0, false);
    mma_tiles(tm, 128, 64, DK, qkh, true, 0, 0, kl, false, 0, true);
    mma_tiles(tm, 128, 64, DK, qkl, true, 0, 0, kh, false, 0, true);
    mma_commit(bar);
  }
  __syncthreads();  // sG complete for everyone
  {  // the low halves go out before L and A overwrite them
    const uint4* src = reinterpret_cast<const uint4*>(smem + S::ql);
    uint4* dst = reinterpret_cast<uint4*>(ws + lay.qkl + cidx * lay.qk_bytes());
    for (int idx = tid; idx < (int)(lay.qk_bytes() / 16); idx += 128) dst[idx] = src[idx];
  }
  bool ok = mbar_wait(bar, 0, err, 10);
  ok = __syncthreads_and(ok);
  tc_fence_after();
  if (ok) {
    const int i = tid & 63;
    const float Gi = sG[i];
    float acc[32];
    unsigned char* mimg = ws + lay.m + cidx * lay.m_bytes();
    float* mf = lay.backward() ? reinterpret_cast<float*>(ws + lay.mf + cidx * lay.ainv_bytes()) + i * 64 : nullptr;
    float* kgf = lay.backward() ? reinterpret_cast<float*>(ws + lay.kg + cidx * lay.ainv_bytes()) + i * 64 : nullptr;
#pragma unroll 1
    for (int half = 0; half < 2; ++half) {
      tmem_ld32(tmem_lane_addr(tm, warp, 32 * half), acc);
      if (tid < 64) {
        float mv[32];
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          const int j = 32 * half + jj;
          mv[jj] = (j <= i) ? acc[jj] * __expf(Gi - sG[j]) : 0.f;
        }
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) store8_bf16(mimg, i, 32 * half + 8 * q8, 64, mv + 8 * q8);
        if (mf != nullptr) {
#pragma unroll
          for (int q8 = 0; q8 < 4; ++q8) store8<float>(mf + 32 * half + 8 * q8, mv + 8 * q8);
        }
      } else {
        const float bi = sB[i];
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          const int j = 32 * half + jj;
          sL[i * 65 + j] = (j < i) ? bi * acc[jj] * __expf(Gi - sG[j]) : 0.f;
        }
        if (kgf != nullptr) {
#pragma unroll
          for (int q8 = 0; q8 < 4; ++q8) store8<float>(kgf + 32 * half + 8 * q8, acc + 8 * q8);
        }
      }
    }
  }
  __syncthreads();
  if (ok) unit_lower_inverse(sL, sAi, reinterpret_cast<float*>(smem + S::T3));

  if (ok) {
    // A diag(beta gamma) and the hi/lo split of A diag(beta) as K-major B operands (rows i, cols j)
    const int i = tid >> 1, j0 = 32 * (tid & 1);
#pragma unroll 1
    for (int q8 = 0; q8 < 4; ++q8) {
      float a1[8], a2[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int j = j0 + 8 * q8 + e;
        const float a = sAi[i * 65 + j];
        a1[e] = a * sB[j] * __expf(sG[j]);
        a2[e] = a * sB[j];
      }
      store8_bf16(smem + S::a1, i, j0 + 8 * q8, 64, a1);
      store8_split(smem + S::a2h, smem + S::a2l, i, j0 + 8 * q8, 64, a2);
    }
    if (lay.backward()) {
      float* ainv = reinterpret_cast<float*>(ws + lay.ainv + cidx * lay.ainv_bytes());
      for (int idx = tid; idx < 64 * 64; idx += 128) ainv[idx] = sAi[(idx >> 6) * 65 + (idx & 63)];
    }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (ok && tid == 0) {
    // W^T [DK x 64] = K^T (A diag(beta gamma))^T ; U^T [DV x 64] = V^T (A diag(beta))^T (hi + lo)
    mma_tiles(tm + 64, DK, 64, 64, Tile{smem_u32(smem + S::k), DK}, false, 0, 0, Tile{smem_u32(smem + S::a1), 64},
              false, 0, false);
    mma_tiles(tm + 128, DV, 64, 64, Tile{smem_u32(smem + S::v), DV}, false, 0, 0, Tile{smem_u32(smem + S::a2h), 64},
              false, 0, false);
    mma_tiles(tm + 128, DV, 64, 64, Tile{smem_u32(smem + S::v), DV}, false, 0, 0, Tile{smem_u32(smem + S::a2l), 64},
              false, 0, true);
    mma_commit(bar);
  }
  // the q / k images and G go out while the MMAs run
  if (ok) {
    const uint4* src = reinterpret_cast<const uint4*>(smem + S::q);
    uint4* dst = reinterpret_cast<uint4*>(ws + lay.qk + cidx * lay.qk_bytes());
    for (int idx = tid; idx < (int)(lay.qk_bytes() / 16); idx += 128) dst[idx] = src[idx];
    if (tid < 64) reinterpret_cast<float*>(ws + lay.gc + cidx * lay.gc_bytes())[tid] = sG[tid];
  }
  if (ok) ok = mbar_wait(bar, 1, err, 11);
  ok = __syncthreads_and(ok);
  tc_fence_after();
  if (ok) {
    float acc[32];
    // W^T row dk = tid -> blocked [DK x 64] image, 16-byte stores
    unsigned char* wimg = ws + lay.wt + cidx * lay.wt_bytes();
    if (tid < DK) {
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        tmem_ld32(tmem_lane_addr(tm, warp, 64 + 32 * half), acc);
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) store8_bf16(wimg, tid, 32 * half + 8 * q8, 64, acc + 8 * q8);
      }
    }
    // U^T row v = tid -> U [64][DV] fp32
    float* u = reinterpret_cast<float*>(ws + lay.u + cidx * lay.u_bytes());
    if (tid < DV) {
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        tmem_ld32(tmem_lane_addr(tm, warp, 128 + 32 * half), acc);
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) u[(32 * half + jj) * DV + tid] = acc[jj];
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tm, 256);
  }
}

// ------------------------------------------------------------------------------------------------------------------
// forward state pass

template <int DK, int DV>
struct StateSmem {
  static constexpr size_t st = 0;                        // [DV x DK] bf16 blocked, S^T (rows v, cols dk)
  static constexpr size_t vh = st + DV * DK * 2;         // [DV x 64] Vn^T hi
  static constexpr size_t vl = vh + DV * 64 * 2;         //            lo
  static constexpr size_t eh = vl + DV * 64 * 2;         // [DV x 64] (e Vn)^T hi
  static constexpr size_t el = eh + DV * 64 * 2;         //               lo
  static constexpr size_t qk = el + DV * 64 * 2;         // stage: [2][64 x DK] q, k images
  static constexpr size_t kl = qk + 2 * 64 * DK * 2;     // stage: [64 x DK] low half of the k image
  static constexpr size_t wt = kl + 64 * DK * 2;         // stage: [DK x 64] W^T image
  static constexpr size_t m = wt + DK * 64 * 2;          // stage: [64 x 64] M image
  static constexpr size_t g = m + 64 * 64 * 2;           // stage: [64] G
  static constexpr size_t u = g + 64 * 4;                // [64][DV] fp32 U
  static constexpr size_t bar = u + 64 * DV * 4;         // 3 mbarriers: mma, inputs, U
  static constexpr size_t tmem = bar + 3 * 8;
  static constexpr size_t total = tmem + 8;
  static constexpr uint32_t stage_bytes = 3 * 64 * DK * 2 + DK * 64 * 2 + 64 * 64 * 2 + 64 * 4;
};

template <int DK, int DV>
__device__ __forceinline__ void issue_stage(unsigned char* smem, const unsigned char* ws, const Layout& lay,
                                            size_t cidx, uint64_t* bar) {
  using S = StateSmem<DK, DV>;
  mbar_arrive_expect_tx(bar, S::stage_bytes);
  bulk_g2s(smem + S::qk, ws + lay.qk + cidx * lay.qk_bytes(), (uint32_t)lay.qk_bytes(), bar);
  bulk_g2s(smem + S::kl, ws + lay.qkl + cidx * lay.qk_bytes() + 64 * DK * 2, 64 * DK * 2, bar);
  bulk_g2s(smem + S::wt, ws + lay.wt + cidx * lay.wt_bytes(), (uint32_t)lay.wt_bytes(), bar);
  bulk_g2s(smem + S::m, ws + lay.m + cidx * lay.m_bytes(), (uint32_t)lay.m_bytes(), bar);
  bulk_g2s(smem + S::g, ws + lay.gc + cidx * lay.gc_bytes(), (uint32_t)lay.gc_bytes(), bar);
}

template <typename T, int DK, int DV>
__global__ void __launch_bounds__(128) state_kernel(const float* __restrict__ s0, T* __restrict__ o,
                                                    float* __restrict__ sT, Layout lay, int flags,
                                                    unsigned char* __restrict__ ws) {
  static_assert(DV == 128, "the state pass maps one thread to each of 128 value columns");
  using S = StateSmem<DK, DV>;
  extern __shared__ __align__(1024) unsigned char smem[];
  ErrorWord* err = reinterpret_cast<ErrorWord*>(ws + lay.err);
  const int h = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int vcol = tid;  // this thread's value column (TMEM lane of every M = 128 accumulator)
  uint64_t* bar_mma = reinterpret_cast<uint64_t*>(smem + S::bar);
  uint64_t* bar_in = bar_mma + 1;
  uint64_t* bar_u = bar_mma + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + S::tmem);
  const float* sG = reinterpret_cast<const float*>(smem + S::g);
  const float* sU = reinterpret_cast<const float*>(smem + S::u);
  const bool store = (flags & GD_STORE_STATES) != 0 && lay.backward();
  const size_t row0 = ((size_t)b * lay.H + h) * lay.NT;  // chunk index of chunk 0

  if (warp == 0) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(bar_mma, 1);
    mbar_init(bar_in, 1);
    mbar_init(bar_u, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) {
    issue_stage<DK, DV>(smem, ws, lay, row0, bar_in);
    mbar_arrive_expect_tx(bar_u, (uint32_t)lay.u_bytes());
    bulk_g2s(smem + S::u, ws + lay.u + row0 * lay.u_bytes(), (uint32_t)lay.u_bytes(), bar_u);
  }

  float Sreg[DK];  // column vcol of S (all key rows), fp32
  {
    const float* s0p = s0 ? s0 + ((size_t)b * lay.H + h) * DK * DV : nullptr;
#pragma unroll
    for (int d = 0; d < DK; ++d) Sreg[d] = s0p ? s0p[(size_t)d * DV + vcol] : 0.f;
#pragma unroll
    for (int d8 = 0; d8 < DK / 8; ++d8) store8_bf16(smem + S::st, vcol, 8 * d8, DK, Sreg + 8 * d8);
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = *tslot;
  const uint32_t tWS = tm + 0, tQS = tm + 64, tMV = tm + 128, tDS = tm + 256;

  uint32_t ph_mma = 0, ph_in = 0, ph_u = 0;
  bool ok = true;
  for (int c = 0; c < lay.NT && ok; ++c) {
    const size_t cidx = row0 + c;
    const int t0 = c * C;
    ok = mbar_wait(bar_in, ph_in, err, 20);
    ph_in ^= 1;
    ok = __syncthreads_and(ok);
    if (!ok) break;
    if (tid == 0) {
      tc_fence_after();
      // (W S)^T = S^T W^T  and  (Q S)^T = S^T Q^T : [DV x 64]
      mma_tiles(tWS, DV, 64, DK, Tile{smem_u32(smem + S::st), DK}, true, 0, 0, Tile{smem_u32(smem + S::wt), 64}, true,
                0, false);
      mma_tiles(tQS, DV, 64, DK, Tile{smem_u32(smem + S::st), DK}, true, 0, 0, Tile{smem_u32(smem + S::qk), DK},
                false, 0, false);
      mma_commit(bar_mma);
    }
    ok = mbar_wait(bar_mma, ph_mma, err, 21);
    ph_mma ^= 1;
    if (ok) ok = mbar_wait(bar_u, ph_u, err, 22);
    ph_u ^= 1;
    ok = __syncthreads_and(ok);
    if (!ok) break;
    tc_fence_after();
    const float Glast = sG[63];
    {
      float acc[32];
      float* vn_out = store ? reinterpret_cast<float*>(ws + lay.vn + cidx * lay.u_bytes()) : nullptr;
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        tmem_ld32(tmem_lane_addr(tWS, warp, 32 * half), acc);
        float vn[32], ev[32];
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          const int i = 32 * half + jj;
          vn[jj] = sU[i * DV + vcol] - acc[jj];
          ev[jj] = vn[jj] * __expf(Glast - sG[i]);
          if (store) vn_out[i * DV + vcol] = vn[jj];
        }
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {
          store8_split(smem + S::vh, smem + S::vl, vcol, 32 * half + 8 * q8, 64, vn + 8 * q8);
          store8_split(smem + S::eh, smem + S::el, vcol, 32 * half + 8 * q8, 64, ev + 8 * q8);
        }
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      if (c + 1 < lay.NT) {  // U is consumed: stream in the next chunk's
        mbar_arrive_expect_tx(bar_u, (uint32_t)lay.u_bytes());
        bulk_g2s(smem + S::u, ws + lay.u + (cidx + 1) * lay.u_bytes(), (uint32_t)lay.u_bytes(), bar_u);
      }
      // (M Vn)^T = Vn^T M^T  [DV x 64];  (K^T e Vn)^T = (e Vn)^T K  [DV x DK]
      mma_tiles(tMV, DV, 64, 64, Tile{smem_u32(smem + S::vh), 64}, true, 0, 0, Tile{smem_u32(smem + S::m), 64}, false,
                0, false);
      mma_tiles(tMV, DV, 64, 64, Tile{smem_u32(smem + S::vl), 64}, true, 0, 0, Tile{smem_u32(smem + S::m), 64}, false,
                0, true);
      // e Vn and k both split: hi hi + hi lo + lo hi (the state carries the sequence: it gets the extra bits)
      const Tile tkh{smem_u32(smem + S::qk + 64 * DK * 2), DK}, tkl{smem_u32(smem + S::kl), DK};
      mma_tiles(tDS, DV, DK, 64, Tile{smem_u32(smem + S::eh), 64}, true, 0, 0, tkh, true, 0, false);
      mma_tiles(tDS, DV, DK, 64, Tile{smem_u32(smem + S::eh), 64}, true, 0, 0, tkl, true, 0, true);
      mma_tiles(tDS, DV, DK, 64, Tile{smem_u32(smem + S::el), 64}, true, 0, 0, tkh, true, 0, true);
      mma_commit(bar_mma);
    }
    ok = mbar_wait(bar_mma, ph_mma, err, 23);
    ph_mma ^= 1;
    ok = __syncthreads_and(ok);
    if (!ok) break;
    tc_fence_after();
    {
      float qs[32], mv[32];
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        tmem_ld32(tmem_lane_addr(tQS, warp, 32 * half), qs);
        tmem_ld32(tmem_lane_addr(tMV, warp, 32 * half), mv);
        if (o != nullptr) {
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) {
            const int i = 32 * half + jj;
            const int t = t0 + i;
            if (t < lay.T) o[(((size_t)b * lay.T + t) * lay.H + h) * DV + vcol] = from_f32<T>(__expf(sG[i]) * qs[jj] + mv[jj]);
          }
        }
      }
      if (store) {
        float* sc = reinterpret_cast<float*>(ws + lay.sc + cidx * lay.s_bytes());
#pragma unroll
        for (int d = 0; d < DK; ++d) sc[(size_t)d * DV + vcol] = Sreg[d];
      }
      const float gl = __expf(Glast);
      float ds[32];
#pragma unroll
      for (int q4 = 0; q4 < DK / 32; ++q4) {
        tmem_ld32(tmem_lane_addr(tDS, warp, 32 * q4), ds);
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) Sreg[32 * q4 + jj] = fmaf(gl, Sreg[32 * q4 + jj], ds[jj]);
      }
#pragma unroll
      for (int d8 = 0; d8 < DK / 8; ++d8) store8_bf16(smem + S::st, vcol, 8 * d8, DK, Sreg + 8 * d8);
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0 && c + 1 < lay.NT) issue_stage<DK, DV>(smem, ws, lay, cidx + 1, bar_in);
  }
  if (ok && sT != nullptr) {
    float* sp = sT + ((size_t)b * lay.H + h) * DK * DV;
#pragma unroll
    for (int d = 0; d < DK; ++d) sp[(size_t)d * DV + vcol] = Sreg[d];
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tm, 512);
  }
}

// ------------------------------------------------------------------------------------------------------------------
// launchers

template <typename T, int DK, int DV>
cudaError_t launch_prep(const void* q, const void* k, const void* v, const float* g, const float* beta,
                        const Layout& lay, int flags, unsigned char* ws, cudaStream_t st) {
  using S = PrepSmem<DK, DV>;
  auto kern = prep_kernel<T, DK, DV>;
  static bool attr_done[kMaxDevices] = {};  // once per device: no attribute call inside a graph capture
  cudaError_t e = set_smem_once(kern, S::total, attr_done);
  if (e != cudaSuccess) return e;
  dim3 grid(lay.NT, lay.H, lay.B);
  kern<<<grid, 128, S::total, st>>>(static_cast<const T*>(q), static_cast<const T*>(k), static_cast<const T*>(v), g,
                                    beta, lay, flags, ws);
  return cudaGetLastError();
}

template <typename T, int DK, int DV>
cudaError_t launch_state(const float* s0, void* o, float* sT, const Layout& lay, int flags, unsigned char* ws,
                         cudaStream_t st) {
  using S = StateSmem<DK, DV>;
  auto kern = state_kernel<T, DK, DV>;
  static bool attr_done[kMaxDevices] = {};  // once per device: no attribute call inside a graph capture
  cudaError_t e = set_smem_once(kern, S::total, attr_done);
  if (e != cudaSuccess) return e;
  dim3 grid(lay.H, lay.B);
  kern<<<grid, 128, S::total, st>>>(s0, static_cast<T*>(o), sT, lay, flags, ws);
  return cudaGetLastError();
}

template cudaError_t launch_prep<__nv_bfloat16, 128, 128>(const void*, const void*, const void*, const float*,
                                                          const float*, const Layout&, int, unsigned char*,
                                                          cudaStream_t);
template cudaError_t launch_prep<__half, 128, 128>(const void*, const void*, const void*, const float*, const float*,
                                                   const Layout&, int, unsigned char*, cudaStream_t);
template cudaError_t launch_prep<float, 128, 128>(const void*, const void*, const void*, const float*, const float*,
                                                  const Layout&, int, unsigned char*, cudaStream_t);
template cudaError_t launch_state<__nv_bfloat16, 128, 128>(const float*, void*, float*, const Layout&, int,
                                                           unsigned char*, cudaStream_t);
template cudaError_t launch_state<__half, 128, 128>(const float*, void*, float*, const Layout&, int, unsigned char*,
                                                    cudaStream_t);
template cudaError_t launch_state<float, 128, 128>(const float*, void*, float*, const Layout&, int, unsigned char*,
                                                   cudaStream_t);

}  // namespace gd
