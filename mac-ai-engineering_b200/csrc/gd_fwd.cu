// Forward kernels of the chunked gated delta rule on B200 (sm_100a):
//   prep_kernel   persistent CTAs of 256 threads (two per SM), each taking (chunk, value head, batch row) items in turn:
//                 l2 prologue, cumulative decay, the C x C products on tcgen05, the unit-lower-triangular inverse, W and
//                 U;
//   state_kernel  two CTAs per (value head, batch row), 64 value columns each (four CTAs of 32 in gd_state_narrow.cu):
//                 the sequential chunk pass with the state in registers (fp32) and every product on tcgen05 from shared
//                 memory, chunk inputs streamed in by the bulk-copy engine.
// Equations (per chunk; src/macai/gated_delta/_chunked.py:1-35, tools/check_chunk_equations.py:29-46 of the reference):
//   G = cumsum(g), gamma = exp(G), e = exp(G_last - G)
//   L = diag(beta) (K K^T) * exp(G_i - G_j) (i > j),  M = (Q K^T) * exp(G_i - G_j) (i >= j),  A = (I + L)^-1
//   W = A diag(beta gamma) K,  U = A diag(beta) V
//   Vn = U - W S,  O = diag(gamma) Q S + M Vn,  S <- exp(G_last) S + K^T diag(e) Vn
// Precision: bf16 operands with fp32 accumulation; q and k (in Q K^T, K K^T), A diag(beta gamma) (in W), A diag(beta)
// (in U), K~ and Vn (in the state update), M and Vn (in M Vn) are split into bf16 hi + lo pairs (two or three MMAs into
// one accumulator); the backward's A and W^T images carry their low halves too; the state is carried in fp32.
#include <type_traits>

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
  static constexpr size_t L = a2l + 64 * 64 * 2;          // [64][68] fp32, L (strictly lower; 16-byte aligned rows)
  static constexpr size_t Ai = L + 64 * 68 * 4;           // [64][68] fp32, A
  static constexpr size_t a1l = L;                        // [64 x 64] A diag(beta gamma), lo (L is dead by then)
  static constexpr size_t ql = L;                         // [64 x DK] low half of q, then k: live only until the
  static constexpr size_t kl = ql + 64 * DK * 2;          //   Q K^T / K K^T product is done (L and A reuse them)
  static_assert(2 * 64 * DK * 2 <= 2 * 64 * 68 * 4, "the q / k low halves must fit in the L and A buffers");
  static constexpr size_t G = Ai + 64 * 68 * 4;           // [64] cumulative log decay
  static constexpr size_t beta = G + 64 * 4;              // [64]
  static constexpr size_t gam = beta + 64 * 4;            // [64] gamma = exp(G)
  static constexpr size_t bgam = gam + 64 * 4;            // [64] beta gamma
  static constexpr size_t scan = bgam + 64 * 4;           // [2] warp totals of the scan
  static constexpr size_t rng = scan + 16;                // [2][2] per-warp max, min of G
  static constexpr size_t colf = rng + 16;                // [64] exp(G_ref - G_j): the decay's column factors
  static constexpr size_t bar = (colf + 64 * 4 + 7) & ~size_t(7);  // [2] MMA commits; raw rows landed (16-bit types)
  static constexpr size_t tmem = bar + 2 * 8;
  static constexpr size_t total = tmem + 16;
};

// A = (I + L)^-1 for the 64 x 64 strictly lower L (fp32, row stride 68) by divide and conquer, all 256 threads:
//   1. the four diagonal 16 x 16 blocks T_b = (I + L_bb)^-1 at once, one column per thread (64 threads: forward
//      substitution x_i = [i == j] - sum_{m < i} L_im x_m, unrolled; the other warps zero A's upper blocks meanwhile);
//   2. the 32 x 32 halves: A_21 = -T_2 (L_21 T_1) for block pairs (0, 1) and (2, 3);
//   3. the whole: A_21 = -A_22 (L_21 A_11) with 32 x 32 blocks.
// Each product is a 4-column strip per thread over float4 rows; Y (32 x 36 floats, 16-byte rows) is scratch. The
// reference's gdc_prep (src/macai/gated_delta/_chunked.py:282-311) inverts by blocked substitution; the blocks are the
// same unit-lower inverse, combined here by the block formula instead of row by row.
// out[i][j0 .. j0 + 3] = sign * sum_{m < N} X[i][m] Z[m][j0 .. j0 + 3] (row strides xs, zs, os floats; 16-byte rows),
// unrolled so that the shared-memory loads run ahead of the four accumulation chains
template <int N>
__device__ __forceinline__ void strip(const float* X, int xs, const float* Z, int zs, float* out, int os, float sign,
                                      int i, int j0) {
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int m4 = 0; m4 < N; m4 += 4) {
    const float4 x4 = *reinterpret_cast<const float4*>(X + i * xs + m4);
    const float xv[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float4 z = *reinterpret_cast<const float4*>(Z + (m4 + u) * zs + j0);
      acc.x = fmaf(xv[u], z.x, acc.x);
      acc.y = fmaf(xv[u], z.y, acc.y);
      acc.z = fmaf(xv[u], z.z, acc.z);
      acc.w = fmaf(xv[u], z.w, acc.w);
    }
  }
  *reinterpret_cast<float4*>(out + i * os + j0) = make_float4(sign * acc.x, sign * acc.y, sign * acc.z, sign * acc.w);
}

// The same for rows i and i + 16 at once: each 16-byte read of Z feeds both rows (8 FMAs), so a 32 x 32 product takes
// 128 threads and ~40 % fewer shared-memory reads than four-column strips on 256 threads.
template <int N>
__device__ __forceinline__ void strip2(const float* X, int xs, const float* Z, int zs, float* out, int os, float sign,
                                       int i, int j0) {
  float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
#pragma unroll
  for (int m4 = 0; m4 < N; m4 += 4) {
    const float4 x0 = *reinterpret_cast<const float4*>(X + i * xs + m4);
    const float4 x1 = *reinterpret_cast<const float4*>(X + (i + 16) * xs + m4);
    const float xv0[4] = {x0.x, x0.y, x0.z, x0.w}, xv1[4] = {x1.x, x1.y, x1.z, x1.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float4 z = *reinterpret_cast<const float4*>(Z + (m4 + u) * zs + j0);
      a0.x = fmaf(xv0[u], z.x, a0.x);
      a0.y = fmaf(xv0[u], z.y, a0.y);
      a0.z = fmaf(xv0[u], z.z, a0.z);
      a0.w = fmaf(xv0[u], z.w, a0.w);
      a1.x = fmaf(xv1[u], z.x, a1.x);
      a1.y = fmaf(xv1[u], z.y, a1.y);
      a1.z = fmaf(xv1[u], z.z, a1.z);
      a1.w = fmaf(xv1[u], z.w, a1.w);
    }
  }
  *reinterpret_cast<float4*>(out + i * os + j0) = make_float4(sign * a0.x, sign * a0.y, sign * a0.z, sign * a0.w);
  *reinterpret_cast<float4*>(out + (i + 16) * os + j0) = make_float4(sign * a1.x, sign * a1.y, sign * a1.z, sign * a1.w);
}

__device__ __forceinline__ void unit_lower_inverse(const float* L, float* A, float* Y, unsigned char* ws,
                                                   const Layout& lay, int tb) {
  const int tid = threadIdx.x;
  if (tid < 64) {
    const int b = tid >> 4, j = tid & 15, r0 = 16 * b;
    float x[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float acc = (i == j) ? 1.f : 0.f;
#pragma unroll
      for (int m4 = 0; m4 < i; m4 += 4) {
        const float4 l4 = *reinterpret_cast<const float4*>(L + (r0 + i) * 68 + r0 + m4);
        const float lv[4] = {l4.x, l4.y, l4.z, l4.w};
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (m4 + u < i) acc = fmaf(-lv[u], x[m4 + u], acc);
      }
      x[i] = acc;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) A[(r0 + i) * 68 + r0 + j] = x[i];
  } else {
    // upper blocks (block row bi < block column bj) are zero: 6 blocks x 16 rows x 4 float4
    for (int idx = tid - 64; idx < 6 * 64; idx += 192) {
      const int blk = idx >> 6, r = (idx >> 2) & 15, c4 = idx & 3;
      const int bi = blk < 3 ? 0 : (blk < 5 ? 1 : 2);
      const int bj = blk < 3 ? blk + 1 : (blk < 5 ? blk - 1 : 3);
      *reinterpret_cast<float4*>(A + (16 * bi + r) * 68 + 16 * bj + 4 * c4) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  GD_TRACE_AT(ws, lay, tb + 16);
  __syncthreads();
  GD_TRACE_AT(ws, lay, tb + 17);
  // 2. pairs p = 0, 1: blocks lo = 2p, hi = 2p + 1 (rows / columns 16 lo .., 16 hi ..)
  const int p = tid >> 6, i16 = (tid >> 2) & 15, j4 = 4 * (tid & 3);
  if (tid < 128)  // Y_p = L[hi][lo] T_lo
    strip<16>(L + (32 * p + 16) * 68 + 32 * p, 68, A + (32 * p) * 68 + 32 * p, 68, Y + 16 * p * 36, 36, 1.f, i16, j4);
  __syncthreads();
  if (tid < 128)  // A[hi][lo] = -T_hi Y_p
    strip<16>(A + (32 * p + 16) * 68 + 32 * p + 16, 68, Y + 16 * p * 36, 36, A + (32 * p + 16) * 68 + 32 * p, 68, -1.f,
              i16, j4);
  __syncthreads();
  GD_TRACE_AT(ws, lay, tb + 18);
  // 3. Y = L[32:64][0:32] A_11 ; A[32:64][0:32] = -A_22 Y (threads 0-127: rows i16 and i16 + 16)
  const int i16b = tid >> 3, j8 = 4 * (tid & 7);
  if (tid < 128) strip2<32>(L + 32 * 68, 68, A, 68, Y, 36, 1.f, i16b, j8);
  __syncthreads();
  GD_TRACE_AT(ws, lay, tb + 19);
  if (tid < 128) strip2<32>(A + 32 * 68 + 32, 68, Y, 36, A + 32 * 68, 68, -1.f, i16b, j8);
  GD_TRACE_AT(ws, lay, tb + 20);
}

// BWD: the backward layout (its extra images); the forward instance carries none of that code
template <typename T, int DK, int DV, bool BWD>
__global__ void __launch_bounds__(256, 2) prep_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                   const T* __restrict__ v, const float* __restrict__ g,
                                                   const float* __restrict__ beta, Layout lay, int flags,
                                                   unsigned char* __restrict__ ws,
                                                   const __grid_constant__ CUtensorMap tm_q,
                                                   const __grid_constant__ CUtensorMap tm_k,
                                                   const __grid_constant__ CUtensorMap tm_v) {
  using S = PrepSmem<DK, DV>;
  extern __shared__ __align__(1024) unsigned char smem[];
  ErrorWord* err = reinterpret_cast<ErrorWord*>(ws + lay.err);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float* sL = reinterpret_cast<float*>(smem + S::L);
  float* sAi = reinterpret_cast<float*>(smem + S::Ai);
  float* sG = reinterpret_cast<float*>(smem + S::G);
  float* sB = reinterpret_cast<float*>(smem + S::beta);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + S::bar);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + S::tmem);
  constexpr bool staged = sizeof(T) == 2;
  // Persistent: CTA x takes the chunks x, x + gridDim.x, ... of the B x H x NT items (chunk index fastest). The next
  // item's raw rows, g and beta are requested as soon as the current item's W / U products have read the tiles, so
  // their latency hides under the W / U epilogue.
  const long long n_items = (long long)lay.NT * lay.H * lay.B;
  auto item_of = [&](long long it, int& c, int& h, int& b) {
    c = (int)(it % lay.NT);
    const long long r = it / lay.NT;
    h = (int)(r % lay.H);
    b = (int)(r / lay.H);
  };
  // this chunk's g and beta (threads 0-63, one token each; padding rows: g = 0, beta = 0, which leaves G constant
  // past the last token)
  auto load_gb = [&](int c, int h, int b, float& gv, float& bv) {
    const ChunkSpan sp = lay.span(ws, c);
    gv = 0.f;
    bv = 0.f;
    if (tid < 64 && sp.t0 + tid < sp.end) {
      gv = __ldg(g + ((size_t)b * lay.Tin + sp.t0 + tid) * lay.H + h);
      bv = __ldg(beta + ((size_t)b * lay.Tin + sp.t0 + tid) * lay.H + h);
    }
  };
  // 16-bit inputs: the chunk's raw q, k, v rows land row-major ([64][D], 256-byte rows) in the q, k, v tile buffers,
  // one tensor-map copy each; rows past T arrive as zeros (thread 0)
  auto issue_rows = [&](int c, int h, int b) {
    const int t0 = lay.span(ws, c).t0, hk = h / lay.rep;
    mbar_arrive_expect_tx(bar + 1, (uint32_t)(64 * (2 * DK + DV) * 2));
    tma_load_4d(smem + S::q, &tm_q, 0, hk, t0, b, bar + 1);
    tma_load_4d(smem + S::k, &tm_k, 0, hk, t0, b, bar + 1);
    tma_load_4d(smem + S::v, &tm_v, 0, h, t0, b, bar + 1);
  };

  GD_TRACE_AT(ws, lay, 0);
  GD_TRACE_CTA(ws, lay, 0);
  long long it = blockIdx.x;
  int c, h, b;
  item_of(it, c, h, b);
  float gi, bi;
  load_gb(c, h, b, gi, bi);
  if (tid == 0) {
    mbar_init(bar, 1);      // MMA commits
    mbar_init(bar + 1, 1);  // raw q / k / v rows landed
    fence_mbar_init();
    if (staged) issue_rows(c, h, b);
  }
  __syncthreads();  // the barriers are initialised before anyone waits on them
  if (warp == 0) {
    tmem_alloc(tslot, 256);
    tmem_relinquish();
  }
  GD_TRACE_AT(ws, lay, 15);
  const bool norm = (flags & GD_L2NORM) != 0;
  const float qscale = q_scale(flags, DK);

  for (int n = 0;; ++n) {
    const int tb = 64 * (n < 3 ? n : 3);  // trace slots of the item (the fourth and later share the last set)
    const int hk = h / lay.rep;
    // the chunk's rows in the caller's arrays: t0 .. t0 + 63, those below tend valid (the sequence's end)
    const ChunkSpan span = lay.span(ws, c);
    const int t0 = span.t0, tend = span.end;
    const size_t cidx = ((size_t)b * lay.H + h) * lay.NT + c;

    // l2 prologue and operand tiles: every row load in flight before any is converted
    const bool bwd = BWD && (h % lay.rep == 0);
    const size_t rrow = (((size_t)b * lay.HK + hk) * lay.NT + c) * 64;  // this chunk's 64 rsqrt slots
    float* rq = bwd ? reinterpret_cast<float*>(ws + lay.rq) + rrow : nullptr;
    float* rk = bwd ? reinterpret_cast<float*>(ws + lay.rk) + rrow : nullptr;
    Rows<T, DK, 8, staged> rq_rows, rk_rows;
    Rows<T, DV, 8, staged> rv_rows;
    GD_TRACE_AT(ws, lay, tb + 21);
    bool landed = true;
    if constexpr (staged) {
      // each warp converts its own 8 rows in place: raw rows 8 w .. 8 w + 7 and tile row block w are the same 2 KB
      landed = mbar_wait(bar + 1, n & 1, err, 13);
      rq_rows.issue_staged(smem + S::q, t0, tend);
      rk_rows.issue_staged(smem + S::k, t0, tend);
      rv_rows.issue_staged(smem + S::v, t0, tend);
      __syncwarp();
    } else {
      rq_rows.issue(q, b, t0, lay.Tin, tend, lay.HK, hk);
      rk_rows.issue(k, b, t0, lay.Tin, tend, lay.HK, hk);
    }
    GD_TRACE_AT(ws, lay, tb + 22);
    rq_rows.finish(t0, tend, norm, qscale, smem + S::q, rq, smem + S::ql);
    GD_TRACE_AT(ws, lay, tb + 23);
    rk_rows.finish(t0, tend, norm, 1.f, smem + S::k, rk, smem + S::kl);
    GD_TRACE_AT(ws, lay, tb + 24);
    if (!staged) rv_rows.issue(v, b, t0, lay.Tin, tend, lay.H, h);
    rv_rows.finish(t0, tend, false, 1.f, smem + S::v, nullptr, nullptr);
    GD_TRACE_AT(ws, lay, tb + 1);

    // cumulative log decay
    if (tid < 64) {
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
    float* sGam = reinterpret_cast<float*>(smem + S::gam);
    float* sBG = reinterpret_cast<float*>(smem + S::bgam);
    float* sRng = reinterpret_cast<float*>(smem + S::rng);
    float* sColf = reinterpret_cast<float*>(smem + S::colf);
    if (tid < 64) {  // each thread finishes its own token: G, gamma, beta gamma, and its warp's range of G
      if (tid >= 32) sG[tid] += reinterpret_cast<float*>(smem + S::scan)[0];
      sGam[tid] = __expf(sG[tid]);
      sBG[tid] = sB[tid] * sGam[tid];
      float mx = sG[tid], mn = mx;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      }
      if (lane == 0) {
        sRng[2 * warp] = mx;
        sRng[2 * warp + 1] = mn;
      }
    }
    tc_fence_after();
    const uint32_t tm = *tslot;
    __syncthreads();  // G, gamma complete for everyone
    // The decay exp(G_i - G_j) of the C x C products factors as exp(G_i - G_ref) exp(G_ref - G_j) with G_ref the middle
    // of the chunk's range of G: 64 column factors here and one row factor per thread below instead of 32 exponentials
    // per thread. Taken when the range is at most 80 (every factor within e^-40 .. e^40, so no product of two factors
    // leaves the normal fp32 range); wider ranges (or NaN) take one exponential per element.
    const float gmax = fmaxf(sRng[0], sRng[2]), gmin = fminf(sRng[1], sRng[3]);
    const float gref = 0.5f * gmax + 0.5f * gmin;
    const bool factored = gmax - gmin <= 80.f;

    // [Q; K] K^T with q and k carried as bf16 hi + lo (three products): lanes 0-63 hold Q K^T rows, 64-127 K K^T rows.
    // Issued after the barrier: the issue blocks thread 0 while the other warps write the images below.
    if (tid == 0) {
      const Tile qkh{smem_u32(smem + S::q), DK}, qkl{smem_u32(smem + S::ql), DK};
      const Tile kh{smem_u32(smem + S::k), DK}, kl{smem_u32(smem + S::kl), DK};
      mma_tiles(tm, 128, 64, DK, qkh, true, 0, 0, kh, false, 0, false);
      mma_tiles(tm, 128, 64, DK, qkh, true, 0, 0, kl, false, 0, true);
      mma_tiles(tm, 128, 64, DK, qkl, true, 0, 0, kh, false, 0, true);
      mma_commit(bar);
    }
    GD_TRACE_AT(ws, lay, tb + 2);
    if (factored && tid >= 192) sColf[tid - 192] = __expf(gref - sG[tid - 192]);
    if constexpr (BWD) {  // the low halves go out (transposed images) before L and A overwrite them
      unsigned char* dst = ws + lay.qkl + cidx * lay.qk_bytes();
      store_tile_transposed<64, DK, 8>(smem + S::ql, dst);
      store_tile_transposed<64, DK, 8>(smem + S::kl, dst + 64 * DK * 2);
    }
    {  // K~ = diag(e) K (e_i = exp(G_last - G_i) <= 1) from k's hi + lo, split again: the state update's operand
      unsigned char* kth = ws + lay.kt + cidx * lay.qk_bytes();
      unsigned char* ktl = kth + 64 * DK * 2;
      const float Glast = sG[63];
      for (int idx = tid; idx < 64 * DK / 8; idx += 256) {
        const int rl = idx & 7, cb = (idx >> 3) % (DK / 8), rb = idx / (8 * (DK / 8));
        const int r = 8 * rb + rl;
        const uint4 uh = *reinterpret_cast<const uint4*>(smem + S::k + blk_off(r, 8 * cb, DK));
        const uint4 ul = *reinterpret_cast<const uint4*>(smem + S::kl + blk_off(r, 8 * cb, DK));
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&uh);
        const __nv_bfloat162* l2 = reinterpret_cast<const __nv_bfloat162*>(&ul);
        const float er = __expf(Glast - sG[r]);
        float x[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 fh = __bfloat1622float2(h2[e]), fl = __bfloat1622float2(l2[e]);
          x[2 * e] = er * (fh.x + fl.x);
          x[2 * e + 1] = er * (fh.y + fl.y);
        }
        store8_split(kth, ktl, r, 8 * cb, DK, x);
      }
    }
    GD_TRACE_AT(ws, lay, tb + 3);
    bool ok = mbar_wait(bar, 0, err, 10) && landed;
    GD_TRACE_AT(ws, lay, tb + 4);
    ok = __syncthreads_and(ok);
    tc_fence_after();
    if (ok) {
      // warp w: accumulator rows 32 (w % 4) + lane (Q K^T for w % 4 < 2, K K^T otherwise), columns 32 (w / 4) .. + 31
      const int i = tid & 63;
      const float Gi = sG[i];
      float acc[32];
      unsigned char* mimg = ws + lay.m + cidx * lay.mm_bytes();
      {
        const int half = warp >> 2;
        GD_TRACE_WARP(ws, lay, 0);
        tmem_ld32(tmem_lane_addr(tm, warp, 32 * half), acc);
        GD_TRACE_AT(ws, lay, tb + 25);
        GD_TRACE_WARP(ws, lay, 1);
        // the decay exp(G_i - G_j), computed for every column and then masked by keep_if (no branches)
        const bool is_m = (warp & 3) < 2;
        const int jmax = is_m ? i : i - 1;  // M keeps j <= i, L keeps j < i
        const float bi = is_m ? 1.f : sB[i];
        if (factored) {
          const float rf = bi * __expf(Gi - gref);
#pragma unroll
          for (int q4 = 0; q4 < 8; ++q4) {
            const float4 c4 = *reinterpret_cast<const float4*>(sColf + 32 * half + 4 * q4);
            const float cv[4] = {c4.x, c4.y, c4.z, c4.w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int jj = 4 * q4 + u;
              acc[jj] = keep_if(acc[jj] * (rf * cv[u]), 32 * half + jj <= jmax);
            }
          }
        } else {
#pragma unroll
          for (int q4 = 0; q4 < 8; ++q4) {
            const float4 g4 = *reinterpret_cast<const float4*>(sG + 32 * half + 4 * q4);
            const float gv[4] = {g4.x, g4.y, g4.z, g4.w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int jj = 4 * q4 + u;
              acc[jj] = keep_if(bi * acc[jj] * __expf(Gi - gv[u]), 32 * half + jj <= jmax);
            }
          }
        }
        GD_TRACE_WARP(ws, lay, 2);
        if (is_m) {
#pragma unroll
          for (int q8 = 0; q8 < 4; ++q8)
            store8_split(mimg, mimg + lay.m_bytes(), i, 32 * half + 8 * q8, 64, acc + 8 * q8);
        } else {
          float4* lrow = reinterpret_cast<float4*>(sL + i * 68 + 32 * half);
#pragma unroll
          for (int q4 = 0; q4 < 8; ++q4)
            lrow[q4] = make_float4(acc[4 * q4], acc[4 * q4 + 1], acc[4 * q4 + 2], acc[4 * q4 + 3]);
        }
      }
    }
    GD_TRACE_AT(ws, lay, tb + 26);
    GD_TRACE_WARP(ws, lay, 3);
    __syncthreads();
    GD_TRACE_AT(ws, lay, tb + 5);
    // (ok is the same in every thread: the barriers inside are reached by all or none)
    if (ok) unit_lower_inverse(sL, sAi, reinterpret_cast<float*>(smem + S::a1), ws, lay, tb);
    __syncthreads();  // A complete for everyone
    GD_TRACE_AT(ws, lay, tb + 6);

    if (ok) {
      // A diag(beta gamma) and the hi/lo split of A diag(beta) as K-major B operands (rows i, cols j). A warp takes 32
      // consecutive rows at one column block: its 16-byte reads of A (row stride 68 floats) and its 16-byte writes of
      // the blocked tiles both fall on distinct banks in every group of eight lanes.
      const int i = tid & 63, j0 = 16 * (tid >> 6);
#pragma unroll
      for (int q8 = 0; q8 < 2; ++q8) {
        const int jb = j0 + 8 * q8;
        const float4 x0 = *reinterpret_cast<const float4*>(sAi + i * 68 + jb);
        const float4 x1 = *reinterpret_cast<const float4*>(sAi + i * 68 + jb + 4);
        const float a0[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
        float a1[8], a2[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          a1[e] = a0[e] * sBG[jb + e];
          a2[e] = a0[e] * sB[jb + e];
        }
        store8_split(smem + S::a1, smem + S::a1l, i, jb, 64, a1);
        store8_split(smem + S::a2h, smem + S::a2l, i, jb, 64, a2);
      }
    }
    // (the backward's A and V^T images go out after the MMAs are issued: global stores ahead of this proxy fence would
    // hold it until they complete)
    fence_async_smem();
    GD_TRACE_AT(ws, lay, tb + 7);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (ok && tid == 0) {
      // W^T [DK x 64] = K^T (A diag(beta gamma))^T ; U^T [DV x 64] = V^T (A diag(beta))^T (both A factors hi + lo:
      // with nearly parallel keys W is a difference of nearly equal rows, which a one-bf16 A diag(beta gamma) loses)
      mma_tiles(tm + 64, DK, 64, 64, Tile{smem_u32(smem + S::k), DK}, false, 0, 0, Tile{smem_u32(smem + S::a1), 64},
                false, 0, false);
      mma_tiles(tm + 64, DK, 64, 64, Tile{smem_u32(smem + S::k), DK}, false, 0, 0, Tile{smem_u32(smem + S::a1l), 64},
                false, 0, true);
      mma_tiles(tm + 128, DV, 64, 64, Tile{smem_u32(smem + S::v), DV}, false, 0, 0, Tile{smem_u32(smem + S::a2h), 64},
                false, 0, false);
      mma_tiles(tm + 128, DV, 64, 64, Tile{smem_u32(smem + S::v), DV}, false, 0, 0, Tile{smem_u32(smem + S::a2l), 64},
                false, 0, true);
      mma_commit(bar);
    }
    GD_TRACE_AT(ws, lay, tb + 10);
    // the q / k images and G go out while the MMAs run (the k image only for the backward), and for the backward the
    // A image and the transposed V image ([DV x 64], rows v)
    if (ok) {
      unsigned char* dst = ws + lay.qk + cidx * lay.qk_bytes();  // transposed images ([DK x 64], rows d)
      store_tile_transposed<64, DK, 8>(smem + S::q, dst);
      GD_TRACE_AT(ws, lay, tb + 11);
      if constexpr (BWD) {
        store_tile_transposed<64, DK, 8>(smem + S::k, dst + 64 * DK * 2);
        store_tile_transposed<64, DV, 8>(smem + S::v, ws + lay.vi + cidx * lay.vi_bytes());
        unsigned char* aimg = ws + lay.ai + cidx * lay.mm_bytes();  // A hi, then lo
        const int i = tid & 63, j0 = 16 * (tid >> 6);
#pragma unroll
        for (int q8 = 0; q8 < 2; ++q8) {
          const float4 x0 = *reinterpret_cast<const float4*>(sAi + i * 68 + j0 + 8 * q8);
          const float4 x1 = *reinterpret_cast<const float4*>(sAi + i * 68 + j0 + 8 * q8 + 4);
          const float a0[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
          store8_split(aimg, aimg + lay.m_bytes(), i, j0 + 8 * q8, 64, a0);
        }
      }
      GD_TRACE_AT(ws, lay, tb + 12);
      if (tid < 64) reinterpret_cast<float*>(ws + lay.gc + cidx * lay.gc_bytes())[tid] = sG[tid];
    }
    GD_TRACE_AT(ws, lay, tb + 27);
    if (ok) ok = mbar_wait(bar, 1, err, 11);
    GD_TRACE_AT(ws, lay, tb + 8);
    ok = __syncthreads_and(ok);
    tc_fence_after();
    // the W / U products have read k and v and every image store has read q, k, v: the next item's rows may land
    const long long nx = it + gridDim.x;
    const bool more = ok && nx < n_items;
    int cn = 0, hn = 0, bn = 0;
    float g_next = 0.f, beta_next = 0.f;
    if (more) {
      item_of(nx, cn, hn, bn);
      if (staged && tid == 0) {
        fence_async_smem();
        issue_rows(cn, hn, bn);
      }
      load_gb(cn, hn, bn, g_next, beta_next);
    }
    if (ok) {
      float acc[32];
      const int row = tid & 127;
      if (warp < 4) {  // W^T row dk = row -> blocked [DK x 64] image (and its low half for the backward), 16-byte stores
        unsigned char* wimg = ws + lay.wt + cidx * lay.wt_bytes();
        unsigned char* wlimg = ws + lay.wtl + cidx * lay.wt_bytes();
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
          tmem_ld32(tmem_lane_addr(tm, warp, 64 + 32 * half), acc);
          if constexpr (BWD) {
#pragma unroll
            for (int q8 = 0; q8 < 4; ++q8) store8_split(wimg, wlimg, row, 32 * half + 8 * q8, 64, acc + 8 * q8);
          } else {
#pragma unroll
            for (int q8 = 0; q8 < 4; ++q8) store8_bf16(wimg, row, 32 * half + 8 * q8, 64, acc + 8 * q8);
          }
        }
      } else {  // U^T row v = row -> U [64][DV] fp32
        float* u = reinterpret_cast<float*>(ws + lay.u + cidx * lay.u_bytes());
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
          tmem_ld32(tmem_lane_addr(tm, warp, 128 + 32 * half), acc);
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) u[(32 * half + jj) * DV + row] = acc[jj];
        }
      }
    }
    GD_TRACE_AT(ws, lay, tb + 9);
    tc_fence_before();
    __syncthreads();  // the accumulators are read before the next item's products overwrite them
    GD_TRACE_AT(ws, lay, tb + 28);
    if (!more) break;
    it = nx;
    c = cn;
    h = hn;
    b = bn;
    gi = g_next;
    bi = beta_next;
  }
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(*tslot, 256);
  }
  GD_TRACE_CTA(ws, lay, 1);
}

// ------------------------------------------------------------------------------------------------------------------
// forward state pass (warp-specialised, value-split)
//
// Two CTAs per (value head, batch row), each owning 64 of the 128 value columns (the recurrence never mixes value
// columns: Vn = U - W S, S <- e S + K~^T Vn and O = gamma Q S + M Vn act on each column of S alone), so the pass runs
// on twice the SMs with half the work per chunk step. 16 epilogue warps, 1 MMA warp, 1 loader warp. Every product is
// M = 64 (the
// CTA's value columns on TMEM lanes 0-15 of each quadrant) and is read whole-warp (16x32bx2): warp w (quadrant w % 4,
// quarter w / 4) thread t holds value column 16 (w % 4) + t % 16 and tokens 16 (w / 4) + 8 (t / 16) .. + 7 of the
// [64 x 64] products, key rows 32 (w / 4) + 16 (t / 16) .. + 15 of the [64 x DK] state update; it keeps the fp32
// state S[those key rows][its column] in registers. One thread of warp 16 issues every MMA (and, with
// GD_STORE_STATES, the bulk copies out); one thread of warp 17 loads the two input stages, so that a refill (whose
// bulk copies queue behind running products) never delays the MMA thread's next hand-off. Hand-offs are mbarriers
// only. Per chunk c:
//   LOAD: wait stage_free of chunk c - 2 -> stage c & 1 <- W^T, q^T, K~ hi / lo, M images of chunk c
//   MMA: wait stage c and the S tile -> (W S)^T -> ws_full; (Q S)^T -> qs_full[c & 1]
//   EPI: wait ws_full -> Vn = U - W S (U and G prefetched into registers) -> Vn^T hi / lo tiles -> vn_full
//   MMA: wait vn_full -> (K~^T Vn)^T, three products (K~ = diag(e) K and Vn split) -> ds_full; (M Vn)^T ->
//        mv_full[c & 1]; stage_free[c & 1]
//   EPI: (after handing Vn of chunk c to the tensor core) O of chunk c - 1 = diag(gamma) Q S + M Vn -> global (16-byte
//        rows after an 8 x 8 transpose): it runs under chunk c's state-update product, off the chain
//   EPI: wait ds_full -> S <- exp(G_last) S + K~^T Vn -> S tile -> st_full
// With GD_STORE_STATES (the backward's recompute, or a training forward that keeps its states) the pass also keeps S_c
// (a bf16 S_c^T image and its low half) and the Vn^T hi / lo images of every chunk for the backward kernels (each CTA
// its 64 rows of them); O is formed when o is not null.

constexpr int kVsplit = 2;  // CTAs per (value head, batch row)

template <int DK, int DV>
struct StateSmem {
  static constexpr int DVH = DV / kVsplit;                 // value columns per CTA
  static constexpr size_t st = 0;                          // [DVH x DK] bf16 S^T (rows v, cols dk)
  static constexpr size_t vh = st + DVH * DK * 2;          // [DVH x 64] Vn^T hi
  static constexpr size_t vl = vh + DVH * 64 * 2;          //             lo
  static constexpr size_t stage0 = vl + DVH * 64 * 2;      // two input stages, each:
  static constexpr size_t s_wt = 0;                        //   [DK x 64] W^T image
  static constexpr size_t s_q = s_wt + DK * 64 * 2;        //   [DK x 64] q image (hi, transposed)
  static constexpr size_t s_kt = s_q + 64 * DK * 2;        //   [2][64 x DK] K~ hi, lo
  static constexpr size_t s_m = s_kt + 2 * 64 * DK * 2;    //   [2][64 x 64] M image: hi, lo
  static constexpr size_t stage_bytes = s_m + 2 * 64 * 64 * 2;
  static constexpr size_t ost = stage0 + 2 * stage_bytes;   // [2][64 x DVH] O staging (row-major, 16-bit outputs)
  static constexpr size_t bar = ost + 2 * 64 * DVH * 2;
  static constexpr int NBAR = 17;
  static constexpr size_t tmem = bar + NBAR * 8;
  static constexpr size_t total = tmem + 8;
};

// A chunk's stage: W^T and K~ always, the q and M images only when O is formed (the Q S and M Vn products)
template <int DK, int DV>
__device__ __forceinline__ void issue_stage(unsigned char* stg, const unsigned char* ws, const Layout& lay,
                                            size_t cidx, uint64_t* bar, bool out) {
  using S = StateSmem<DK, DV>;
  mbar_arrive_expect_tx(bar, (uint32_t)(out ? S::stage_bytes : lay.wt_bytes() + lay.qk_bytes()));
  bulk_g2s(stg + S::s_wt, ws + lay.wt + cidx * lay.wt_bytes(), (uint32_t)lay.wt_bytes(), bar);
  bulk_g2s(stg + S::s_kt, ws + lay.kt + cidx * lay.qk_bytes(), (uint32_t)lay.qk_bytes(), bar);
  if (out) {
    bulk_g2s(stg + S::s_q, ws + lay.qk + cidx * lay.qk_bytes(), 64 * DK * 2, bar);
    bulk_g2s(stg + S::s_m, ws + lay.m + cidx * lay.mm_bytes(), (uint32_t)lay.mm_bytes(), bar);
  }
}

template <typename T, int DK, int DV>
__global__ void __launch_bounds__(576) state_kernel(const float* __restrict__ s0, T* __restrict__ o,
                                                       float* __restrict__ sT, Layout lay, int flags,
                                                       unsigned char* __restrict__ ws,
                                                       const __grid_constant__ CUtensorMap tm_o) {
  static_assert(DV == 128 && DK == 128, "64 value columns per CTA on TMEM lanes 0-15 of each quadrant");
  using S = StateSmem<DK, DV>;
  constexpr int DVH = S::DVH;
  extern __shared__ __align__(1024) unsigned char smem[];
  ErrorWord* err = reinterpret_cast<ErrorWord*>(ws + lay.err);
  GD_TRACE_AT(ws, lay, 4000);
  const int half = blockIdx.x % kVsplit, h = blockIdx.x / kVsplit;
  int z, b, cfirst, clast;  // z: batch row or sequence (s0 and sT are indexed by it); b: the workspace's batch row;
                            // the chunks [cfirst, clast) walked here
  lay.chunks_of(ws, blockIdx.y, z, b, cfirst, clast);
  const int vbase = DVH * half;  // this CTA's first value column
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (clast <= cfirst) {  // a sequence without tokens: the state passes through
    if (sT != nullptr)
      for (int i = tid; i < DK * DVH; i += blockDim.x) {
        const size_t at = ((size_t)z * lay.H + h) * DK * DV + (size_t)(i / DVH) * DV + vbase + i % DVH;
        sT[at] = s0 ? s0[at] : 0.f;
      }
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::bar);
  uint64_t* full = bars + 0;        // [2] stage loaded (bulk-copy bytes)
  uint64_t* stage_free = bars + 2;  // [2] every MMA that reads the stage is done
  uint64_t* ws_full = bars + 4;
  uint64_t* qs_full = bars + 5;     // [2]
  uint64_t* ds_full = bars + 7;
  uint64_t* mv_full = bars + 8;     // [2]
  uint64_t* vn_full = bars + 10;    // 16 epilogue warps
  uint64_t* st_full = bars + 11;    // 16 epilogue warps
  uint64_t* o_full = bars + 12;     // [2] 16 epilogue warps: O staging buffer written
  uint64_t* o_free = bars + 14;     // [2] thread 0: the tensor store has read the buffer
  uint64_t* never = bars + 16;      // GD_TEST_WAIT_EXPIRES: a barrier nothing signals
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + S::tmem);
  const bool store = (flags & GD_STORE_STATES) != 0 && lay.backward();
  const bool out = o != nullptr;  // both at once: the stored-states training forward
  const int NT = clast - cfirst;                                     // chunks this CTA pair walks
  const size_t row0 = ((size_t)b * lay.H + h) * lay.NT + cfirst;    // the first one's workspace index
  const int trow0 = cfirst * C;                                      // its first row of o

  if (warp == 0) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int i = 0; i < 10; ++i) mbar_init(bars + i, 1);
    mbar_init(vn_full, 16);
    mbar_init(st_full, 16);
    mbar_init(o_full, 16);
    mbar_init(o_full + 1, 16);
    mbar_init(o_free, 1);
    mbar_init(o_free + 1, 1);
    mbar_init(never, 1);
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = *tslot;
  GD_TRACE_AT(ws, lay, 4001);
  // TMEM: (W S)^T at tm, (Q S)^T at tm + 64 + 64 (c & 1), (M Vn)^T at tm + 192 + 64 (c & 1), (K~^T Vn)^T (128 wide)
  const uint32_t tWS = tm, tDS = tm + 320;
  const Tile tSt{smem_u32(smem + S::st), DK};
  const Tile tVh{smem_u32(smem + S::vh), 64}, tVl{smem_u32(smem + S::vl), 64};
  bool ok = true;

  if (warp == 16) {
    // ---------------- MMA and bulk-copy issuer (one thread)
    if (lane == 0) {
      // test only: a wait that expires before any product is issued (the failure path, with nothing in flight on
      // the tensor core); the other roles then give up in their own bounded waits and the CTA frees its TMEM
      if (flags & GD_TEST_WAIT_EXPIRES) ok = mbar_wait_for(never, 0, err, 28, kTestWaitCycles);
      for (int c = 0; c < NT && ok; ++c) {
        const int s = c & 1;
        const uint32_t par2 = (c >> 1) & 1;
        unsigned char* stg = smem + S::stage0 + s * S::stage_bytes;
        ok = mbar_wait(full + s, par2, err, 20) && mbar_wait(st_full, c & 1, err, 21);
        if (!ok) break;
        GD_TRACE_ONE(ws, lay, 1024 + 8 * c + 0);
        tc_fence_after();
        if (store) {  // this CTA's rows of the S_c^T image (bulk copy out; done reading before the tile is rewritten)
          bulk_s2g(ws + lay.sci + (row0 + c) * lay.si_bytes() + (size_t)vbase * DK * 2, smem + S::st, DVH * DK * 2);
          bulk_commit();
        }
        mma_tiles(tWS, DVH, 64, DK, tSt, true, 0, 0, Tile{smem_u32(stg + S::s_wt), 64}, true, 0, false);
        mma_commit(ws_full);
        GD_TRACE_ONE(ws, lay, 1024 + 8 * c + 1);
        if (out) {
          mma_tiles(tm + 64 + 64 * s, DVH, 64, DK, tSt, true, 0, 0, Tile{smem_u32(stg + S::s_q), 64}, true, 0,
                    false);
          mma_commit(qs_full + s);
        }
        GD_TRACE_ONE(ws, lay, 1024 + 8 * c + 2);
        GD_TRACE_ONE(ws, lay, 1024 + 8 * c + 3);
        ok = mbar_wait(vn_full, c & 1, err, 22);
        if (!ok) break;
        GD_TRACE_ONE(ws, lay, 1024 + 8 * c + 4);
        tc_fence_after();
        if (store) {  // this CTA's rows of the Vn^T hi and lo images
          unsigned char* vn = ws + lay.vni + (row0 + c) * lay.vn_bytes() + (size_t)vbase * 64 * 2;
          bulk_s2g(vn, smem + S::vh, DVH * 64 * 2);
          bulk_s2g(vn + DV * 64 * 2, smem + S::vl, DVH * 64 * 2);
          bulk_commit();
        }
        const Tile tKh{smem_u32(stg + S::s_kt), DK}, tKl{smem_u32(stg + S::s_kt + 64 * DK * 2), DK};
        mma_tiles(tDS, DVH, DK, 64, tVh, true, 0, 0, tKh, true, 0, false);
        mma_tiles(tDS, DVH, DK, 64, tVh, true, 0, 0, tKl, true, 0, true);
        mma_tiles(tDS, DVH, DK, 64, tVl, true, 0, 0, tKh, true, 0, true);
        if (store) bulk_wait_read0();  // the S^T and Vn^T tiles may be rewritten once ds_full fires
        mma_commit(ds_full);
        GD_TRACE_ONE(ws, lay, 1024 + 8 * c + 5);
        if (out) {
          const Tile tM{smem_u32(stg + S::s_m), 64}, tMl{smem_u32(stg + S::s_m + 64 * 64 * 2), 64};
          mma_tiles(tm + 192 + 64 * s, DVH, 64, 64, tVh, true, 0, 0, tM, false, 0, false);
          mma_tiles(tm + 192 + 64 * s, DVH, 64, 64, tVh, true, 0, 0, tMl, false, 0, true);
          mma_tiles(tm + 192 + 64 * s, DVH, 64, 64, tVl, true, 0, 0, tM, false, 0, true);
          mma_commit(mv_full + s);
        }
        mma_commit(stage_free + s);
        GD_TRACE_ONE(ws, lay, 1024 + 8 * c + 6);
      }
      if (store) bulk_wait0();
    }
    __syncwarp();
  } else if (warp == 17) {
    // ---------------- stage loader (one thread)
    if (lane == 0) {
      int c = 0;
      for (; c < NT; ++c) {
        const int s = c & 1;
        if (c >= 2 && !mbar_wait(stage_free + s, ((c - 2) >> 1) & 1, err, 23)) break;
        issue_stage<DK, DV>(smem + S::stage0 + s * S::stage_bytes, ws, lay, row0 + c, full + s, out);
      }
      // every copy issued here lands before the CTA may exit, also after a failed wait
      for (int l = c >= 2 ? c - 2 : 0; l < c; ++l) mbar_wait(full + (l & 1), (l >> 1) & 1, err, 29);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue warps
    const int qd = warp & 3, quarter = warp >> 2;
    const int vl_ = 16 * qd + (lane & 15);               // local value column (TMEM lane within the quadrant)
    const int v = vbase + vl_;                           // value column
    const int tk = 16 * quarter + 8 * (lane >> 4);       // tokens tk .. tk + 7 of the [64 x 64] products
    const int dk0 = 32 * quarter + 16 * (lane >> 4);     // key rows dk0 .. dk0 + 15 of the state held here
    float Sr[16];                                        // S[dk0 + j][v]
    {
      const float* p = s0 ? s0 + ((size_t)z * lay.H + h) * DK * DV : nullptr;
#pragma unroll
      for (int j = 0; j < 16; ++j) Sr[j] = p ? p[(size_t)(dk0 + j) * DV + v] : 0.f;
#pragma unroll
      for (int q8 = 0; q8 < 2; ++q8) store8_bf16(smem + S::st, vl_, dk0 + 8 * q8, DK, Sr + 8 * q8);
      fence_async_smem();
      mbar_arrive_warp(st_full);
    }
    // the low half of the state entering chunk c, for the backward's <S_c, dS_{c+1}> (its high half is the S_c^T image
    // the MMA thread copies out of the S tile): this CTA's rows of the [DV x DK] image, 16-byte pieces
    auto store_slo = [&](int c) {
      unsigned char* lo = ws + lay.scl + (row0 + c) * lay.si_bytes();
      float hi[16], l[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) split_bf16(Sr[j], hi[j], l[j]);
#pragma unroll
      for (int q8 = 0; q8 < 2; ++q8) store8_bf16(lo, v, dk0 + 8 * q8, DK, l + 8 * q8);
    };
    if (store) store_slo(0);
    // U of the next chunk, and G (cumulative log gates) at tokens tk .. tk + 7 and the chunk's last token: read from L2
    // one pass ahead so that no stage holds G for the late O product
    float Ur[8], gcur[8], gcur_last, gprev[8];
    auto load_u = [&](size_t cidx) {
      const float* u = reinterpret_cast<const float*>(ws + lay.u + cidx * lay.u_bytes());
#pragma unroll
      for (int j = 0; j < 8; ++j) Ur[j] = __ldg(u + (tk + j) * DV + v);
      const float* gp = reinterpret_cast<const float*>(ws + lay.gc + cidx * lay.gc_bytes());
      const float4 g0 = __ldg(reinterpret_cast<const float4*>(gp + tk)), g1 = __ldg(reinterpret_cast<const float4*>(gp + tk + 4));
      gcur[0] = g0.x; gcur[1] = g0.y; gcur[2] = g0.z; gcur[3] = g0.w;
      gcur[4] = g1.x; gcur[5] = g1.y; gcur[6] = g1.z; gcur[7] = g1.w;
      gcur_last = __ldg(gp + 63);
    };
    load_u(row0);
    // O of one chunk. 16-bit outputs: row-major into staging buffer p & 1 (every warp arrives on o_full), then one
    // tensor store (rows past T are not written) issued by thread 0 once all have; thread 0 marks a buffer free
    // (o_free) when the next chunk's O begins and the store has read it, and writers wait for that before reusing
    // the buffer two chunks later. All waits bounded. fp32 outputs: 16-byte token rows after an 8 x 8 transpose.
    float o8[8];
    auto store_o = [&](int p) -> bool {
      if constexpr (sizeof(T) == 2) {
        const int bi = p & 1;
        T* stg = reinterpret_cast<T*>(smem + S::ost + bi * 64 * DVH * 2);
        if (tid == 0 && p >= 1) {
          bulk_wait_read0();
          mbar_arrive(o_free + ((p - 1) & 1));
        }
        if (p >= 2 && !mbar_wait(o_free + bi, ((p - 2) >> 1) & 1, err, 50)) return false;
#pragma unroll
        for (int j = 0; j < 8; ++j) stg[(tk + j) * DVH + vl_] = cvt_out<T>(o8[j]);
        fence_async_smem();
        mbar_arrive_warp(o_full + bi);
        if (tid == 0) {
          if (!mbar_wait(o_full + bi, (p >> 1) & 1, err, 51)) return false;
          tma_store_4d(&tm_o, vbase, h, trow0 + p * C, b, stg);
          bulk_commit();
        }
      } else {
        store_token_rows8<T>(o8, o + ((size_t)b * lay.T * lay.H + h) * DV, (size_t)lay.H * DV, trow0 + p * C + tk,
                             lay.T,
                             vbase + 16 * qd + 8 * ((lane >> 3) & 1));
      }
      return true;
    };
    // pass c computes Vn and the state update of chunk c (c < NT) and, between them, O of chunk c - 1 (c >= 1)
    for (int c = 0; c <= NT; ++c) {
      const size_t cidx = row0 + c;
      if (c < NT) {
        // * Vn = U - W S
        GD_TRACE_AT(ws, lay, 8 * c + 0);
        if (!mbar_wait(ws_full, c & 1, err, 24)) { ok = false; break; }
        GD_TRACE_AT(ws, lay, 8 * c + 1);
        tc_fence_after();
        float acc[8];
        tmem_ld8h(tmem_lane_addr(tWS, warp, 16 * quarter), acc);
        GD_TRACE_AT(ws, lay, 2048 + 8 * c + 0);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = Ur[j] - acc[j];
        store8_split(smem + S::vh, smem + S::vl, vl_, tk, 64, acc);
        GD_TRACE_AT(ws, lay, 2048 + 8 * c + 1);
        tc_fence_before();
        fence_async_smem();
        GD_TRACE_AT(ws, lay, 2048 + 8 * c + 2);
        mbar_arrive_warp(vn_full);
        GD_TRACE_AT(ws, lay, 8 * c + 2);
      }
      if (out && c >= 1) {
        // * O of chunk c - 1 = diag(gamma) Q S + M Vn, formed under this chunk's state-update product and stored after
        // the update (under the next W S). Its (Q S)^T and (M Vn)^T are complete: ws_full of chunk c, waited above,
        // tracks every earlier product; after the last chunk they are waited for here.
        const int p = c - 1, s = p & 1;
        if (c == NT &&
            (!mbar_wait(qs_full + s, (p >> 1) & 1, err, 26) || !mbar_wait(mv_full + s, (p >> 1) & 1, err, 27))) {
          ok = false;
          break;
        }
        GD_TRACE_AT(ws, lay, 8 * c + 5);
        tc_fence_after();
        float mv[8];
        tmem_ld8hx2(tmem_lane_addr(tm + 64 + 64 * s, warp, 16 * quarter), o8,
                    tmem_lane_addr(tm + 192 + 64 * s, warp, 16 * quarter), mv);
        GD_TRACE_AT(ws, lay, 8 * c + 6);
#pragma unroll
        for (int j = 0; j < 8; ++j) o8[j] = fmaf(__expf(gprev[j]), o8[j], mv[j]);
        tc_fence_before();
      }
      if (c == NT) {
        if (out && !store_o(NT - 1)) ok = false;
        break;
      }
      GD_TRACE_AT(ws, lay, 8 * c + 7);
      const float gl = __expf(gcur_last);
#pragma unroll
      for (int j = 0; j < 8; ++j) gprev[j] = gcur[j];
      if (c + 1 < NT) load_u(cidx + 1);  // next chunk's U and G into registers while the tensor core works
      // * S <- exp(G_last) S + K~^T Vn
      if (!mbar_wait(ds_full, c & 1, err, 25)) { ok = false; break; }
      GD_TRACE_AT(ws, lay, 8 * c + 3);
      tc_fence_after();
      {
        float d[16];
        tmem_ld16h(tmem_lane_addr(tDS, warp, 32 * quarter), d);
        GD_TRACE_AT(ws, lay, 2048 + 8 * c + 3);
#pragma unroll
        for (int j = 0; j < 16; ++j) Sr[j] = fmaf(gl, Sr[j], d[j]);
#pragma unroll
        for (int q8 = 0; q8 < 2; ++q8) store8_bf16(smem + S::st, vl_, dk0 + 8 * q8, DK, Sr + 8 * q8);
        GD_TRACE_AT(ws, lay, 2048 + 8 * c + 4);
        tc_fence_before();
        fence_async_smem();
        GD_TRACE_AT(ws, lay, 2048 + 8 * c + 5);
        mbar_arrive_warp(st_full);
      }
      if (store && c + 1 < NT) store_slo(c + 1);  // off the chain: the next MMAs are already unblocked
      if (out && c >= 1 && !store_o(c - 1)) {  // likewise
        ok = false;
        break;
      }
      GD_TRACE_AT(ws, lay, 8 * c + 4);
    }
    GD_TRACE_AT(ws, lay, 4002);
    if (sizeof(T) == 2 && out && tid == 0) bulk_wait0();  // the O tensor stores complete before the CTA ends
    if (ok && sT != nullptr) {
      float* sp = sT + ((size_t)z * lay.H + h) * DK * DV;
#pragma unroll
      for (int j = 0; j < 16; ++j) sp[(size_t)(dk0 + j) * DV + v] = Sr[j];
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tm, 512);
  }
  GD_TRACE_AT(ws, lay, 4003);
}
// ------------------------------------------------------------------------------------------------------------------
// launchers


template <typename T, int DK, int DV>
cudaError_t launch_prep(const void* q, const void* k, const void* v, const float* g, const float* beta,
                        const Layout& lay, int flags, unsigned char* ws, cudaStream_t st) {
  using S = PrepSmem<DK, DV>;
  auto kern = lay.backward() ? prep_kernel<T, DK, DV, true> : prep_kernel<T, DK, DV, false>;
  static bool attr_done[2][kMaxDevices] = {};  // once per device and instance: no attribute call inside a capture
  cudaError_t e = set_smem_once(kern, S::total, attr_done[lay.backward() ? 1 : 0]);
  if (e != cudaSuccess) return e;
  CUtensorMap mq{}, mk{}, mv{};  // 16-bit inputs only (fp32 rows are read by plain loads)
  if (sizeof(T) == 2) {
    const CUtensorMapDataType dt = map_dtype<T>();
    if (!rows_map(&mq, q, dt, lay.B, lay.Tin, lay.HK, DK) || !rows_map(&mk, k, dt, lay.B, lay.Tin, lay.HK, DK) ||
        !rows_map(&mv, v, dt, lay.B, lay.Tin, lay.H, DV))
      return cudaErrorInvalidValue;
  }
  // persistent: as many CTAs as fit on the GPU at once, at most one per item. Two per SM by the launch bounds
  // (registers), fewer if the SM's shared memory (less the per-block reservation) holds fewer.
  static int slots[kMaxDevices] = {};
  int dev = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (slots[dev] == 0) {
    int sms = 0, smem_sm = 0, reserved = 0;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev)) != cudaSuccess)
      return e;
    if ((e = cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev)) != cudaSuccess) return e;
    const int fit = smem_sm / (int)(S::total + reserved);
    slots[dev] = sms * (fit < 2 ? (fit < 1 ? 1 : fit) : 2);
  }
  const int n_slots = slots[dev];
  const long long items = (long long)lay.NT * lay.H * lay.B;
  const int grid = (int)(items < n_slots ? items : n_slots);
  kern<<<grid, 256, S::total, st>>>(static_cast<const T*>(q), static_cast<const T*>(k), static_cast<const T*>(v), g,
                                    beta, lay, flags, ws, mq, mk, mv);
  return cudaGetLastError();
}

template <typename T, int DK, int DV>
cudaError_t launch_state_narrow(const float* s0, void* o, float* sT, const Layout& lay, int flags, unsigned char* ws,
                                cudaStream_t st);

template <typename T, int DK, int DV>
cudaError_t launch_state(const float* s0, void* o, float* sT, const Layout& lay, int flags, unsigned char* ws,
                         cudaStream_t st) {
  // the value split: four CTAs per (head, row) for the forward with O when they all fit at once (gd_state_narrow.cu),
  // else two
  if (o != nullptr && !(flags & (GD_STORE_STATES | GD_WIDE_STATE_PASS))) {
    static int sms[kMaxDevices] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    if (sms[dev] == 0 && (e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
      return e;
    const long long pairs = (long long)lay.H * (lay.packed() ? lay.N : lay.B);
    if (4 * pairs <= sms[dev]) return launch_state_narrow<T, DK, DV>(s0, o, sT, lay, flags, ws, st);
  }
  using S = StateSmem<DK, DV>;
  auto kern = state_kernel<T, DK, DV>;
  static bool attr_done[kMaxDevices] = {};  // once per device: no attribute call inside a graph capture
  cudaError_t e = set_smem_once(kern, S::total, attr_done);
  if (e != cudaSuccess) return e;
  dim3 grid(lay.H * kVsplit, lay.packed() ? lay.N : lay.B);  // one CTA pair per (head, batch row or sequence)
  CUtensorMap mo{};  // 16-bit O: chunk tiles of one CTA's 64 value columns leave by tensor store
  if (sizeof(T) == 2 && o != nullptr && !rows_map(&mo, o, map_dtype<T>(), lay.B, lay.T, lay.H, DV, DV / kVsplit))
    return cudaErrorInvalidValue;
  kern<<<grid, 576, S::total, st>>>(s0, static_cast<T*>(o), sT, lay, flags, ws, mo);
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
