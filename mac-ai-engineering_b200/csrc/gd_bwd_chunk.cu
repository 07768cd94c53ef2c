// Per-chunk gradients of the chunked gated delta rule on B200 (sm_100a).
//
// A persistent kernel: one CTA per SM walks work items (chunk c, key head hk, batch row b) in a fixed order; an item has
// one sub-item per value head of the key head (GQA), and d(normalised q / k) are summed over the sub-items in registers
// in a fixed order (one writer per gradient element: no atomics, bitwise reproducible).
//
// Inputs per sub-item, all bf16 images from the workspace copied whole by the bulk-copy engine: S_c^T and Vn^T (the
// forward recompute), dS_{c+1}^T (hi, lo), dVn^T (hi, lo) and dO (the reverse pass), A (hi, lo), V^T and the
// transposed q / k images (prep); G (prep) and the partial sums of <S_c, dS_{c+1}> (reverse pass) in fp32. From the caller:
// beta and, for the l2 prologue's backward, q and k.
//
// Products, all tcgen05 from blocked shared-memory tiles into TMEM ("[D x 64]" accumulators put the head dimension on
// the 128 TMEM lanes; C x C ones use M = 64). TMEM blocks of 64 columns B0..B7:
//   G1:  B0 dO Vn^T, B1 (dO S^T)^T, B2 (dVn S^T)^T, B3 (A^T dVn)^T (dVn and A split), B4 dVn V^T (dVn split)
//   G3:  B6 (dM K)^T, B7 (dM^T Q)^T (dM, q and k split), B2 (A^T dW)^T (A split; one commit), B1 dW K^T,
//        B3 Q K^T (q and k split: M = Q K^T * Gamma in fp32 precision for R);   dW = -dVn S^T
//   G2:  B5 (Vn dS^T)^T (Vn and dS split); after e2: B1 K K^T (k split, for L and the dbeta term)
//   tail: B6 T1 = dA A^T, B7 A^T T1 (dL = -A^T T1; dA, A and T1 split), B5 (K^T (P_beta + P_beta^T))
//         with P_beta = diag(beta) (dL * Gamma)
// Equations: tools/check_chunk_equations.py:49-76 and src/macai/gated_delta/_chunked.py:20-34 of the reference; dg is
// summed without cancellation (the regrouping of _chunked.py:1138-1142, extended to the decay-mask terms):
//   dg_t = sum_{s>=t} (a_s + w_s) + gamma_last <S_c, dS_{c+1}> + sum_{r<t} E_r + sum_{i>=t>j} R_ij
//   a_s = gamma_s q_s . (dO S_c^T)_s, w_s = beta_s gamma_s k_s . X_s, E_r = e_r k_r . (Vn dS^T)_r,
//   R_ij = dM_ij (Q K^T)_ij + dL_ij L_ij,  X = A^T dW.
//
// Roles (18 warps): warps 0-15 epilogue (warp w: TMEM lane quadrant w % 4, 16 columns from 16 (w / 4)); warp 16 one
// thread issuing every MMA (in dependency order, whichever is ready first); warp 17 one thread issuing every bulk copy.
// Shared memory holds one sub-item's tiles; each region is refilled for the next sub-item as soon as its last reader is
// done (the TMEM block plan lets the next sub-item's G1 run under this one's tail):
//   IN1 (S_c^T, dO, V^T; then dS^T)   free after G2
//   IN2 first half (dVn^T hi; then dM hi + lo)                          free after G3
//   IN2 second half (dVn^T lo; then dW^T; then dA lo; then T1 lo)       free after A^T T1
//   IN3 (Vn^T)                        free after G2        A hi, A lo (tail)            free after A^T T1
//   tail (dA hi; then T1 hi; then P_beta)                               free after K^T P_beta
//   QK (q^T, k^T hi + lo, rsqrt)      free after the item's last sub-item (the l2 backward reads x_hat from it)
// dV, dq and dk (16-bit) are staged row-major in regions free at that moment and leave by tensor store.
// All hand-offs are mbarriers; every wait is bounded and reports GD_ERR_TIMEOUT.
#include "gd_common.cuh"
#include "gd_layout.cuh"

namespace gd {

template <int DK, int DV>
struct ChunkSmem {
  static constexpr size_t qk = 0;                           // [2][DK x 64] q^T, k^T (hi)
  static constexpr size_t qkl = qk + 2 * DK * 64 * 2;       //              their low halves
  static constexpr size_t a = qkl + 2 * DK * 64 * 2;        // [64 x 64] A
  static constexpr size_t in1 = a + 64 * 64 * 2;            // 64 KB
  static constexpr size_t sc = in1;                         //   [DV x DK] S_c^T
  static constexpr size_t dO = sc + DV * DK * 2;            //   [64 x DV] dO
  static constexpr size_t vt = dO + 64 * DV * 2;            //   [DV x 64] V^T
  static constexpr size_t dsh = in1;                        //   then [DV x DK] dS^T hi
  static constexpr size_t dsl = in1 + DV * DK * 2;          //                     lo
  static constexpr size_t in2 = in1 + 2 * DV * DK * 2;      // 32 KB
  static constexpr size_t dvh = in2;                        //   [DV x 64] dVn^T hi
  static constexpr size_t dvl = in2 + DV * 64 * 2;          //                   lo
  static constexpr size_t dmh = in2;                        //   then [64 x 64] dM hi
  static constexpr size_t dml = in2 + 64 * 64 * 2;          //                  lo
  static constexpr size_t dwt = in2 + 2 * 64 * 64 * 2;      //        [DK x 64] dW^T
  static constexpr size_t in3 = in2 + 2 * DV * 64 * 2;      // 32 KB: [DV x 64] Vn^T hi, lo
  static constexpr size_t vnh = in3;
  static constexpr size_t vnl = in3 + DV * 64 * 2;
  static constexpr size_t lo2 = dwt;                        // then [64 x 64] dA lo, then T1 lo (after G3)
  static constexpr size_t tail = in3 + 2 * DV * 64 * 2;     // 16 KB
  static constexpr size_t alo = tail;                       //   [64 x 64] A lo
  static constexpr size_t da = tail + 64 * 64 * 2;          //   [64 x 64] dA hi, then T1 hi, then P_beta
  static constexpr size_t g = tail + 2 * 64 * 64 * 2;       // fp32 [2][64] G (by sub-item parity)
  static constexpr size_t beta = g + 2 * 64 * 4;            // fp32 [64]
  static constexpr size_t part = beta + 64 * 4;             // fp32 [6][4][64] per-token partial sums (see kernel)
  static constexpr size_t scr = part + 6 * 4 * 64 * 4;      // fp32 [2][4][64] exchange scratch
  static constexpr size_t rqk = scr + 2 * 4 * 64 * 4;       // fp32 [2][64] the item's l2 rsqrt of q, k rows
  static constexpr size_t sl = rqk + 2 * 64 * 4;            // fp32 [2][32] <S_c, dS_{c+1}> partials (by parity)
  static constexpr size_t tok = sl + 2 * 32 * 4;            // fp32 [3][64] the sub-item's gamma_t, e_t, beta_t gamma_t
  static constexpr size_t xch = tok + 3 * 64 * 4;           // fp32 [4] the dg scans' cross-warp totals
  static constexpr size_t bar = xch + 16;
  static constexpr int NBAR = 23;
  static constexpr size_t tmem = bar + NBAR * 8;
  static constexpr size_t total = tmem + 16;
  static_assert(dwt + DK * 64 * 2 <= in3, "dM and dW^T fit in the dVn region");
  static_assert(scr % 16 == 0, "scr is read as float4");
  static_assert(total <= 232448, "within the 227 KB a CTA can have");
};

// partial-sum arrays (index into ChunkSmem::part): by TMEM lane quadrant [4][64] unless noted
enum { P_A = 0, P_KX = 1, P_VY = 2, P_E = 3, P_RECT = 4, P_PK = 5 /* by column quarter */ };

__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 512;" ::: "memory"); }

// every epilogue thread gets the AND of all epilogue threads' flags (keeps the 16 warps on one path)
__device__ __forceinline__ bool epi_all(bool ok) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, 512, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"(ok ? 1u : 0u)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ void unpack8(uint4 u, float* x) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    x[2 * e] = __uint_as_float(w[e] << 16);
    x[2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
  }
}

// columns c0 .. c0 + 15 of row r of a blocked [R x 64] image (shared or global), as floats; plus the low-half image
template <bool LO>
__device__ __forceinline__ void row16(const unsigned char* hi, const unsigned char* lo, int r, int c0, float (&x)[16]) {
  unpack8(*reinterpret_cast<const uint4*>(hi + blk_off(r, c0, 64)), x);
  unpack8(*reinterpret_cast<const uint4*>(hi + blk_off(r, c0 + 8, 64)), x + 8);
  if (LO) {
    float y[16];
    unpack8(*reinterpret_cast<const uint4*>(lo + blk_off(r, c0, 64)), y);
    unpack8(*reinterpret_cast<const uint4*>(lo + blk_off(r, c0 + 8, 64)), y + 8);
#pragma unroll
    for (int j = 0; j < 16; ++j) x[j] += y[j];
  }
}

struct Item {
  int b, hk, c, r, h;
  size_t cidx;   // this sub-item's chunk (value head h)
  size_t cidx0;  // the chunk of the key head's first value head (its q / k images)
};

__device__ __forceinline__ Item item_of(const Layout& lay, int n) {
  const int kk = n / lay.rep;
  const int g = blockIdx.x + kk * gridDim.x;
  Item it;
  it.c = g % lay.NT;
  const int bh = g / lay.NT;
  it.hk = bh % lay.HK;
  it.b = bh / lay.HK;
  it.r = n - kk * lay.rep;
  it.h = it.hk * lay.rep + it.r;
  it.cidx = ((size_t)it.b * lay.H + it.h) * lay.NT + it.c;
  it.cidx0 = ((size_t)it.b * lay.H + (size_t)it.hk * lay.rep) * lay.NT + it.c;
  return it;
}

// The sub-item after `it` without divisions (item_of's runtime divides, redone by every epilogue warp per sub-item,
// cost hundreds of issue cycles): the grid stride gridDim.x as (chunk, key head, batch) digits, added with carries.
struct ItemStep {
  int dc, dhk, db;
  __device__ explicit ItemStep(const Layout& lay) {
    const int G = gridDim.x;
    dc = G % lay.NT;
    const int q = G / lay.NT;
    dhk = q % lay.HK;
    db = q / lay.HK;
  }
  __device__ __forceinline__ Item next(const Layout& lay, Item it) const {
    if (it.r + 1 < lay.rep) {  // the key head's next value head
      ++it.r;
      ++it.h;
      it.cidx += lay.NT;
      return it;
    }
    it.r = 0;
    it.c += dc;  // c, dc < NT and hk, dhk < HK: one carry each at most
    int carry = it.c >= lay.NT;
    if (carry) it.c -= lay.NT;
    it.hk += dhk + carry;
    carry = it.hk >= lay.HK;
    if (carry) it.hk -= lay.HK;
    it.b += db + carry;
    it.h = it.hk * lay.rep;
    it.cidx0 = ((size_t)it.b * lay.H + it.h) * lay.NT + it.c;
    it.cidx = it.cidx0;
    return it;
  }
};

template <typename T, int DK, int DV>
__global__ void __launch_bounds__(576, 1) bwd_chunk_kernel(const T* __restrict__ qraw, const T* __restrict__ kraw,
                                                           const float* __restrict__ beta, T* __restrict__ dq,
                                                           T* __restrict__ dk, T* __restrict__ dv,
                                                           float* __restrict__ dg, float* __restrict__ dbeta,
                                                           Layout lay, int flags, unsigned char* __restrict__ ws,
                                                           const __grid_constant__ CUtensorMap tm_dq,
                                                           const __grid_constant__ CUtensorMap tm_dk,
                                                           const __grid_constant__ CUtensorMap tm_dv) {
  static_assert(DK == 128 && DV == 128, "the head dimension maps onto the 128 TMEM lanes");
  using S = ChunkSmem<DK, DV>;
  extern __shared__ __align__(1024) unsigned char smem[];
  ErrorWord* err = reinterpret_cast<ErrorWord*>(ws + lay.err);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::bar);
  uint64_t* in_full = bars + 0;    // IN1, IN2's first half, IN3, G of a sub-item (bulk-copy bytes)
  uint64_t* a_full = bars + 1;     // A hi and lo, IN2's second half (dVn^T lo)
  uint64_t* qk_full = bars + 2;    // once per item
  uint64_t* ds_full = bars + 3;
  uint64_t* g1_full = bars + 4;    // MMA commits
  uint64_t* g3_full = bars + 5;
  uint64_t* g2_full = bars + 6;
  uint64_t* t1_full = bars + 7;
  uint64_t* dl_full = bars + 8;
  uint64_t* p11_full = bars + 9;
  uint64_t* e1_done = bars + 10;   // 16 epilogue warps each
  uint64_t* e2_done = bars + 11;
  uint64_t* e3_done = bars + 12;
  uint64_t* e4_done = bars + 13;
  uint64_t* b5_free = bars + 14;
  uint64_t* epi_done = bars + 15;  // [2] by sub-item parity
  uint64_t* drain = bars + 17;
  uint64_t* qk_free = bars + 18;   // 16 epilogue warps, once per item
  uint64_t* kk_full = bars + 20;   // MMA commit: K K^T
  uint64_t* g3a_full = bars + 21;  // MMA commit: the first part of G3 (B6, B7, B2)
  uint64_t* dv_read = bars + 22;   // thread 0: the dV tensor store has read its staging rows (the dO tile)
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + S::tmem);

  const int NG = lay.B * lay.HK * lay.NT;
  const int nsub = ((NG - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x) * lay.rep;

  GD_TRACE_CTA(ws, lay, 0);
  if (warp == 0) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int i = 0; i < 10; ++i) mbar_init(bars + i, 1);
    for (int i = 10; i < 17; ++i) mbar_init(bars + i, 16);
    mbar_init(drain, 1);
    mbar_init(qk_free, 16);
    mbar_init(kk_full, 1);
    mbar_init(g3a_full, 1);
    mbar_init(dv_read, 1);
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = *tslot;
  if (warp < 16) GD_TRACE_AT(ws, lay, 4000);
  const uint32_t B0 = tm, B1 = tm + 64, B2 = tm + 128, B3 = tm + 192, B4 = tm + 256, B5 = tm + 320, B6 = tm + 384,
                 B7 = tm + 448;

  const Tile tQ{smem_u32(smem + S::qk), 64}, tK{smem_u32(smem + S::qk + DK * 64 * 2), 64};
  const Tile tQl{smem_u32(smem + S::qkl), 64}, tKl{smem_u32(smem + S::qkl + DK * 64 * 2), 64};
  const Tile tA{smem_u32(smem + S::a), 64};

  if (warp == 17) {
    // ---------------- bulk-copy issuer
    if (lane == 0) {
      bool ok = true;
      int last_in = -1, last_a = -1, last_qk = -1, last_ds = -1;
      const uint32_t half_vn = (uint32_t)lay.vn_bytes() / 2;  // one [DV x 64] image
      const uint32_t in_bytes =
          (uint32_t)(lay.si_bytes() + 2 * lay.vi_bytes() + lay.vn_bytes() + lay.gc_bytes() + lay.sl_bytes()) +
          half_vn;
      for (int n = 0; n < nsub && ok; ++n) {
        const Item it = item_of(lay, n);
        if (n >= 1) ok = mbar_wait(g3_full, (n - 1) & 1, err, 60);  // dM / dW^T (the IN2 region) consumed
        if (!ok) break;
        mbar_arrive_expect_tx(in_full, in_bytes);
        GD_TRACE_ONE(ws, lay, 3500 + 4 * n + 0);
        last_in = n;
        // dVn^T hi now; its lo half (the IN2 slot that carries dW^T, dA lo and T1 lo until dL) with A: both into L2 now
        const unsigned char* dvn = ws + lay.dvni + it.cidx * lay.vn_bytes();
        bulk_g2s(smem + S::dvh, dvn, half_vn, in_full);
        prefetch_l2(dvn + half_vn, half_vn);
        prefetch_l2(ws + lay.ai + it.cidx * lay.mm_bytes(), (uint32_t)lay.mm_bytes());
        if (n >= 1) ok = mbar_wait(g2_full, (n - 1) & 1, err, 61);                // dS^T and Vn^T consumed
        if (ok && n >= 2) ok = mbar_wait(epi_done + (n & 1), ((n - 2) >> 1) & 1, err, 62);  // G buffer n & 1 read
        if (!ok) break;
        GD_TRACE_ONE(ws, lay, 3500 + 4 * n + 1);
        bulk_g2s(smem + S::sc, ws + lay.sci + it.cidx * lay.si_bytes(), (uint32_t)lay.si_bytes(), in_full);
        bulk_g2s(smem + S::dO, ws + lay.doi + it.cidx * lay.vi_bytes(), (uint32_t)lay.vi_bytes(), in_full);
        bulk_g2s(smem + S::vt, ws + lay.vi + it.cidx * lay.vi_bytes(), (uint32_t)lay.vi_bytes(), in_full);
        bulk_g2s(smem + S::in3, ws + lay.vni + it.cidx * lay.vn_bytes(), (uint32_t)lay.vn_bytes(), in_full);
        bulk_g2s(smem + S::g + (n & 1) * 256, ws + lay.gc + it.cidx * lay.gc_bytes(), (uint32_t)lay.gc_bytes(),
                 in_full);
        bulk_g2s(smem + S::sl + (n & 1) * 128, ws + lay.sl + it.cidx * lay.sl_bytes(), (uint32_t)lay.sl_bytes(), in_full);
        if (n >= 1) ok = mbar_wait(dl_full, (n - 1) & 1, err, 63);  // A hi / lo and T1 lo consumed
        if (!ok) break;
        mbar_arrive_expect_tx(a_full, (uint32_t)lay.mm_bytes() + half_vn);
        GD_TRACE_ONE(ws, lay, 3500 + 4 * n + 2);
        last_a = n;
        const unsigned char* aimg = ws + lay.ai + it.cidx * lay.mm_bytes();
        bulk_g2s(smem + S::a, aimg, (uint32_t)lay.m_bytes(), a_full);
        bulk_g2s(smem + S::alo, aimg + lay.m_bytes(), (uint32_t)lay.m_bytes(), a_full);
        bulk_g2s(smem + S::dvl, dvn + half_vn, half_vn, a_full);
        if (it.r == 0) {
          const int m = n / lay.rep;
          if (m >= 1) ok = mbar_wait(qk_free, (m - 1) & 1, err, 64);  // the previous item's q / k consumed
          if (!ok) break;
          mbar_arrive_expect_tx(qk_full, 2 * (uint32_t)lay.qk_bytes() + 2 * 256);
          GD_TRACE_ONE(ws, lay, 3500 + 4 * n + 3);
          last_qk = m;
          bulk_g2s(smem + S::qk, ws + lay.qk + it.cidx0 * lay.qk_bytes(), (uint32_t)lay.qk_bytes(), qk_full);
          bulk_g2s(smem + S::qkl, ws + lay.qkl + it.cidx0 * lay.qk_bytes(), (uint32_t)lay.qk_bytes(), qk_full);
          const size_t rrow = (((size_t)it.b * lay.HK + it.hk) * lay.NT + it.c) * 64 * 4;
          bulk_g2s(smem + S::rqk, ws + lay.rq + rrow, 256, qk_full);
          bulk_g2s(smem + S::rqk + 256, ws + lay.rk + rrow, 256, qk_full);
        }
        ok = mbar_wait(e1_done, n & 1, err, 65);  // S_c^T, dO, V^T consumed (G1 and e1): dS^T goes over them
        ok = ok && mbar_wait(dv_read, n & 1, err, 66);  // and the dV rows staged in the dO tile are out
        if (!ok) break;
        mbar_arrive_expect_tx(ds_full, 2 * (uint32_t)lay.si_bytes());
        GD_TRACE_ONE(ws, lay, 3900 + n);
        last_ds = n;
        bulk_g2s(smem + S::dsh, ws + lay.dsi + it.cidx * 2 * lay.si_bytes(), 2 * (uint32_t)lay.si_bytes(), ds_full);
      }
      if (!ok) {  // let copies already issued land before the CTA can exit (short bound, no second report)
        const long long t0 = clock64();
        auto settle = [&](uint64_t* bar, int phase) {
          if (phase < 0) return;
          while (!mbar_try_wait(bar, phase & 1) && clock64() - t0 < 20000000ll) {
          }
        };
        settle(in_full, last_in);
        settle(a_full, last_a);
        settle(qk_full, last_qk);
        settle(ds_full, last_ds);
      }
    }
    __syncwarp();
  } else if (warp == 16) {
    // ---------------- MMA issuer: per sub-item n, in dependency order, whichever is ready first
    if (lane == 0) {
      const Tile tSc{smem_u32(smem + S::sc), DK}, tDO{smem_u32(smem + S::dO), DV}, tVt{smem_u32(smem + S::vt), 64};
      const Tile tDvh{smem_u32(smem + S::dvh), 64}, tDvl{smem_u32(smem + S::dvl), 64};
      const Tile tVnh{smem_u32(smem + S::vnh), 64}, tVnl{smem_u32(smem + S::vnl), 64};
      const Tile tDsh{smem_u32(smem + S::dsh), DK}, tDsl{smem_u32(smem + S::dsl), DK};
      const Tile tDmh{smem_u32(smem + S::dmh), 64}, tDml{smem_u32(smem + S::dml), 64};
      const Tile tDwt{smem_u32(smem + S::dwt), 64};
      const Tile tDa{smem_u32(smem + S::da), 64}, tLo2{smem_u32(smem + S::lo2), 64};
      const Tile tAl{smem_u32(smem + S::alo), 64};
      auto issue_g1 = [&]() {
        mma_tiles(B0, 64, 64, DV, tDO, true, 0, 0, tVnh, true, 0, false);    // dO Vn^T
        mma_tiles(B1, DK, 64, DV, tSc, false, 0, 0, tDO, false, 0, false);   // S dO^T
        mma_tiles(B2, DK, 64, DV, tSc, false, 0, 0, tDvh, true, 0, false);   // S dVn^T
        mma_tiles(B3, DV, 64, 64, tDvh, true, 0, 0, tA, true, 0, false);     // dVn^T A (dVn and A split)
        mma_tiles(B3, DV, 64, 64, tDvl, true, 0, 0, tA, true, 0, true);
        mma_tiles(B3, DV, 64, 64, tDvh, true, 0, 0, tAl, true, 0, true);
        mma_tiles(B4, 64, 64, DV, tDvh, false, 0, 0, tVt, true, 0, false);   // dVn V^T (dVn split)
        mma_tiles(B4, 64, 64, DV, tDvl, false, 0, 0, tVt, true, 0, true);
        mma_commit(g1_full);
      };
      bool ok = nsub > 0;
      if (ok) ok = mbar_wait(in_full, 0, err, 70) && mbar_wait(a_full, 0, err, 71);
      if (ok) {
        tc_fence_after();
        GD_TRACE_ONE(ws, lay, 3000);
        issue_g1();
        GD_TRACE_ONE(ws, lay, 3000 + 7);
      }
      for (int n = 0; n < nsub && ok; ++n) {
        const uint32_t par = n & 1;
        const uint32_t qpar = (n / lay.rep) & 1;
        bool g3 = false, g2 = false, kk = false, t1 = false, dl = false, p11 = false, g1n = (n + 1 >= nsub);
        long long t0 = clock64();
        while (!(g3 && g2 && kk && t1 && dl && p11 && g1n)) {
          bool progressed = false;
          if (!g3 && mbar_test(e1_done, par) && mbar_test(qk_full, qpar)) {
            tc_fence_after();
            GD_TRACE_ONE(ws, lay, 3000 + 8 * n + 1);
            mma_tiles(B6, DK, 64, 64, tK, true, 0, 0, tDmh, false, 0, false);    // (dM K)^T = K^T dM^T
            mma_tiles(B6, DK, 64, 64, tKl, true, 0, 0, tDmh, false, 0, true);
            mma_tiles(B6, DK, 64, 64, tK, true, 0, 0, tDml, false, 0, true);
            mma_tiles(B7, DK, 64, 64, tQ, true, 0, 0, tDmh, true, 0, false);     // (dM^T Q)^T = Q^T dM
            mma_tiles(B7, DK, 64, 64, tQl, true, 0, 0, tDmh, true, 0, true);
            mma_tiles(B7, DK, 64, 64, tQ, true, 0, 0, tDml, true, 0, true);
            mma_tiles(B2, DK, 64, 64, tDwt, true, 0, 0, tA, true, 0, false);     // (A^T dW)^T = dW^T A (A split)
            mma_tiles(B2, DK, 64, 64, tDwt, true, 0, 0, tAl, true, 0, true);
            mma_commit(g3a_full);
            mma_tiles(B1, 64, 64, DK, tDwt, false, 0, 0, tK, true, 0, false);    // dW K^T
            mma_tiles(B3, 64, 64, DK, tQ, false, 0, 0, tK, true, 0, false);      // Q K^T
            mma_tiles(B3, 64, 64, DK, tQ, false, 0, 0, tKl, true, 0, true);
            mma_tiles(B3, 64, 64, DK, tQl, false, 0, 0, tK, true, 0, true);
            mma_commit(g3_full);
            GD_TRACE_ONE(ws, lay, 3300 + 8 * n + 1);
            g3 = progressed = true;
          }
          // G2 after G3: its result is read after G3's
          if (g3 && !g2 && mbar_test(ds_full, par) && (n == 0 || mbar_test(b5_free, (n - 1) & 1))) {
            tc_fence_after();
            GD_TRACE_ONE(ws, lay, 3000 + 8 * n + 2);
            mma_tiles(B5, DK, 64, DV, tDsh, false, 0, 0, tVnh, true, 0, false);  // (Vn dS^T)^T = dS Vn^T
            mma_tiles(B5, DK, 64, DV, tDsh, false, 0, 0, tVnl, true, 0, true);
            mma_tiles(B5, DK, 64, DV, tDsl, false, 0, 0, tVnh, true, 0, true);
            mma_commit(g2_full);
            GD_TRACE_ONE(ws, lay, 3300 + 8 * n + 2);
            g2 = progressed = true;
          }
          if (g3 && !t1 && mbar_test(e2_done, par)) {
            tc_fence_after();
            GD_TRACE_ONE(ws, lay, 3000 + 8 * n + 4);
            mma_tiles(B6, 64, 64, 64, tDa, true, 0, 0, tA, false, 0, false);     // T1 = dA A^T (dA and A split)
            mma_tiles(B6, 64, 64, 64, tLo2, true, 0, 0, tA, false, 0, true);
            mma_tiles(B6, 64, 64, 64, tDa, true, 0, 0, tAl, false, 0, true);
            mma_commit(t1_full);
            t1 = progressed = true;
          }
          // K K^T into B1 (free from e2_done until the next sub-item's G1) right behind T1, so that dL, on the chain
          // to e4, is issued as soon as e3 is done
          if (t1 && !kk) {
            tc_fence_after();
            GD_TRACE_ONE(ws, lay, 3000 + 8 * n + 3);
            mma_tiles(B1, 64, 64, DK, tK, false, 0, 0, tK, true, 0, false);      // K K^T
            mma_tiles(B1, 64, 64, DK, tK, false, 0, 0, tKl, true, 0, true);
            mma_tiles(B1, 64, 64, DK, tKl, false, 0, 0, tK, true, 0, true);
            mma_commit(kk_full);
            kk = progressed = true;
          }
          if (t1 && !dl && mbar_test(e3_done, par)) {
            tc_fence_after();
            GD_TRACE_ONE(ws, lay, 3000 + 8 * n + 5);
            mma_tiles(B7, 64, 64, 64, tA, false, 0, 0, tDa, true, 0, false);     // A^T T1 (A and T1 split: with
            mma_tiles(B7, 64, 64, 64, tA, false, 0, 0, tLo2, true, 0, true);     //  nearly parallel keys the
            mma_tiles(B7, 64, 64, 64, tAl, false, 0, 0, tDa, true, 0, true);     //  chain dA -> T1 -> dL cancels)
            mma_commit(dl_full);
            dl = progressed = true;
          }
          // the next sub-item's G1 after P11 (P11 is on the chain; G1 has the whole final phase to run)
          if (p11 && !g1n && mbar_test(in_full, par ^ 1) && mbar_test(a_full, par ^ 1)) {
            tc_fence_after();
            GD_TRACE_ONE(ws, lay, 3000 + 8 * (n + 1));
            issue_g1();  // the next sub-item's first products (B2, B4 were read before e2_done, B0, B1, B3 before e4_done)
            GD_TRACE_ONE(ws, lay, 3000 + 8 * (n + 1) + 7);
            g1n = progressed = true;
          }
          if (dl && kk && !p11 && mbar_test(e4_done, par)) {
            tc_fence_after();
            GD_TRACE_ONE(ws, lay, 3000 + 8 * n + 6);
            mma_tiles(B5, DK, 64, 64, tK, true, 0, 0, tDa, true, 0, false);      // K^T P_beta
            mma_tiles(B5, DK, 64, 64, tK, true, 0, 0, tDa, false, 0, true);      //  + K^T P_beta^T
            mma_commit(p11_full);
            p11 = progressed = true;
          }
          if (progressed) {
            t0 = clock64();
          } else {
            __nanosleep(32);  // leave the sub-partition's issue slots to the epilogue warps
          }
          if (!progressed && clock64() - t0 > kWaitCycles) {
            report(err, GD_ERR_TIMEOUT, 100 + (g3 ? 1 : 0) + (g2 ? 2 : 0) + (t1 ? 4 : 0) + (dl ? 8 : 0) + (kk ? 16 : 0));
            ok = false;
            break;
          }
        }
      }
      // every MMA issued has completed before TMEM is freed
      mma_commit(drain);
      mbar_wait(drain, 0, err, 99);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue warps
    const int qd = warp & 3, quarter = warp >> 2;
    const int dcol = 32 * qd + lane;  // head-dimension row of the [D x 64] accumulators
    const int tok0 = 16 * quarter;    // their 16 token columns / the C x C columns of this warp
    // C x C (M = 64) accumulators are read whole-warp (tmem_ld8h): row ri, columns c8 .. c8 + 7
    const int ri = 16 * qd + (lane & 15);
    const int c8 = tok0 + 8 * (lane >> 4);
    float* sB = reinterpret_cast<float*>(smem + S::beta);
    float* part = reinterpret_cast<float*>(smem + S::part);
    float* scr = reinterpret_cast<float*>(smem + S::scr);
    auto P = [&](int which, int row, int t) -> float& { return part[(which * 4 + row) * 64 + t]; };
    const bool norm = (flags & GD_L2NORM) != 0;
    const float qscale = q_scale(flags, DK);
    const unsigned char* qh = smem + S::qk;
    const unsigned char* ql = smem + S::qkl;
    const unsigned char* kh = smem + S::qk + DK * 64 * 2;
    const unsigned char* kl = smem + S::qkl + DK * 64 * 2;

    // rect_t += sum_{i >= t} sum_{j < t} R_ij for this thread's columns t, from R's row segment rv (row ri, columns
    // c8 .. c8 + 7): row totals by 8-column group through scr, exclusive row prefixes, masked sums over the
    // half-warp's 16 rows
    auto rect = [&](const float (&rv)[8], bool init) {
      const int grp = c8 >> 3;
      float tot = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) tot += rv[j];
      scr[grp * 64 + ri] = tot;
      epi_sync();
      float run = 0.f;
      for (int g2 = 0; g2 < grp; ++g2) run += scr[g2 * 64 + ri];
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[j] = (ri >= c8 + j) ? run : 0.f;
        run += rv[j];
      }
      const float s = halfwarp_reduce_scatter8(v);
      if ((lane & 8) == 0) {
        float& dst = P(P_RECT, qd, c8 + (lane & 7));
        dst = init ? s : dst + s;
      }
    };

    float dQ[16], dK[16];  // d(normalised q / k)[token tok0 + j][dcol], summed over the item's value heads
#pragma unroll
    for (int j = 0; j < 16; ++j) dQ[j] = dK[j] = 0.f;
    if (nsub > 0 && tid < 64) {
      const Item it = item_of(lay, 0);
      const ChunkSpan sp = lay.span(ws, it.c);
      const int t = sp.t0 + tid;
      sB[tid] = (t < sp.end) ? beta[((size_t)it.b * lay.Tin + t) * lay.H + it.h] : 0.f;
    }
    epi_sync();
    bool ok = true;
    const ItemStep istep(lay);
    Item nx = item_of(lay, 0);
    for (int n = 0; n < nsub; ++n) {
      const Item it = nx;
      nx = istep.next(lay, it);  // read only while n + 1 < nsub
      const uint32_t par = n & 1;
      const int t0 = it.c * C;                    // the chunk's first row of dq, dk, dv (chunk-aligned)
      const ChunkSpan sp = lay.span(ws, it.c);  // its rows of beta, dg, dbeta (the caller's rows)
      const float* sG = reinterpret_cast<const float*>(smem + S::g + (n & 1) * 256);
      // ---- e1: dV and the vy partials, dW^T and dM tiles, dQ's first term and the a partials
      ok = mbar_wait(in_full, par, err, 80);
      GD_TRACE_AT(ws, lay, 32 * n + 30);
      ok = ok && mbar_wait(g1_full, par, err, 81);
      if (!(ok = epi_all(ok))) break;
      tc_fence_after();
      GD_TRACE_AT(ws, lay, 32 * n + 0);
      // the sub-item's per-token factors gamma_t = exp(G_t), e_t = exp(G_last - G_t), beta_t gamma_t, once (the
      // phases read them after the next epilogue barrier)
      float* sGam = reinterpret_cast<float*>(smem + S::tok);
      if (tid < 64) {
        const float gt = __expf(sG[tid]);
        sGam[tid] = gt;
        sGam[64 + tid] = __expf(sG[63] - sG[tid]);
        sGam[128 + tid] = sB[tid] * gt;
      }
      // dV rows: 16-bit outputs are staged row-major ([64 tokens][DV]) in the dO tile (dead once G1 is done) and
      // leave by one tensor store after the next barrier, so no later proxy fence waits for them; the dS refill of
      // IN1 waits for the store to have read them (dv_read). fp32 rows are stored after the e1 hand-off (its proxy
      // fence would wait for global stores in flight)
      float dvr[16];
      float dec[8];  // exp(G_ri - G_j) for this thread's row ri, columns c8 .. c8 + 7: dM, R and dL all use it
      // two row-dot partials share one 32-value reduce-scatter (31 shuffles for both): v . Y with q . (dO S^T) in
      // e1, k . X with k . (Vn dS^T) across e2 / eg2; the first of each pair waits in registers
      float vy[16], kx[16];
      {
        tmem_ld16(tmem_lane_addr(B3, warp, tok0), dvr);  // Y^T: v . Y, and dV = diag(beta) Y
        row16<false>(smem + S::vt, nullptr, dcol, tok0, vy);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          vy[j] *= dvr[j];
          dvr[j] *= sB[tok0 + j];
        }
        if constexpr (sizeof(T) == 2) {
          T* sv = reinterpret_cast<T*>(smem + S::dO);
#pragma unroll
          for (int j = 0; j < 16; ++j) sv[(tok0 + j) * DV + dcol] = cvt_out<T>(dvr[j]);
          fence_async_smem();
        }
      }
      {
        float y[16], x[8];
        tmem_ld16(tmem_lane_addr(B2, warp, tok0), y);  // dW^T
#pragma unroll
        for (int j = 0; j < 16; ++j) y[j] = -y[j];
        store8_bf16(smem + S::dwt, dcol, tok0, 64, y);
        store8_bf16(smem + S::dwt, dcol, tok0 + 8, 64, y + 8);
        tmem_ld8h(tmem_lane_addr(B0, warp, tok0), x);  // dO Vn^T -> dM
        const float Gi = sG[ri];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          dec[j] = __expf(Gi - sG[c8 + j]);
          x[j] = keep_if(x[j] * dec[j], c8 + j <= ri);
        }
        store8_split(smem + S::dmh, smem + S::dml, ri, c8, 64, x);
      }
      GD_TRACE_AT(ws, lay, 32 * n + 1);
      ok = mbar_wait(qk_full, (n / lay.rep) & 1, err, 82);
      if (!(ok = epi_all(ok))) break;
      if (sizeof(T) == 2 && tid == 0) {  // every warp's dV rows are staged
        tma_store_4d(&tm_dv, 0, it.h, t0, it.b, smem + S::dO);
        bulk_commit();
      }
      GD_TRACE_AT(ws, lay, 32 * n + 2);
      {
        float av[16], x[16];
        tmem_ld16(tmem_lane_addr(B1, warp, tok0), av);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          av[j] *= sGam[tok0 + j];  // gamma_t (dO S^T)_t
          dQ[j] += av[j];
        }
        tc_fence_before();
        fence_async_smem();
        mbar_arrive_warp(e1_done);
        if constexpr (sizeof(T) != 2)
          store_token_rows<T>(dvr, dv + ((size_t)it.b * lay.T * lay.H + it.h) * DV, (size_t)lay.H * DV, t0 + tok0,
                              lay.T, 32 * qd + 8 * (lane >> 3));
        row16<true>(qh, ql, dcol, tok0, x);
        float v[32];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          v[j] = vy[j];
          v[16 + j] = av[j] * x[j];
        }
        const float s = warp_reduce_scatter32(v);
        P(lane < 16 ? P_VY : P_A, qd, tok0 + (lane & 15)) = s;
      }
      if (tid == 0) {  // the dV store has read the staging rows (no-op for fp32): IN1 may take dS
        bulk_wait_read0();
        mbar_arrive(dv_read);
      }
      GD_TRACE_AT(ws, lay, 32 * n + 3);
      // ---- e2: dQ / dK terms, dA (and R's first term)
      ok = mbar_wait(g3a_full, par, err, 83);
      if (!(ok = epi_all(ok))) break;
      tc_fence_after();
      GD_TRACE_AT(ws, lay, 32 * n + 4);
      {
        float y[16], x[16];
        GD_TRACE_AT(ws, lay, 32 * n + 5);
        tmem_ld16x2(tmem_lane_addr(B6, warp, tok0), x, tmem_lane_addr(B7, warp, tok0), y);  // (dM K)^T, (dM^T Q)^T
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          dQ[j] += x[j];
          dK[j] += y[j];
        }
        tmem_ld16(tmem_lane_addr(B2, warp, tok0), x);  // X^T
        row16<true>(kh, kl, dcol, tok0, kx);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int i = tok0 + j;
          dK[j] = fmaf(sGam[128 + i], x[j], dK[j]);  // beta_i gamma_i
          kx[j] *= x[j];
        }
        GD_TRACE_AT(ws, lay, 32 * n + 6);
      }
      ok = mbar_wait(g3_full, par, err, 89);
      if (!(ok = epi_all(ok))) break;
      tc_fence_after();
      {
        float a10[8], a5[8];
        tmem_ld8hx2(tmem_lane_addr(B1, warp, tok0), a10, tmem_lane_addr(B4, warp, tok0), a5);  // dW K^T, dVn V^T
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int jj = c8 + j;
          a10[j] = keep_if(sB[jj] * fmaf(sGam[jj], a10[j], a5[j]), jj < ri);
        }
        store8_split(smem + S::da, smem + S::lo2, ri, c8, 64, a10);  // dW^T's last reader (G3) is done
      }
      GD_TRACE_AT(ws, lay, 32 * n + 7);
      tc_fence_before();
      fence_async_smem();
      mbar_arrive_warp(e2_done);
      GD_TRACE_AT(ws, lay, 32 * n + 8);
      GD_TRACE_AT(ws, lay, 32 * n + 9);
      // ---- eg2: (Vn dS^T)^T -> dK's decay-path term and the E partials
      ok = mbar_wait(g2_full, par, err, 84);
      if (!(ok = epi_all(ok))) break;
      tc_fence_after();
      GD_TRACE_AT(ws, lay, 32 * n + 10);
      {
        float x[16], y[16], v[32];
        tmem_ld16(tmem_lane_addr(B5, warp, tok0), x);
        row16<true>(kh, kl, dcol, tok0, y);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          x[j] *= sGam[64 + tok0 + j];  // e_t
          dK[j] += x[j];
          v[j] = kx[j];
          v[16 + j] = y[j] * x[j];
        }
        const float s = warp_reduce_scatter32(v);
        P(lane < 16 ? P_KX : P_E, qd, tok0 + (lane & 15)) = s;
      }
      GD_TRACE_AT(ws, lay, 32 * n + 11);
      // ---- e3: T1 tile
      GD_TRACE_AT(ws, lay, 32 * n + 12);
      ok = mbar_wait(t1_full, par, err, 85);
      if (!(ok = epi_all(ok))) break;
      tc_fence_after();
      GD_TRACE_AT(ws, lay, 32 * n + 13);
      {  // T1 hi and lo over dA hi and lo (their last reader, the T1 product, is complete; P_beta overwrites T1 hi
         // only after dl_full, when the dL product has read it)
        float x[8];
        tmem_ld8h(tmem_lane_addr(B6, warp, tok0), x);
        store8_split(smem + S::da, smem + S::lo2, ri, c8, 64, x);
      }
      tc_fence_before();
      fence_async_smem();
      mbar_arrive_warp(e3_done);
      GD_TRACE_AT(ws, lay, 32 * n + 14);
      // ---- e4: dL = -A^T T1 (strictly lower): R's second term, P_beta tile, the pk partials
      ok = mbar_wait(dl_full, par, err, 86) && mbar_wait(kk_full, par, err, 88);
      if (!(ok = epi_all(ok))) break;
      tc_fence_after();
      GD_TRACE_AT(ws, lay, 32 * n + 15);
      // R = dM * (Q K^T) + dL * L (strictly lower), both terms summed here for one rect pass: R's first term from
      // dO Vn^T and Q K^T (still in TMEM: the next sub-item's G1 overwrites them only after e4_done)
      float rv[8];
      {
        float x[8], kgrow[8];
        tmem_ld8hx2(tmem_lane_addr(B0, warp, tok0), x, tmem_lane_addr(B3, warp, tok0), kgrow);
#pragma unroll
        for (int j = 0; j < 8; ++j) rv[j] = x[j] * kgrow[j] * dec[j];  // masked with the dL term below
        tmem_ld8hx2(tmem_lane_addr(B7, warp, tok0), x, tmem_lane_addr(B1, warp, tok0), kgrow);  // A^T T1, K K^T
        float pk = 0.f;
        const float bi = sB[ri];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const bool in = c8 + j < ri;
          const float dl = -x[j];
          const float gam = dec[j];
          const float p = keep_if(dl * gam, in);
          rv[j] = keep_if(fmaf(dl * bi, kgrow[j] * gam, rv[j]), in);
          pk = fmaf(p, kgrow[j], pk);
          x[j] = bi * p;
        }
        store8_bf16(smem + S::da, ri, c8, 64, x);
        pk += __shfl_xor_sync(0xffffffffu, pk, 16);  // the row's other 8 columns of this quarter
        if (lane < 16) P(P_PK, quarter, ri) = pk;
      }
      tc_fence_before();
      fence_async_smem();
      mbar_arrive_warp(e4_done);
      GD_TRACE_AT(ws, lay, 32 * n + 16);
      rect(rv, true);
      GD_TRACE_AT(ws, lay, 32 * n + 17);
      // ---- final: dK's last term; dg and dbeta of this value head; dq / dk after the item's last value head
      float bnext = 0.f;  // the next sub-item's beta, fetched early (thread t alone reads and writes sB[t])
      if (n + 1 < nsub && tid < 64) {
        const ChunkSpan nsp = lay.span(ws, nx.c);
        const int t = nsp.t0 + tid;
        if (t < nsp.end) bnext = beta[((size_t)nx.b * lay.Tin + t) * lay.H + nx.h];
      }
      ok = mbar_wait(p11_full, par, err, 87);
      if (!(ok = epi_all(ok))) break;
      tc_fence_after();
      GD_TRACE_AT(ws, lay, 32 * n + 18);
      {
        float x[16];
        tmem_ld16(tmem_lane_addr(B5, warp, tok0), x);
#pragma unroll
        for (int j = 0; j < 16; ++j) dK[j] += x[j];
      }
      tc_fence_before();
      mbar_arrive_warp(b5_free);
      epi_sync();  // every partial of this sub-item is in place
      GD_TRACE_AT(ws, lay, 32 * n + 19);
      if (tid < 64) {
        const int t = tid;
        float a = 0.f, kx = 0.f, vy = 0.f, E = 0.f, rc = 0.f, pk = 0.f;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          a += P(P_A, w, t);
          kx += P(P_KX, w, t);
          vy += P(P_VY, w, t);
          E += P(P_E, w, t);
          rc += P(P_RECT, w, t);
          pk += P(P_PK, w, t);
        }
        // <S_c, dS_{c+1}> from its 32 partial sums: one per lane, a butterfly (the same order in both warps)
        const float sl = warp_sum(reinterpret_cast<const float*>(smem + S::sl + (n & 1) * 128)[lane]);
        const float gt = sGam[t];
        const float w_ = sB[t] * gt * kx;
        const float db = fmaf(gt, kx, vy) + pk;
        // suffix sum of (a + w) over the chunk and exclusive prefix of E (two warps), without subtraction
        float suf = a + w_, pre = E;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y = __shfl_down_sync(0xffffffffu, suf, o);
          if (lane + o < 32) suf += y;
          const float z = __shfl_up_sync(0xffffffffu, pre, o);
          if (lane >= o) pre += z;
        }
        float* xch = reinterpret_cast<float*>(smem + S::xch);  // [2] cross-warp totals (not in scr: the other
                                                                 // warps' l2 dot products may be writing it now)
        if (lane == 0 && warp == 1) xch[0] = suf;
        if (lane == 31 && warp == 0) xch[1] = pre;
        float pre_excl = __shfl_up_sync(0xffffffffu, pre, 1);
        if (lane == 0) pre_excl = 0.f;
        asm volatile("bar.sync 2, 64;" ::: "memory");
        if (warp == 0) suf += xch[0];
        if (warp == 1) pre_excl += xch[1];
        const float dgt = suf + sGam[63] * sl + pre_excl + rc;
        const int tt = sp.t0 + t;
        if (tt < sp.end) {
          dg[((size_t)it.b * lay.Tin + tt) * lay.H + it.h] = dgt;
          dbeta[((size_t)it.b * lay.Tin + tt) * lay.H + it.h] = db;
        }
        sB[t] = bnext;
      }
      GD_TRACE_AT(ws, lay, 32 * n + 20);
      if (it.r == lay.rep - 1) {
        // l2 prologue backward (src/macai/gated_delta/_norm.py:6-9): dx = scale r (dy - x_hat (x_hat . dy)), with
        // x_hat from the q / k images (hi + lo) and the prologue's rsqrt r, both in shared memory
        const float* sRq = reinterpret_cast<const float*>(smem + S::rqk);
        const float* sRk = sRq + 64;
        float* dotq = scr;  // [64 tokens][4 head-dimension quarters]: one 16-byte read per token below
        float* dotk = scr + 4 * 64;
        const float inv_qscale = 1.f / qscale;
        GD_TRACE_AT(ws, lay, 32 * n + 24);
        // no barrier after the dg / dbeta threads: they read part, sl and xch, none of which is written here
        float x[16];
        if (norm) {  // x_hat . dy per token for q and k at once: lanes 0-15 get q's tokens, lanes 16-31 k's
          float v[32];
          row16<true>(qh, ql, dcol, tok0, x);
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = x[j] * (inv_qscale * dQ[j]);
          row16<true>(kh, kl, dcol, tok0, x);
#pragma unroll
          for (int j = 0; j < 16; ++j) v[16 + j] = x[j] * dK[j];
          const float s = warp_reduce_scatter32(v);
          ((lane < 16) ? dotq : dotk)[(tok0 + (lane & 15)) * 4 + qd] = s;
          GD_TRACE_AT(ws, lay, 32 * n + 25);
        }
        epi_sync();
        GD_TRACE_AT(ws, lay, 32 * n + 21);
        // per token, once: dx = a dy - b img with a = scale r, b = r <x_hat, dy> (img = scale x_hat, the q / k image):
        // threads 0-63 the q tokens, 64-127 the k tokens, into the partial-sum area (read by the dg threads already)
        float2* coef = reinterpret_cast<float2*>(part);  // [2][64]: q, then k
        if (norm) {
          if (tid < 128) {
            const int t = tid & 63;
            const bool isk = tid >= 64;
            const float4 d4 = *reinterpret_cast<const float4*>((isk ? dotk : dotq) + 4 * t);
            const float r = isk ? sRk[t] : sRq[t];
            coef[tid] = make_float2(isk ? r : qscale * r, r * (d4.x + d4.y + d4.z + d4.w));
          }
          epi_sync();
        }
        T* dq0 = dq + ((size_t)it.b * lay.T * lay.HK + it.hk) * DK;
        T* dk0 = dk + ((size_t)it.b * lay.T * lay.HK + it.hk) * DK;
        const int d0 = 32 * qd + 8 * (lane >> 3);
        float xk[16];
        if (norm) {
          row16<true>(qh, ql, dcol, tok0, x);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float2 ab = coef[tok0 + j];
            x[j] = fmaf(ab.x, dQ[j], -ab.y * x[j]);
          }
          row16<true>(kh, kl, dcol, tok0, xk);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float2 ab = coef[64 + tok0 + j];
            xk[j] = fmaf(ab.x, dK[j], -ab.y * xk[j]);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            x[j] = qscale * dQ[j];
            xk[j] = dK[j];
          }
        }
        GD_TRACE_AT(ws, lay, 32 * n + 26);
        if constexpr (sizeof(T) == 2) {
          // dq, dk tiles as row-major [64 tokens][DK] in the q^T / k^T image buffers (every thread is done reading
          // them), then one tensor store each (rows past T are not written); the images' next fill waits for the
          // stores' reads (qk_free: warp 0 arrives after them)
          epi_sync();
          GD_TRACE_AT(ws, lay, 32 * n + 27);
          T* sq = reinterpret_cast<T*>(smem + S::qk);
          T* sk = reinterpret_cast<T*>(smem + S::qk + DK * 64 * 2);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            sq[(tok0 + j) * DK + dcol] = cvt_out<T>(x[j]);
            sk[(tok0 + j) * DK + dcol] = cvt_out<T>(xk[j]);
          }
          fence_async_smem();
          GD_TRACE_AT(ws, lay, 32 * n + 28);
          epi_sync();
          GD_TRACE_AT(ws, lay, 32 * n + 29);
          if (tid == 0) {
            tma_store_4d(&tm_dq, 0, it.hk, t0, it.b, sq);
            tma_store_4d(&tm_dk, 0, it.hk, t0, it.b, sk);
            bulk_commit();
            bulk_wait_read0();
          }
        } else {
          store_token_rows<T>(x, dq0, (size_t)lay.HK * DK, t0 + tok0, lay.T, d0);
          store_token_rows<T>(xk, dk0, (size_t)lay.HK * DK, t0 + tok0, lay.T, d0);
        }
        mbar_arrive_warp(qk_free);  // the q / k images may be replaced by the next item's
#pragma unroll
        for (int j = 0; j < 16; ++j) dQ[j] = dK[j] = 0.f;
      }
      GD_TRACE_AT(ws, lay, 32 * n + 22);
      epi_sync();  // partials and scratch read; next beta in place
      mbar_arrive_warp(epi_done + (n & 1));
      GD_TRACE_AT(ws, lay, 32 * n + 23);
    }
    if (tid == 0) bulk_wait0();  // the tensor stores of dq / dk complete before the CTA ends
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tm, 512);
  }
  GD_TRACE_CTA(ws, lay, 1);
}

template <typename T, int DK, int DV>
cudaError_t launch_bwd_chunk(const void* q, const void* k, const void* v, const float* beta, const void* d_o, void* dq,
                             void* dk, void* dv, float* dg, float* dbeta, const Layout& lay, int flags,
                             unsigned char* ws, cudaStream_t st) {
  (void)v;
  (void)d_o;  // dO and V reach this kernel as workspace images
  using S = ChunkSmem<DK, DV>;
  auto kern = bwd_chunk_kernel<T, DK, DV>;
  static bool attr_done[kMaxDevices] = {};  // once per device: no attribute call inside a graph capture
  static int sms[kMaxDevices] = {};
  cudaError_t e = set_smem_once(kern, S::total, attr_done);
  if (e != cudaSuccess) return e;
  int dev = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (sms[dev] == 0 && (e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
    return e;
  const int ngroups = lay.B * lay.HK * lay.NT;
  const int grid = ngroups < sms[dev] ? ngroups : sms[dev];
  CUtensorMap mdq{}, mdk{}, mdv{};  // 16-bit outputs: dq / dk / dv tiles leave by tensor store (fp32 by plain stores)
  if (sizeof(T) == 2 && (!rows_map(&mdq, dq, map_dtype<T>(), lay.B, lay.T, lay.HK, DK) ||
                         !rows_map(&mdk, dk, map_dtype<T>(), lay.B, lay.T, lay.HK, DK) ||
                         !rows_map(&mdv, dv, map_dtype<T>(), lay.B, lay.T, lay.H, DV)))
    return cudaErrorInvalidValue;
  kern<<<grid, 576, S::total, st>>>(static_cast<const T*>(q), static_cast<const T*>(k), beta, static_cast<T*>(dq),
                                    static_cast<T*>(dk), static_cast<T*>(dv), dg, dbeta, lay, flags, ws, mdq, mdk, mdv);
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
