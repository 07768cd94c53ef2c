// Reverse state pass of the chunked gated delta rule on B200 (sm_100a).
//
// Two CTAs per (value head, batch row), each owning 64 value columns (column v of dVn and dS depends on column v of dO
// and dS alone), walk the chunks last to first carrying dS = dLoss/dS (fp32, in registers):
//   dVn = M^T dO + K~ dS_{c+1}                       (K~ = diag(e) K: the decay e of the state update)
//   dS_c = exp(G_last) dS_{c+1} + (diag(gamma) Q)^T dO - W^T dVn
// (tools/check_chunk_equations.py:51-52 and src/macai/gated_delta/_chunked.py:20-24 of the reference). Only K~ dS and
// W^T dVn are on the sequential chain; M^T dO and (gamma Q)^T dO do not depend on dS and are issued one chunk ahead.
// It keeps, per chunk, the images the per-chunk gradient kernel reads: dS_{c+1}^T (hi, lo), dVn^T (hi, lo), dO, and
// the 16 partial sums of <S_c, dS_{c+1}> (S_c = hi + lo from the forward recompute's two bf16 images).
//
// Warp specialisation as in the forward pass: 16 epilogue warps reading the M = 64 products whole-warp (thread t of
// warp w: local value column 16 (w % 4) + t % 16, 8 tokens and 16 key rows of dS held in registers; they also write
// the per-chunk images to global memory straight from registers), one MMA thread and one loader thread (every refill
// waits on the product that frees its buffer, which is also the product whose next phase needs that refill); all
// hand-offs are mbarriers. Per chunk the MMA thread issues only: K~ dS (chain) -> -W^T dVn (chain, added onto the
// chunk's (gamma Q)^T dO) -> the next chunk's dS-independent products. Precision: dS and K~, dVn and W split into
// bf16 hi + lo (three products each); (gamma Q)^T dO as q^T (diag(gamma) dO) with q and gamma dO split; M split, dO
// exact in bf16.
#include "gd_common.cuh"
#include "gd_layout.cuh"

namespace gd {

template <int DK, int DV>
struct BwdStateSmem {
  static constexpr int DVH = DV / 2;                       // value columns per CTA (two CTAs per head and row)
  static constexpr size_t dsh = 0;                         // [DVH x DK] dS^T hi (rows v, cols dk)
  static constexpr size_t dsl = dsh + DVH * DK * 2;        //             lo
  static constexpr size_t dvh = dsl + DVH * DK * 2;        // [DVH x 64] dVn^T hi
  static constexpr size_t dvl = dvh + DVH * 64 * 2;        //              lo
  static constexpr size_t crit0 = dvl + DVH * 64 * 2;      // two stages of the sequential chain, each:
  static constexpr size_t c_kt = 0;                        //   [2][64 x DK] K~ hi, lo
  static constexpr size_t c_g = c_kt + 2 * 64 * DK * 2;    //   [64] G
  static constexpr size_t crit_bytes = c_g + 64 * 4;
  static constexpr size_t wt = crit0 + 2 * crit_bytes;     // [2][DK x 64] W^T hi, lo (one buffer)
  static constexpr size_t m = wt + 2 * DK * 64 * 2;        // [2][64 x 64] M hi, lo } inputs of the dS-independent
  static constexpr size_t qh = m + 2 * 64 * 64 * 2;        // [DK x 64] q^T hi  } inputs of the dS-independent
  static constexpr size_t ql = qh + DK * 64 * 2;           // [DK x 64] q^T lo  }  products, one chunk ahead
  static constexpr size_t dO = ql + DK * 64 * 2;           // [64 x DVH] dO     }
  static constexpr size_t gdo = dO + 64 * DVH * 2;         // [2][64 x DVH] diag(gamma) dO hi, lo }
  static constexpr size_t bar = gdo + 2 * 64 * DVH * 2;
  static constexpr int NBAR = 12;
  static constexpr size_t tmem = bar + NBAR * 8;
  static constexpr size_t total = tmem + 8;
  static_assert(total <= 232448, "within the 227 KB a CTA can have");
};

template <typename T, int DK, int DV>
__global__ void __launch_bounds__(576) bwd_state_kernel(const T* __restrict__ d_o, const float* __restrict__ dsT,
                                                        float* __restrict__ ds0, Layout lay, int flags,
                                                        unsigned char* __restrict__ ws) {
  static_assert(DV == 128 && DK == 128, "64 value columns per CTA on TMEM lanes 0-15 of each quadrant");
  using S = BwdStateSmem<DK, DV>;
  constexpr int DVH = S::DVH;
  extern __shared__ __align__(1024) unsigned char smem[];
  ErrorWord* err = reinterpret_cast<ErrorWord*>(ws + lay.err);
  const int half = blockIdx.x & 1, h = blockIdx.x >> 1;
  int z, b, cfirst, clast;  // z: batch row or sequence (dsT and ds0 are indexed by it); b: the workspace's batch
                            // row; the chunks [cfirst, clast) walked here
  lay.chunks_of(ws, blockIdx.y, z, b, cfirst, clast);
  const int vbase = DVH * half;  // this CTA's first value column
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (clast <= cfirst) {  // a sequence without tokens: the state's gradient passes through
    if (ds0 != nullptr)
      for (int i = tid; i < DK * DVH; i += blockDim.x) {
        const size_t at = ((size_t)z * lay.H + h) * DK * DV + (size_t)(i / DVH) * DV + vbase + i % DVH;
        ds0[at] = dsT ? dsT[at] : 0.f;
      }
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::bar);
  uint64_t* crit_full = bars + 0;   // [2] K~, G loaded
  uint64_t* wt_full = bars + 2;
  uint64_t* pre_full = bars + 3;    // M, gamma Q loaded
  uint64_t* a_full = bars + 4;      // (M^T dO)^T and ((gamma Q)^T dO)^T done
  uint64_t* b_full = bars + 5;      // (K~ dS)^T done
  uint64_t* d_full = bars + 6;      // -(W^T dVn)^T added to ((gamma Q)^T dO)^T
  uint64_t* ds_ready = bars + 7;    // 16 warps: dS tiles written
  uint64_t* do_full = bars + 8;     // 16 warps: dO tile written
  uint64_t* dvn_full = bars + 9;    // 16 warps: dVn tile written, G read
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + S::tmem);
  const int NT = clast - cfirst;                                   // chunks this CTA pair walks
  const size_t row0 = ((size_t)b * lay.H + h) * lay.NT + cfirst;  // the first one's workspace index

  if (warp == 0) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int i = 0; i < 7; ++i) mbar_init(bars + i, 1);
    for (int i = 7; i < 10; ++i) mbar_init(bars + i, 16);
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = *tslot;
  // TMEM: (M^T dO)^T at tm; (K~ dS)^T at tm + 64 as two 64-column halves (dS hi K~ hi + dS lo K~ hi | dS hi K~ lo)
  // whose sum is the product; ((gamma Q)^T dO - W^T dVn)^T at tm + 192 + 128 (n & 1)
  const uint32_t tA = tm, tB = tm + 64;
  bool ok = true;

  auto load_crit = [&](int c, int s) {
    unsigned char* st = smem + S::crit0 + s * S::crit_bytes;
    mbar_arrive_expect_tx(crit_full + s, (uint32_t)S::crit_bytes);
    bulk_g2s(st + S::c_kt, ws + lay.kt + (row0 + c) * lay.qk_bytes(), (uint32_t)lay.qk_bytes(), crit_full + s);
    bulk_g2s(st + S::c_g, ws + lay.gc + (row0 + c) * lay.gc_bytes(), (uint32_t)lay.gc_bytes(), crit_full + s);
  };
  auto load_wt = [&](int c) {
    mbar_arrive_expect_tx(wt_full, 2 * (uint32_t)lay.wt_bytes());
    bulk_g2s(smem + S::wt, ws + lay.wt + (row0 + c) * lay.wt_bytes(), (uint32_t)lay.wt_bytes(), wt_full);
    bulk_g2s(smem + S::wt + DK * 64 * 2, ws + lay.wtl + (row0 + c) * lay.wt_bytes(), (uint32_t)lay.wt_bytes(),
             wt_full);
  };
  auto prefetch_state = [&](int c) {  // S_c's hi and lo images into L2, for the epilogue's <S_c, dS_{c+1}> partials
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(ws + lay.sci + (row0 + c) * lay.si_bytes()),
                 "r"((uint32_t)lay.si_bytes())
                 : "memory");
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(ws + lay.scl + (row0 + c) * lay.si_bytes()),
                 "r"((uint32_t)lay.si_bytes())
                 : "memory");
  };
  auto load_pre = [&](int c) {
    mbar_arrive_expect_tx(pre_full, (uint32_t)(lay.mm_bytes() + lay.qk_bytes()));
    bulk_g2s(smem + S::m, ws + lay.m + (row0 + c) * lay.mm_bytes(), (uint32_t)lay.mm_bytes(), pre_full);
    bulk_g2s(smem + S::qh, ws + lay.qk + (row0 + c) * lay.qk_bytes(), DK * 64 * 2, pre_full);   // the q halves of
    bulk_g2s(smem + S::ql, ws + lay.qkl + (row0 + c) * lay.qk_bytes(), DK * 64 * 2, pre_full);  //  the q / k images
  };
  const Tile tDO{smem_u32(smem + S::dO), DVH};
  // (M^T dO)^T = dO^T M [DVH x 64] (M hi + lo); ((gamma Q)^T dO)^T [DVH x DK] as below
  auto issue_pre = [&](int n) {
    mma_tiles(tA, DVH, 64, 64, tDO, false, 0, 0, Tile{smem_u32(smem + S::m), 64}, true, 0, false);
    mma_tiles(tA, DVH, 64, 64, tDO, false, 0, 0, Tile{smem_u32(smem + S::m + 64 * 64 * 2), 64}, true, 0, true);
    const uint32_t tC = tm + 192 + 128 * (n & 1);
    // ((gamma Q)^T dO)^T = (diag(gamma) dO)^T Q: gamma dO and q split, q^T images as K-major B
    const Tile tGh{smem_u32(smem + S::gdo), DVH}, tGl{smem_u32(smem + S::gdo + 64 * DVH * 2), DVH};
    const Tile tQh{smem_u32(smem + S::qh), 64}, tQl{smem_u32(smem + S::ql), 64};
    mma_tiles(tC, DVH, DK, 64, tGh, false, 0, 0, tQh, false, 0, false);
    mma_tiles(tC, DVH, DK, 64, tGh, false, 0, 0, tQl, false, 0, true);
    mma_tiles(tC, DVH, DK, 64, tGl, false, 0, 0, tQh, false, 0, true);
    mma_commit(a_full);
  };

  if (warp == 16) {
    // ---------------- MMA issuer (one thread); iteration n handles chunk c = NT - 1 - n
    if (lane == 0) {
      ok = mbar_wait(pre_full, 0, err, 30) && mbar_wait(do_full, 0, err, 31);
      if (ok) {
        tc_fence_after();
        issue_pre(0);
      }
      for (int n = 0; n < NT && ok; ++n) {
        const int c = NT - 1 - n, s = n & 1;
        unsigned char* st = smem + S::crit0 + s * S::crit_bytes;
        ok = mbar_wait(crit_full + s, (n >> 1) & 1, err, 32) && mbar_wait(ds_ready, n & 1, err, 33);
        if (!ok) break;
        GD_TRACE_ONE(ws, lay, 1024 + 8 * n + 0);
        tc_fence_after();
        // * (K~ dS)^T = dS^T K~^T [DVH x 64]: dS hi against [K~ hi; K~ lo] (the two images are adjacent: one N = 128
        // operand) into both halves, then dS lo K~ hi onto the first half
        const Tile tKh{smem_u32(st + S::c_kt), DK};
        const Tile tDh{smem_u32(smem + S::dsh), DK}, tDl{smem_u32(smem + S::dsl), DK};
        mma_tiles(tB, DVH, 128, DK, tDh, true, 0, 0, tKh, false, 0, false);
        mma_tiles(tB, DVH, 64, DK, tDl, true, 0, 0, tKh, false, 0, true);
        mma_commit(b_full);
        GD_TRACE_ONE(ws, lay, 1024 + 8 * n + 1);
        ok = mbar_wait(dvn_full, n & 1, err, 35) && mbar_wait(wt_full, n & 1, err, 36);
        if (!ok) break;
        GD_TRACE_ONE(ws, lay, 1024 + 8 * n + 3);
        tc_fence_after();
        // * -(W^T dVn)^T = -dVn^T W [DVH x DK], onto this chunk's ((gamma Q)^T dO)^T, dVn and W split (three
        // products: with nearly parallel keys W^T dVn cancels to a small fraction of its terms)
        {
          const uint32_t tC = tm + 192 + 128 * (n & 1);
          const Tile tVh{smem_u32(smem + S::dvh), 64}, tVl{smem_u32(smem + S::dvl), 64};
          const Tile tWh{smem_u32(smem + S::wt), 64}, tWl{smem_u32(smem + S::wt + DK * 64 * 2), 64};
          mma_tiles(tC, DVH, DK, 64, tVh, true, 0, 0, tWh, false, 0, true, true);
          mma_tiles(tC, DVH, DK, 64, tVl, true, 0, 0, tWh, false, 0, true, true);
          mma_tiles(tC, DVH, DK, 64, tVh, true, 0, 0, tWl, false, 0, true, true);
        }
        mma_commit(d_full);
        GD_TRACE_ONE(ws, lay, 1024 + 8 * n + 4);
        if (c > 0) {  // the next chunk's dS-independent products, under this chunk's dS update
          ok = mbar_wait(pre_full, (n + 1) & 1, err, 39) && mbar_wait(do_full, (n + 1) & 1, err, 40);
          if (!ok) break;
          tc_fence_after();
          issue_pre(n + 1);
        }
        GD_TRACE_ONE(ws, lay, 1024 + 8 * n + 5);
      }
    }
    __syncwarp();
  } else if (warp == 17) {
    // ---------------- loader (one thread). Each refill waits for the product that frees its buffer; that product's
    // barrier cannot move on a further phase before this refill (its next phase needs the refilled data).
    if (lane == 0) {
      int nl = 0, nw = 0, np = 0;  // crit stages, W^T and pre loads issued
      load_crit(NT - 1, 0);
      ++nl;
      if (NT > 1) {
        load_crit(NT - 2, 1);
        ++nl;
      }
      load_wt(NT - 1);
      load_pre(NT - 1);
      prefetch_state(NT - 1);
      ++nw;
      ++np;
      for (int n = 0; n + 1 < NT && ok; ++n) {
        const int c = NT - 1 - n;
        ok = mbar_wait(a_full, n & 1, err, 34);  // chunk c's dS-independent products have read M and gamma Q
        if (!ok) break;
        // the next chunk's fp32 state into L2, for the epilogue's <S, dS> partial sums
        prefetch_state(c - 1);
        load_pre(c - 1);
        ++np;
        ok = mbar_wait(d_full, n & 1, err, 38);  // -W^T dVn of chunk c has read W^T; K~ dS read stage n & 1
        if (!ok) break;
        load_wt(c - 1);
        ++nw;
        if (c > 1) {
          load_crit(c - 2, n & 1);
          ++nl;
        }
      }
      // every copy issued here lands before the CTA may exit, also after a failed wait
      for (int l = nl > 2 ? nl - 2 : 0; l < nl; ++l) mbar_wait(crit_full + (l & 1), (l >> 1) & 1, err, 44);
      mbar_wait(wt_full, (nw - 1) & 1, err, 45);
      mbar_wait(pre_full, (np - 1) & 1, err, 46);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue warps: thread t of warp w holds local value column 16 (w % 4) + t % 16, tokens
    // 16 (w / 4) + 8 (t / 16) .. + 7 of the [64 x 64] products and key rows 32 (w / 4) + 16 (t / 16) .. + 15 of dS
    const int qd = warp & 3, quarter = warp >> 2;
    const int vl_ = 16 * qd + (lane & 15), v = vbase + vl_;
    const int tk = 16 * quarter + 8 * (lane >> 4);
    const int dk0 = 32 * quarter + 16 * (lane >> 4);
    float Dr[16];  // dS[dk0 + j][v]
    // the dS tiles for the next K~ dS, then (after the hand-off: the proxy fence would wait for global stores in
    // flight) this CTA's rows of chunk ci's dS_{ci+1}^T images (hi, lo) for the per-chunk kernel, from registers
    auto write_ds = [&](int ci) {
      uint4 h[2], l[2];
#pragma unroll
      for (int q8 = 0; q8 < 2; ++q8) {
        split8_bf16(Dr + 8 * q8, h[q8], l[q8]);
        store8_pair(smem + S::dsh, smem + S::dsl, vl_, dk0 + 8 * q8, DK, h[q8], l[q8]);
      }
      fence_async_smem();
      mbar_arrive_warp(ds_ready);
      unsigned char* gh = ws + lay.dsi + (row0 + ci) * 2 * lay.si_bytes() + (size_t)vbase * DK * 2;
#pragma unroll
      for (int q8 = 0; q8 < 2; ++q8) store8_pair(gh, gh + lay.si_bytes(), vl_, dk0 + 8 * q8, DK, h[q8], l[q8]);
    };
    // a chunk's dO tile (this CTA's 64 columns): 512 16-byte pieces, one per thread, eight consecutive threads per
    // 128-byte core matrix; fetched raw into registers early, written to the tile once the tile's readers are done
    Piece<T> dox;
    float dog = 0.f;  // G of the piece's token
    const int prl = tid & 7, pcb = (tid >> 3) & 7, prb = tid >> 6;
    auto fetch_do = [&](int c) {  // rows of the chunk's span in the caller's dO (zero past the sequence's end)
      const ChunkSpan sp = lay.span(ws, cfirst + c);
      const int t = sp.t0 + 8 * prb + prl;
      if (d_o != nullptr && t < sp.end) {
        dox.load(d_o + (((size_t)b * lay.Tin + t) * lay.H + h) * DV + vbase + 8 * pcb);
      } else {
        dox.zero();
      }
      dog = __ldg(reinterpret_cast<const float*>(ws + lay.gc + (row0 + c) * lay.gc_bytes()) + 8 * prb + prl);
    };
    // chunk c's dO: the tile and diag(gamma) dO split hi / lo (with q's images, (gamma Q)^T dO without a gamma Q
    // image), then this CTA's columns of the [64 x DV] dO image
    auto put_do = [&](int c) {
      float x[8], y[8];
      dox.to_f32(x);
      const float gam = __expf(dog);
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = gam * x[j];
      store8_bf16(smem + S::dO, 8 * prb + prl, 8 * pcb, DVH, x);
      store8_split(smem + S::gdo, smem + S::gdo + 64 * DVH * 2, 8 * prb + prl, 8 * pcb, DVH, y);
      fence_async_smem();
      mbar_arrive_warp(do_full);
      store8_bf16(ws + lay.doi + (row0 + c) * lay.vi_bytes(), 8 * prb + prl, vbase + 8 * pcb, DV, x);
    };
    {
      const float* p = dsT ? dsT + ((size_t)z * lay.H + h) * DK * DV : nullptr;
#pragma unroll
      for (int j = 0; j < 16; ++j) Dr[j] = p ? p[(size_t)(dk0 + j) * DV + v] : 0.f;
      write_ds(NT - 1);
      fetch_do(NT - 1);
      put_do(NT - 1);
    }
    for (int n = 0; n < NT; ++n) {
      const int c = NT - 1 - n, s = n & 1;
      const size_t cidx = row0 + c;
      const float* sG = reinterpret_cast<const float*>(smem + S::crit0 + s * S::crit_bytes + S::c_g);
      if (c > 0) fetch_do(c - 1);  // the next chunk's dO, in flight during this chunk's waits
      // * dVn = M^T dO + K~ dS_{c+1}
      GD_TRACE_AT(ws, lay, 8 * n + 0);
      if (!mbar_wait(b_full, n & 1, err, 41) || !mbar_wait(a_full, n & 1, err, 42)) { ok = false; break; }
      tc_fence_after();
      GD_TRACE_AT(ws, lay, 8 * n + 1);
      const float gl = __expf(sG[63]);
      {
        float a[8], bb[8], b2[8];
        tmem_ld8hx3(tmem_lane_addr(tA, warp, 16 * quarter), a, tmem_lane_addr(tB, warp, 16 * quarter), bb,
                    tmem_lane_addr(tB + 64, warp, 16 * quarter), b2);
#pragma unroll
        for (int j = 0; j < 8; ++j) a[j] += bb[j] + b2[j];
        uint4 hi, lo;
        split8_bf16(a, hi, lo);
        store8_pair(smem + S::dvh, smem + S::dvl, vl_, tk, 64, hi, lo);
        tc_fence_before();
        fence_async_smem();
        mbar_arrive_warp(dvn_full);
        unsigned char* gi = ws + lay.dvni + cidx * lay.vn_bytes();  // the image's halves straight from registers
        store8_pair(gi, gi + DV * 64 * 2, v, tk, 64, hi, lo);
      }
      GD_TRACE_AT(ws, lay, 8 * n + 2);
      // the next chunk's dO tile (this chunk's dO products are done: a_full), published before any new load is in
      // flight
      if (c > 0) put_do(c - 1);
      // partial <S_c, dS_{c+1}> of this thread's 16 entries: S_c = hi + lo from the forward recompute's two bf16
      // images (row v, key rows dk0 .. dk0 + 15: two 16-byte pieces each; prefetched into L2 a chunk ahead), dS_{c+1}
      // exact in registers; loads in flight through the wait for -(W^T dVn)^T
      const unsigned char* sch = ws + lay.sci + cidx * lay.si_bytes();
      const unsigned char* scl = ws + lay.scl + cidx * lay.si_bytes();
      const uint4 sh0 = __ldg(reinterpret_cast<const uint4*>(sch + blk_off(v, dk0, DK)));
      const uint4 sh1 = __ldg(reinterpret_cast<const uint4*>(sch + blk_off(v, dk0 + 8, DK)));
      const uint4 sl0 = __ldg(reinterpret_cast<const uint4*>(scl + blk_off(v, dk0, DK)));
      const uint4 sl1 = __ldg(reinterpret_cast<const uint4*>(scl + blk_off(v, dk0 + 8, DK)));
      // * dS_c = exp(G_last) dS_{c+1} + (gamma Q)^T dO - W^T dVn
      GD_TRACE_AT(ws, lay, 8 * n + 3);
      if (!mbar_wait(d_full, n & 1, err, 43)) { ok = false; break; }
      tc_fence_after();
      GD_TRACE_AT(ws, lay, 8 * n + 4);
      float sacc = 0.f;
      {
        const uint32_t wh[8] = {sh0.x, sh0.y, sh0.z, sh0.w, sh1.x, sh1.y, sh1.z, sh1.w};  // bf16 pairs, low half first
        const uint32_t wl[8] = {sl0.x, sl0.y, sl0.z, sl0.w, sl1.x, sl1.y, sl1.z, sl1.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float s0 = __uint_as_float(wh[e] << 16) + __uint_as_float(wl[e] << 16);
          const float s1 = __uint_as_float(wh[e] & 0xffff0000u) + __uint_as_float(wl[e] & 0xffff0000u);
          sacc = fmaf(s0, Dr[2 * e], sacc);
          sacc = fmaf(s1, Dr[2 * e + 1], sacc);
        }
      }
      {
        float cc[16];
        tmem_ld16h(tmem_lane_addr(tm + 192 + 128 * (n & 1), warp, 32 * quarter), cc);
#pragma unroll
        for (int j = 0; j < 16; ++j) Dr[j] = fmaf(gl, Dr[j], cc[j]);
        tc_fence_before();
      }
      if (c > 0) write_ds(c - 1);
      // the warp's partial sum goes out after the hand-off (the proxy fence there would wait for the store)
      sacc = warp_sum(sacc);
      if (lane == 0) reinterpret_cast<float*>(ws + lay.sl + cidx * lay.sl_bytes())[16 * half + warp] = sacc;
      GD_TRACE_AT(ws, lay, 8 * n + 5);
    }
    if (ok && ds0 != nullptr) {
      float* p = ds0 + ((size_t)z * lay.H + h) * DK * DV;
#pragma unroll
      for (int j = 0; j < 16; ++j) p[(size_t)(dk0 + j) * DV + v] = Dr[j];
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
cudaError_t launch_bwd_state(const void* d_o, const float* dsT, float* ds0, const Layout& lay, int flags,
                             unsigned char* ws, cudaStream_t st) {
  using S = BwdStateSmem<DK, DV>;
  auto kern = bwd_state_kernel<T, DK, DV>;
  static bool attr_done[kMaxDevices] = {};
  cudaError_t e = set_smem_once(kern, S::total, attr_done);
  if (e != cudaSuccess) return e;
  dim3 grid(lay.H * 2, lay.packed() ? lay.N : lay.B);  // one CTA pair per (head, batch row or sequence)
  kern<<<grid, 576, S::total, st>>>(static_cast<const T*>(d_o), dsT, ds0, lay, flags, ws);
  return cudaGetLastError();
}

#define INST(T)                                                                                                    \
  template cudaError_t launch_bwd_state<T, 128, 128>(const void*, const float*, float*, const Layout&, int,         \
                                                     unsigned char*, cudaStream_t);
INST(__nv_bfloat16)
INST(__half)
INST(float)
#undef INST

}  // namespace gd
