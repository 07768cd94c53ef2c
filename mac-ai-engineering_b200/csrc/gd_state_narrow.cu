// The forward state pass for few (value head, batch row) pairs: four CTAs per pair, 32 value columns each (the value
// split chosen from the pairs and the SM count, as the reference's VALUE_SPLIT rule does, src/macai/gated_delta/
// op.py:75-87).
//
// The wide pass (gd_fwd.cu) runs two CTAs per pair with the CTA's 64 value columns on the MMA's M side; a product
// cannot be narrower than M = 64 on the tensor core, so more CTAs per pair in that form would repeat the same
// per-chunk product work for fewer columns. This pass puts the tokens (or key rows) on M and the CTA's value columns
// on N:
//   (W S)_c  = W S_c          [64 tokens x 32]   M = 64,  N = 32, K = DK   (W^T image as an MN-major A operand)
//   (Q S)_c  = Q S_c          [64 tokens x 32]   M = 64,  N = 32, K = DK
//   dS_c     = K~^T Vn_c      [DK x 32]          M = 128, N = 32, K = 64   (K~ and Vn split: three products)
//   (M Vn)_c = M Vn_c         [64 tokens x 32]   M = 64,  N = 32, K = 64   (M and Vn split: three products)
// with the state S (fp32, registers) and Vn as MN-major B tiles: the same products, operand splits and fp32 epilogue
// (Vn = U - W S, S <- exp(G_last) S + dS, O = exp(G) Q S + M Vn) as the wide pass; with the operands' roles swapped
// the tensor core's fp32 sums round differently in the last bits, so the two passes agree to rounding, not bit for
// bit. Each thread owns one key row of S with 8 value columns (a 32x32b read of dS) and one token row of Vn and O
// with 4 value columns (a 16x32bx2 read): half the per-thread work of the wide pass's chunk step. Measured on one
// B200, the chunk step stays ~4k cycles all the same (the chain waits on MMA issue and drain and on the hand-offs,
// not on the per-thread work): config 3 (1 x 32768 x 32 heads) 1,041 against 1,045 us, 16 heads 1,011 against
// 1,041 us, 8 heads of 8,192 tokens 257 against 264 us. Used for the forward pass with O and without GD_STORE_STATES
// when four CTAs per pair all fit on the GPU at once (4 x pairs <= SMs) unless GD_WIDE_STATE_PASS is given; the
// drop-in passes that flag for training forwards, whose results must not depend on the mode or on how many heads
// share the call. Hand-offs, roles and stage ring are those of the wide pass: one MMA thread, one loader thread, 16
// epilogue warps.
#include "gd_common.cuh"
#include "gd_layout.cuh"

namespace gd {

constexpr int kNarrowSplit = 4;  // CTAs per (value head, batch row)

template <int DK, int DV>
struct NarrowSmem {
  static constexpr int DVH = DV / kNarrowSplit;            // value columns per CTA
  static constexpr size_t st = 0;                          // [DK x DVH] bf16 S (rows dk): B of W S and Q S
  static constexpr size_t vh = st + DK * DVH * 2;          // [64 x DVH] Vn hi (rows t): B of K~^T Vn and M Vn
  static constexpr size_t vl = vh + 64 * DVH * 2;          //                lo
  static constexpr size_t stage0 = vl + 64 * DVH * 2;      // two input stages, each (the wide pass's images):
  static constexpr size_t s_wt = 0;                        //   [DK x 64] W^T
  static constexpr size_t s_q = s_wt + DK * 64 * 2;        //   [DK x 64] q^T (hi)
  static constexpr size_t s_kt = s_q + DK * 64 * 2;        //   [2][64 x DK] K~ hi, lo
  static constexpr size_t s_m = s_kt + 2 * 64 * DK * 2;    //   [2][64 x 64] M hi, lo
  static constexpr size_t stage_bytes = s_m + 2 * 64 * 64 * 2;
  static constexpr size_t ost = stage0 + 2 * stage_bytes;  // [2][64 x DVH] O staging (row-major, 16-bit outputs)
  static constexpr size_t bar = ost + 2 * 64 * DVH * 2;
  static constexpr int NBAR = 17;
  static constexpr size_t tmem = bar + NBAR * 8;
  static constexpr size_t total = tmem + 8;
  static_assert(total <= 232448, "within the 227 KB a CTA can have");
};

template <int DK, int DV>
__device__ __forceinline__ void narrow_stage(unsigned char* stg, const unsigned char* ws, const Layout& lay,
                                             size_t cidx, uint64_t* bar) {
  using S = NarrowSmem<DK, DV>;
  mbar_arrive_expect_tx(bar, (uint32_t)S::stage_bytes);
  bulk_g2s(stg + S::s_wt, ws + lay.wt + cidx * lay.wt_bytes(), (uint32_t)lay.wt_bytes(), bar);
  bulk_g2s(stg + S::s_q, ws + lay.qk + cidx * lay.qk_bytes(), 64 * DK * 2, bar);
  bulk_g2s(stg + S::s_kt, ws + lay.kt + cidx * lay.qk_bytes(), (uint32_t)lay.qk_bytes(), bar);
  bulk_g2s(stg + S::s_m, ws + lay.m + cidx * lay.mm_bytes(), (uint32_t)lay.mm_bytes(), bar);
}

template <typename T, int DK, int DV>
__global__ void __launch_bounds__(576) state_narrow_kernel(const float* __restrict__ s0, T* __restrict__ o,
                                                           float* __restrict__ sT, Layout lay, int flags,
                                                           unsigned char* __restrict__ ws,
                                                           const __grid_constant__ CUtensorMap tm_o) {
  static_assert(DV == 128 && DK == 128, "key rows on the 128 TMEM lanes");
  using S = NarrowSmem<DK, DV>;
  constexpr int DVH = S::DVH;
  extern __shared__ __align__(1024) unsigned char smem[];
  ErrorWord* err = reinterpret_cast<ErrorWord*>(ws + lay.err);
  const int part = blockIdx.x % kNarrowSplit, h = blockIdx.x / kNarrowSplit;
  int z, b, cfirst, clast;  // as in the wide pass: states indexed by z, workspace by b, chunks [cfirst, clast)
  lay.chunks_of(ws, blockIdx.y, z, b, cfirst, clast);
  const int vbase = DVH * part;  // this CTA's first value column
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
  const int NT = clast - cfirst;
  const size_t row0 = ((size_t)b * lay.H + h) * lay.NT + cfirst;
  const int trow0 = cfirst * C;

  if (warp == 0) {
    tmem_alloc(tslot, 256);
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
  // TMEM (32 columns each): (W S) at tm, (Q S) at tm + 32 + 32 (c & 1), (M Vn) at tm + 96 + 32 (c & 1), dS at
  // tm + 160
  const uint32_t tWS = tm, tDS = tm + 160;
  const Tile tSt{smem_u32(smem + S::st), DVH};
  const Tile tVh{smem_u32(smem + S::vh), DVH}, tVl{smem_u32(smem + S::vl), DVH};
  bool ok = true;

  if (warp == 16) {
    // ---------------- MMA issuer (one thread)
    if (lane == 0) {
      if (flags & GD_TEST_WAIT_EXPIRES) ok = mbar_wait_for(never, 0, err, 28, kTestWaitCycles);
      for (int c = 0; c < NT && ok; ++c) {
        const int s = c & 1;
        const uint32_t par2 = (c >> 1) & 1;
        unsigned char* stg = smem + S::stage0 + s * S::stage_bytes;
        ok = mbar_wait(full + s, par2, err, 20) && mbar_wait(st_full, c & 1, err, 21);
        if (!ok) break;
        tc_fence_after();
        // W S and Q S: the W^T / q^T images [DK x 64] as MN-major A (M = tokens), S as MN-major B
        mma_tiles(tWS, 64, DVH, DK, Tile{smem_u32(stg + S::s_wt), 64}, false, 0, 0, tSt, true, 0, false);
        mma_commit(ws_full);
        mma_tiles(tm + 32 + 32 * s, 64, DVH, DK, Tile{smem_u32(stg + S::s_q), 64}, false, 0, 0, tSt, true, 0,
                  false);
        mma_commit(qs_full + s);
        ok = mbar_wait(vn_full, c & 1, err, 22);
        if (!ok) break;
        tc_fence_after();
        // dS = K~^T Vn: the K~ images [64 x DK] as MN-major A (M = key rows); K~ and Vn split
        const Tile tKh{smem_u32(stg + S::s_kt), DK}, tKl{smem_u32(stg + S::s_kt + 64 * DK * 2), DK};
        mma_tiles(tDS, DK, DVH, 64, tKh, false, 0, 0, tVh, true, 0, false);
        mma_tiles(tDS, DK, DVH, 64, tKh, false, 0, 0, tVl, true, 0, true);
        mma_tiles(tDS, DK, DVH, 64, tKl, false, 0, 0, tVh, true, 0, true);
        mma_commit(ds_full);
        // M Vn: the M images [64 x 64] as K-major A; M and Vn split
        const Tile tM{smem_u32(stg + S::s_m), 64}, tMl{smem_u32(stg + S::s_m + 64 * 64 * 2), 64};
        mma_tiles(tm + 96 + 32 * s, 64, DVH, 64, tM, true, 0, 0, tVh, true, 0, false);
        mma_tiles(tm + 96 + 32 * s, 64, DVH, 64, tM, true, 0, 0, tVl, true, 0, true);
        mma_tiles(tm + 96 + 32 * s, 64, DVH, 64, tMl, true, 0, 0, tVh, true, 0, true);
        mma_commit(mv_full + s);
        mma_commit(stage_free + s);
      }
    }
    __syncwarp();
  } else if (warp == 17) {
    // ---------------- stage loader (one thread)
    if (lane == 0) {
      int c = 0;
      for (; c < NT; ++c) {
        const int s = c & 1;
        if (c >= 2 && !mbar_wait(stage_free + s, ((c - 2) >> 1) & 1, err, 23)) break;
        narrow_stage<DK, DV>(smem + S::stage0 + s * S::stage_bytes, ws, lay, row0 + c, full + s);
      }
      // every copy issued here lands before the CTA may exit, also after a failed wait
      for (int l = c >= 2 ? c - 2 : 0; l < c; ++l) mbar_wait(full + (l & 1), (l >> 1) & 1, err, 29);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue warps: warp w (quadrant qd = w % 4, quarter w / 4), lane l
    //   S:     key row dk = 32 qd + l, value columns sc .. sc + 7 (sc = 8 quarter) of the CTA's 32 (fp32 registers)
    //   Vn, O: token t = 16 qd + l % 16, value columns vc .. vc + 3 (vc = 8 quarter + 4 (l / 16))
    const int qd = warp & 3, quarter = warp >> 2;
    const int dk = 32 * qd + lane, sc = 8 * quarter;
    const int t = 16 * qd + (lane & 15), vc = 8 * quarter + 4 * (lane >> 4);
    float Sr[8];
    {
      const float* p = s0 ? s0 + ((size_t)z * lay.H + h) * DK * DV + (size_t)dk * DV + vbase + sc : nullptr;
#pragma unroll
      for (int j = 0; j < 8; ++j) Sr[j] = p ? p[j] : 0.f;
      store8_bf16(smem + S::st, dk, sc, DVH, Sr);
      fence_async_smem();
      mbar_arrive_warp(st_full);
    }
    // U and G of the next chunk read from L2 one pass ahead: U[t][vbase + vc .. + 3], G_t and G_last
    float Ur[4], gcur, gcur_last, gprev = 0.f;
    auto load_u = [&](size_t cidx) {
      const float4 u = __ldg(reinterpret_cast<const float4*>(ws + lay.u + cidx * lay.u_bytes()) +
                             ((size_t)t * DV + vbase + vc) / 4);
      Ur[0] = u.x; Ur[1] = u.y; Ur[2] = u.z; Ur[3] = u.w;
      const float* gp = reinterpret_cast<const float*>(ws + lay.gc + cidx * lay.gc_bytes());
      gcur = __ldg(gp + t);
      gcur_last = __ldg(gp + 63);
    };
    load_u(row0);
    // O of chunk p: 16-bit outputs through staging buffer p & 1 and one tensor store of the CTA's [64 x 32] box
    // (thread 0; o_free / o_full as in the wide pass), fp32 outputs as 16-byte row pieces
    float o4[4] = {0.f, 0.f, 0.f, 0.f};
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
        for (int j = 0; j < 4; ++j) stg[t * DVH + vc + j] = cvt_out<T>(o4[j]);
        fence_async_smem();
        mbar_arrive_warp(o_full + bi);
        if (tid == 0) {
          if (!mbar_wait(o_full + bi, (p >> 1) & 1, err, 51)) return false;
          tma_store_4d(&tm_o, vbase, h, trow0 + p * C, b, stg);
          bulk_commit();
        }
      } else {
        const int row = trow0 + p * C + t;
        if (row < lay.T)
          *reinterpret_cast<float4*>(o + (((size_t)b * lay.T + row) * lay.H + h) * DV + vbase + vc) =
              make_float4(o4[0], o4[1], o4[2], o4[3]);
      }
      return true;
    };
    // pass c computes Vn and the state update of chunk c (c < NT) and, between them, O of chunk c - 1 (c >= 1)
    for (int c = 0; c <= NT; ++c) {
      const size_t cidx = row0 + c;
      if (c < NT) {
        // * Vn = U - W S
        if (!mbar_wait(ws_full, c & 1, err, 24)) { ok = false; break; }
        tc_fence_after();
        float acc[4];
        tmem_ld4h(tmem_lane_addr(tWS, warp, 8 * quarter), acc);
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[j] = Ur[j] - acc[j];
        store4_split(smem + S::vh, smem + S::vl, t, vc, DVH, acc);
        tc_fence_before();
        fence_async_smem();
        mbar_arrive_warp(vn_full);
      }
      if (c >= 1) {
        // * O of chunk c - 1 = diag(gamma) Q S + M Vn, formed under this chunk's state-update product (its Q S and
        // M Vn are complete: ws_full of chunk c tracks every earlier product; after the last chunk, waited here)
        const int p = c - 1, s = p & 1;
        if (c == NT &&
            (!mbar_wait(qs_full + s, (p >> 1) & 1, err, 26) || !mbar_wait(mv_full + s, (p >> 1) & 1, err, 27))) {
          ok = false;
          break;
        }
        tc_fence_after();
        float mv[4];
        tmem_ld4hx2(tmem_lane_addr(tm + 32 + 32 * s, warp, 8 * quarter), o4,
                    tmem_lane_addr(tm + 96 + 32 * s, warp, 8 * quarter), mv);
        const float gam = __expf(gprev);
#pragma unroll
        for (int j = 0; j < 4; ++j) o4[j] = fmaf(gam, o4[j], mv[j]);
        tc_fence_before();
      }
      if (c == NT) {
        if (!store_o(NT - 1)) ok = false;
        break;
      }
      const float gl = __expf(gcur_last);
      gprev = gcur;
      if (c + 1 < NT) load_u(cidx + 1);  // the next chunk's U and G while the tensor core works
      // * S <- exp(G_last) S + K~^T Vn
      if (!mbar_wait(ds_full, c & 1, err, 25)) { ok = false; break; }
      tc_fence_after();
      {
        float d[8];
        tmem_ld8(tmem_lane_addr(tDS, warp, sc), d);
#pragma unroll
        for (int j = 0; j < 8; ++j) Sr[j] = fmaf(gl, Sr[j], d[j]);
        store8_bf16(smem + S::st, dk, sc, DVH, Sr);
        tc_fence_before();
        fence_async_smem();
        mbar_arrive_warp(st_full);
      }
      if (c >= 1 && !store_o(c - 1)) {  // off the chain: the next MMAs are already unblocked
        ok = false;
        break;
      }
    }
    if (sizeof(T) == 2 && tid == 0) bulk_wait0();  // the O tensor stores complete before the CTA ends
    if (ok && sT != nullptr) {
      float* sp = sT + ((size_t)z * lay.H + h) * DK * DV + (size_t)dk * DV + vbase + sc;
#pragma unroll
      for (int j = 0; j < 8; ++j) sp[j] = Sr[j];
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tm, 256);
  }
}

template <typename T, int DK, int DV>
cudaError_t launch_state_narrow(const float* s0, void* o, float* sT, const Layout& lay, int flags, unsigned char* ws,
                                cudaStream_t st) {
  using S = NarrowSmem<DK, DV>;
  auto kern = state_narrow_kernel<T, DK, DV>;
  static bool attr_done[kMaxDevices] = {};  // once per device: no attribute call inside a graph capture
  cudaError_t e = set_smem_once(kern, S::total, attr_done);
  if (e != cudaSuccess) return e;
  dim3 grid(lay.H * kNarrowSplit, lay.packed() ? lay.N : lay.B);  // four CTAs per (head, batch row or sequence)
  CUtensorMap mo{};  // 16-bit O: chunk tiles of one CTA's 32 value columns leave by tensor store
  if (sizeof(T) == 2 && !rows_map(&mo, o, map_dtype<T>(), lay.B, lay.T, lay.H, DV, DV / kNarrowSplit))
    return cudaErrorInvalidValue;
  kern<<<grid, 576, S::total, st>>>(s0, static_cast<T*>(o), sT, lay, flags, ws, mo);
  return cudaGetLastError();
}

#define INST(T)                                                                                                  \
  template cudaError_t launch_state_narrow<T, 128, 128>(const float*, void*, float*, const Layout&, int,        \
                                                        unsigned char*, cudaStream_t);
INST(__nv_bfloat16)
INST(__half)
INST(float)
#undef INST

}  // namespace gd
