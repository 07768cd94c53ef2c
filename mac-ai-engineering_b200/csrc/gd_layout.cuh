// Workspace layout shared by the host entry points and the kernels.
//
// All intermediates of one call live in one caller-provided buffer. Per chunk (index cidx = (b * H + h) * NT + c, h a
// value head) the prep kernel writes:
//   qk   [2][64 x DK] bf16 blocked   normalised q (scaled DK^-1/2) then normalised k, the MMA-ready images
//   wt   [DK x 64]    bf16 blocked   W^T, W = A diag(beta gamma) K
//   m    [64 x 64]    bf16 blocked   M = (Q K^T) * exp(G_i - G_j), lower with the diagonal
//   u    [64][DV]     fp32           U = A diag(beta) V
//   gc   [64]         fp32           G, the in-chunk inclusive cumulative sum of g
//   qkl  [2][64 x DK] bf16 blocked   the low halves of normalised q and k (q = hi + lo to ~16 significant bits)
// and for the backward also
//   ainv [64][64]     fp32           A = (I + L)^-1
//   mf, kg [64][64]   fp32           M (with its decay mask) and K K^T
//   rq, rk [B*T*HK]   fp32           the l2 prologue's rsqrt per raw q / k row
// The state pass with GD_STORE_STATES writes sc [DK][DV] fp32 (the state entering the chunk) and vn [64][DV] fp32;
// the reverse pass writes dsn [DK][DV] fp32 (dLoss/dS_{c+1}) and dvn [64][DV] fp32.
// Every array starts on a 256-byte boundary (bulk copies need 16).
#pragma once

#include <cstddef>
#include <cstdint>

namespace gd {

struct Layout {
  int B, T, H, HK, DK, DV, NT, rep;
  size_t nch;  // B * H * NT chunks
  size_t err, qk, wt, m, u, gc, qkl, ainv, mf, kg, rq, rk, sc, vn, dsn, dvn, total;

  __host__ __device__ static size_t up(size_t x) { return (x + 255) & ~size_t(255); }

  __host__ __device__ size_t qk_bytes() const { return (size_t)2 * 64 * DK * 2; }
  __host__ __device__ size_t wt_bytes() const { return (size_t)DK * 64 * 2; }
  __host__ __device__ size_t m_bytes() const { return (size_t)64 * 64 * 2; }
  __host__ __device__ size_t u_bytes() const { return (size_t)64 * DV * 4; }
  __host__ __device__ size_t gc_bytes() const { return (size_t)64 * 4; }
  __host__ __device__ size_t ainv_bytes() const { return (size_t)64 * 64 * 4; }
  __host__ __device__ size_t s_bytes() const { return (size_t)DK * DV * 4; }

  __host__ static Layout make(int B, int T, int H, int HK, int DK, int DV, bool backward) {
    Layout L{};
    L.B = B; L.T = T; L.H = H; L.HK = HK; L.DK = DK; L.DV = DV;
    L.NT = (T + 63) / 64;
    L.rep = HK > 0 ? H / HK : 1;
    L.nch = (size_t)B * H * L.NT;
    size_t o = 0;
    L.err = o; o = up(o + 64);
    L.qk = o; o = up(o + L.nch * L.qk_bytes());
    L.wt = o; o = up(o + L.nch * L.wt_bytes());
    L.m = o; o = up(o + L.nch * L.m_bytes());
    L.u = o; o = up(o + L.nch * L.u_bytes());
    L.gc = o; o = up(o + L.nch * L.gc_bytes());
    L.qkl = o; o = up(o + L.nch * L.qk_bytes());
    if (backward) {
      L.ainv = o; o = up(o + L.nch * L.ainv_bytes());
      L.mf = o; o = up(o + L.nch * L.ainv_bytes());
      L.kg = o; o = up(o + L.nch * L.ainv_bytes());
      L.rq = o; o = up(o + (size_t)B * T * HK * 4);
      L.rk = o; o = up(o + (size_t)B * T * HK * 4);
      L.sc = o; o = up(o + L.nch * L.s_bytes());
      L.vn = o; o = up(o + L.nch * L.u_bytes());
      L.dsn = o; o = up(o + L.nch * L.s_bytes());
      L.dvn = o; o = up(o + L.nch * L.u_bytes());
    } else {
      L.ainv = L.mf = L.kg = L.rq = L.rk = L.sc = L.vn = L.dsn = L.dvn = 0;
    }
    L.total = o;
    return L;
  }
  __host__ __device__ bool backward() const { return sc != 0; }
};

}  // namespace gd
