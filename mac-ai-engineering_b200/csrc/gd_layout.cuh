// Workspace layout shared by the host entry points and the kernels.
//
// All intermediates of one call live in one caller-provided buffer. Per chunk (index cidx = (b * H + h) * NT + c, h a
// value head), "image" = an MMA-ready bf16 tile in the blocked layout of gd_common.cuh, copied to and from shared
// memory whole by the bulk-copy engine. The prep kernel writes:
//   qk   [2][DK x 64] image   normalised q (scaled), then normalised k (bf16 high halves), transposed (rows d); the
//                             k half only for the backward
//   kt   [2][64 x DK] image   K~ = diag(e) K, e_i = exp(G_last - G_i): hi, then lo (the state updates' operand)
//   wt   [DK x 64]    image   W^T, W = A diag(beta gamma) K
//   m    [2][64 x 64] image   M = (Q K^T) * exp(G_i - G_j), lower with the diagonal: hi, then lo
//   u    [64][DV]     fp32    U = A diag(beta) V
//   gc   [64]         fp32    G, the in-chunk inclusive cumulative sum of g
// and for the backward also
//   qkl  [2][DK x 64] image   the low halves of qk (q = hi + lo to ~16 significant bits)
//   ai   [2][64 x 64] image   A = (I + L)^-1: hi, then lo
//   wtl  [DK x 64]    image   the low half of wt (W^T = hi + lo)
//   vi   [DV x 64]    image   V^T
//   rq, rk [B][HK][NT * 64] fp32  the l2 prologue's rsqrt per raw q / k row (a chunk's 64 rows contiguous)
// The state pass with GD_STORE_STATES writes per chunk (S_c the state entering the chunk)
//   sci  [DV x DK]    image   S_c^T, bf16 (its high half)
//   scl  [DV x DK]    image   the low half of S_c^T (S_c = hi + lo to ~16 significant bits)
//   vni  [2][DV x 64] image   Vn^T: hi, then lo
// and the reverse pass
//   dsi  [2][DV x DK] image   dS_{c+1}^T: hi, then lo
//   dvni [2][DV x 64] image   dVn^T: hi, then lo
//   doi  [64 x DV]    image   dO
//   sl   [32]         fp32    partial sums of <S_c, dS_{c+1}> (one per epilogue warp of the chunk's two CTAs)
// Packed rows (N > 0 sequences of lengths from cu_seqlens, concatenated in the caller's arrays as one batch row of Tin
// rows): B = 1, each sequence starts a new chunk, NT = Tin / 64 + N bounds the chunk count (every sequence adds at most
// one partial chunk) and T = NT * 64 is the chunk-aligned row count. Then also
//   ctab [NT]   int2     chunk c's first row in the caller's arrays and its sequence's end row (rows t with
//                        t0 <= t < end are the chunk's; (0, 0) for chunks past the last sequence's)
//   seg  [N+1]  int      each sequence's first chunk; seg[N] = the chunks in use
//   ord  [N]    int      the sequences by descending chunk count: the state passes' grid row z walks sequence
//                        ord[z], so the longest chains start first (the block scheduler dispatches rows in order)
//   opad / dqpad / dkpad / dvpad  [T][heads][D] in the caller's dtype (4 bytes an element reserved): the chunk-aligned
//                        o, dq, dk, dv the kernels write, scattered to the caller's packed rows afterwards
// Every array starts on a 256-byte boundary (bulk copies need 16).
#pragma once

#include <cstddef>
#include <cstdint>

namespace gd {

// chunk c's rows in the caller's token arrays: rows t0 .. t0 + 63, those below `end` valid
struct ChunkSpan {
  int t0, end;
};

struct Layout {
  int B, T, H, HK, DK, DV, NT, rep;
  int N;    // packed rows: the number of sequences (0: a [B, T] batch)
  int Tin;  // rows a batch row has in the caller's token arrays (T, or the packed total)
  size_t nch;  // B * H * NT chunks
  size_t err, trace, ctab, seg, ord, opad, dqpad, dkpad, dvpad, qk, qkl, kt, wt, m, u, gc;
  size_t ai, wtl, vi, rq, rk, sci, scl, vni, dsi, dvni, doi, sl, total;

  __host__ __device__ static size_t up(size_t x) { return (x + 255) & ~size_t(255); }

  __host__ __device__ size_t qk_bytes() const { return (size_t)2 * 64 * DK * 2; }   // a [2][64 x DK] image pair
  __host__ __device__ size_t wt_bytes() const { return (size_t)DK * 64 * 2; }
  __host__ __device__ size_t m_bytes() const { return (size_t)64 * 64 * 2; }       // one C x C image
  __host__ __device__ size_t mm_bytes() const { return (size_t)2 * 64 * 64 * 2; }  // the M hi / lo pair
  __host__ __device__ size_t u_bytes() const { return (size_t)64 * DV * 4; }
  __host__ __device__ size_t gc_bytes() const { return (size_t)64 * 4; }
  __host__ __device__ size_t vi_bytes() const { return (size_t)64 * DV * 2; }
  __host__ __device__ size_t si_bytes() const { return (size_t)DK * DV * 2; }      // one state image
  __host__ __device__ size_t vn_bytes() const { return (size_t)2 * DV * 64 * 2; }  // a [2][DV x 64] image pair
  __host__ __device__ size_t sl_bytes() const { return (size_t)32 * 4; }           // <S, dS> partial sums

  // N > 0: packed rows, T = the packed total (B must be 1)
  __host__ static Layout make(int B, int T, int H, int HK, int DK, int DV, bool backward, int N = 0) {
    Layout L{};
    L.B = B; L.H = H; L.HK = HK; L.DK = DK; L.DV = DV;
    L.N = N;
    L.Tin = T;
    L.NT = N > 0 ? T / 64 + N : (T + 63) / 64;
    L.T = N > 0 ? L.NT * 64 : T;
    L.rep = HK > 0 ? H / HK : 1;
    L.nch = (size_t)B * H * L.NT;
    size_t o = 0;
    auto take = [&](size_t bytes) { size_t at = o; o = up(o + bytes); return at; };
    L.err = take(64);
#ifdef GD_TRACE
    L.trace = take(4 * 4096 * 8);  // phase timestamps (profiling builds only)
#else
    L.trace = 0;
#endif
    L.ctab = L.seg = L.ord = L.opad = L.dqpad = L.dkpad = L.dvpad = 0;
    if (N > 0) {
      L.ctab = take((size_t)L.NT * 8);
      L.seg = take((size_t)(N + 1) * 4);
      L.ord = take((size_t)N * 4);
      L.opad = take((size_t)L.T * H * DV * 4);
      if (backward) {
        L.dqpad = take((size_t)L.T * HK * DK * 4);
        L.dkpad = take((size_t)L.T * HK * DK * 4);
        L.dvpad = take((size_t)L.T * H * DV * 4);
      }
    }
    L.qk = take(L.nch * L.qk_bytes());
    L.kt = take(L.nch * L.qk_bytes());
    L.wt = take(L.nch * L.wt_bytes());
    L.m = take(L.nch * L.mm_bytes());
    L.u = take(L.nch * L.u_bytes());
    L.gc = take(L.nch * L.gc_bytes());
    if (backward) {
      L.qkl = take(L.nch * L.qk_bytes());
      L.ai = take(L.nch * L.mm_bytes());
      L.wtl = take(L.nch * L.wt_bytes());
      L.vi = take(L.nch * L.vi_bytes());
      L.rq = take((size_t)B * HK * L.NT * 64 * 4);
      L.rk = take((size_t)B * HK * L.NT * 64 * 4);
      L.sci = take(L.nch * L.si_bytes());
      L.scl = take(L.nch * L.si_bytes());
      L.vni = take(L.nch * L.vn_bytes());
      L.dsi = take(L.nch * 2 * L.si_bytes());
      L.dvni = take(L.nch * L.vn_bytes());
      L.doi = take(L.nch * L.vi_bytes());
      L.sl = take(L.nch * L.sl_bytes());
    } else {
      L.qkl = L.ai = L.wtl = L.vi = L.rq = L.rk = L.sci = L.scl = L.vni = L.dsi = L.dvni = L.doi = L.sl = 0;
    }
    L.total = o;
    return L;
  }
  __host__ __device__ bool backward() const { return sci != 0; }
  __host__ __device__ bool packed() const { return N > 0; }

  // chunk c's rows (regular batches: c * 64 up to T; packed rows: from the chunk table)
  __device__ ChunkSpan span(const unsigned char* ws, int c) const {
    if (N == 0) return ChunkSpan{c * 64, T};
    const int2 e = reinterpret_cast<const int2*>(ws + ctab)[c];
    return ChunkSpan{e.x, e.y};
  }
  // the chunks a state pass walks for grid row y: [first, last) of batch row y, or of sequence ord[y] (returned in
  // z: the index of the row's states)
  __device__ void chunks_of(const unsigned char* ws, int y, int& z, int& b, int& first, int& last) const {
    if (N == 0) {
      z = b = y;
      first = 0;
      last = NT;
    } else {
      const int* sg = reinterpret_cast<const int*>(ws + seg);
      z = reinterpret_cast<const int*>(ws + ord)[y];
      b = 0;
      first = sg[z];
      last = sg[z + 1];
    }
  }
};

}  // namespace gd
