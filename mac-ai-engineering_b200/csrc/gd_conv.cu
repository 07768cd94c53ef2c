// The linear-attention layer's convolution path in one pass each way (the step that produces the rule's q, k, v),
// mirroring the reference's conv_fwd / conv_bwd kernels (src/macai/layer/_conv.py:1-21 formulas, :52-137 kernels,
// :159-167 weight-gradient sum) and its autograd function (:188-237):
//   u[t, c] = sum_j w[c, j] x[t - 3 + j, c]        (kernel 4, no bias, zero before the sequence start; fp32)
//   y = u sigmoid(u)                               (on the fp32 u, one rounding)
//   q, k = y's first two KD-channel blocks as [B, T, H_v, DK] in x's dtype, each key head written REP times (the
//          repeat_interleave of q and k over the value heads, without a copy); v = the last VD channels as
//          [B, T, H_v, DV] in fp32
// backward (x saved; u recomputed):
//   du = dy sigmoid(u) (1 + u (1 - sigmoid(u)))   (dy of q and k summed over the REP value heads a key head serves)
//   dx[t, c] = sum_j w[c, j] du[t + 3 - j, c]     (du = 0 past the sequence end), [B, T, C] in x's dtype
//   dw[c, j] = sum_{b, t} du[t, c] x[t - 3 + j, c] (when asked: fp32 partial rows in a fixed order, then a tree sum)
// A thread owns 4 adjacent channels and walks a tile of L time steps, with a batch of rows' loads in flight at once,
// keeping the last three inputs (and in the backward the last three du) in registers: each x row is read once per
// tile plus a 3-row halo, q / k / v rows are written once (q, k REP times). HBM-bound, with no shared memory.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

#include "gated_delta_b200.h"

namespace {

constexpr int kThreads = 256;
constexpr int kTileF = 32;       // time steps a forward thread walks (L)
constexpr int kFillCTAs = 2 * 2 * 148;  // backward: two waves of 2 CTAs an SM on 148 SMs (see tile_for)
constexpr int kBatch = 4;        // forward: x rows loaded before any is used
constexpr int kBatchB = 4;       // backward: x and cotangent rows loaded before any is used
constexpr int kMaxPartials = 256;  // partial rows of dw: tiles are grouped into at most this many row blocks
constexpr int kMaxGridY = 65535;

template <typename T>
struct Vec {
  static constexpr int V = 4;  // channels a thread (8 bytes of x at 16 bits, 16 at fp32): the taps, the rows of
                               // history and a batch of rows in flight fit in registers
};

// 4 channels of T <-> float
__device__ __forceinline__ void ld(const float* p, float (&v)[4]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
}
__device__ __forceinline__ void st(float* p, const float (&v)[4]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}
// 4 channels of a 16-bit type (8 bytes)
template <typename T>
__device__ __forceinline__ void ld(const T* p, float (&v)[4]) {
  const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
  float2 a, b;
  if constexpr (std::is_same<T, __half>::value) {
    a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  } else {
    a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
    b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  }
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}
__device__ __forceinline__ uint32_t pack2(float a, float b, const __nv_bfloat16*) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}
__device__ __forceinline__ uint32_t pack2(float a, float b, const __half*) {
  const __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}
template <typename T>
__device__ __forceinline__ void st(T* p, const float (&v)[4]) {
  const T* tag = nullptr;
  *reinterpret_cast<uint2*>(p) = make_uint2(pack2(v[0], v[1], tag), pack2(v[2], v[3], tag));
}
// V fp32 values (v and dv, 16-byte aligned)
template <int V>
__device__ __forceinline__ void ldf(const float* p, float (&v)[V]) {
#pragma unroll
  for (int i = 0; i < V; i += 4) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p + i));
    v[i] = a.x; v[i + 1] = a.y; v[i + 2] = a.z; v[i + 3] = a.w;
  }
}
template <int V>
__device__ __forceinline__ void stf(float* p, const float (&v)[V]) {
#pragma unroll
  for (int i = 0; i < V; i += 4) *reinterpret_cast<float4*>(p + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
}

template <typename TW>
__device__ __forceinline__ float ldw(const TW* p) {
  if constexpr (sizeof(TW) == 4) {
    return __ldg(p);
  } else if constexpr (std::is_same<TW, __half>::value) {
    return __half2float(p[0]);
  } else {
    return __bfloat162float(p[0]);
  }
}

template <typename T>
__device__ __forceinline__ T cvt(float x);
template <>
__device__ __forceinline__ float cvt<float>(float x) { return x; }
template <>
__device__ __forceinline__ __half cvt<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 cvt<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// silu(u) = u / (1 + exp(-u)) and sigmoid(u) with the fast divide (2 ulp; a denominator past 2^126, u < -87, gives 0)
__device__ __forceinline__ float silu(float u) { return __fdividef(u, 1.f + expf(-u)); }
__device__ __forceinline__ float sigmoid(float u) { return __fdividef(1.f, 1.f + expf(-u)); }

// where channel c's outputs go: q (c < KD) or k (KD <= c < 2 KD), key head h, column d (the REP copies at
// h REP DK + r DK + d of a [H_v DK] row); or v (c >= 2 KD), column cc of a [VD] row
struct Route {
  bool isv;
  bool isk;
  int cc;
  long long qcol;
};
__device__ __forceinline__ Route route(int c, int KD, int DK, int REP) {
  Route r;
  r.isv = c >= 2 * KD;
  r.isk = !r.isv && c >= KD;
  r.cc = r.isv ? c - 2 * KD : (r.isk ? c - KD : c);
  const int h = r.cc / DK, d = r.cc % DK;
  r.qcol = (long long)h * REP * DK + d;
  return r;
}

template <typename TW, int V>
__device__ __forceinline__ void load_taps(const TW* w, int c, float (&tp)[4][V]) {
#pragma unroll
  for (int i = 0; i < V; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) tp[j][i] = ldw(w + (size_t)(c + i) * 4 + j);
}

// grid (channel groups / 256, tiles of L steps, batch rows)
template <typename T, typename TW>
__global__ void __launch_bounds__(kThreads, 4) conv_fwd_kernel(const T* __restrict__ x, const TW* __restrict__ w,
                                                            T* __restrict__ qo, T* __restrict__ ko,
                                                            float* __restrict__ vo, int Tn, int C, int KD, int DK,
                                                            int REP) {
  constexpr int V = Vec<T>::V;
  const int c = (blockIdx.x * kThreads + threadIdx.x) * V;
  if (c >= C) return;
  const int t0 = blockIdx.y * kTileF, b = blockIdx.z;
  float tp[4][V];
  load_taps<TW, V>(w, c, tp);
  const T* xb = x + (size_t)b * Tn * C + c;
  float xm3[V], xm2[V], xm1[V];
#pragma unroll
  for (int i = 0; i < V; ++i) xm3[i] = xm2[i] = xm1[i] = 0.f;
  if (t0 >= 3) ld(xb + (size_t)(t0 - 3) * C, xm3);
  if (t0 >= 2) ld(xb + (size_t)(t0 - 2) * C, xm2);
  if (t0 >= 1) ld(xb + (size_t)(t0 - 1) * C, xm1);
  const Route rt = route(c, KD, DK, REP);
  const long long qrow = (long long)KD * REP, vrow = C - 2 * KD;
  const long long bt0 = (long long)b * Tn + t0;
  // running pointers at row t0, advanced a row at a time
  const T* xp = xb + (size_t)t0 * C;
  T* qkp = rt.isv ? nullptr : (rt.isk ? ko : qo) + bt0 * qrow + rt.qcol;
  float* vp = rt.isv ? vo + bt0 * vrow + rt.cc : nullptr;
  const int te = t0 + kTileF < Tn ? t0 + kTileF : Tn;
  // kBatch rows of x in flight before any is used
  for (int tb = t0; tb < te; tb += kBatch) {
    const int n = te - tb;
    float xr[kBatch][V];
#pragma unroll
    for (int s = 0; s < kBatch; ++s) {
#pragma unroll
      for (int i = 0; i < V; ++i) xr[s][i] = 0.f;
      if (s < n) ld(xp + (size_t)s * C, xr[s]);
    }
    xp += (size_t)kBatch * C;
#pragma unroll
    for (int s = 0; s < kBatch; ++s) {
      if (s >= n) break;
      float y[V];
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const float u =
            fmaf(tp[3][i], xr[s][i], fmaf(tp[2][i], xm1[i], fmaf(tp[1][i], xm2[i], tp[0][i] * xm3[i])));
        y[i] = silu(u);
        xm3[i] = xm2[i];
        xm2[i] = xm1[i];
        xm1[i] = xr[s][i];
      }
      if (rt.isv) {
        stf<V>(vp, y);
        vp += vrow;
      } else {
        for (int r = 0; r < REP; ++r) st(qkp + (long long)r * DK, y);
        qkp += qrow;
      }
    }
  }
}

// grid (channel groups / 256, row blocks): row block p walks tiles [p tpb, (p + 1) tpb) of the (batch row, tile)
// order; with DW its fp32 sums of du x go to partial row p ([P, C, 4]). RP: REP known at compile time (1 or 2: every
// cotangent load of a batch in flight at once), or 0 (REP read at run time).
template <typename T, typename TW, bool DW, int RP>
__global__ void __launch_bounds__(kThreads, 2) conv_bwd_kernel(const T* __restrict__ x, const TW* __restrict__ w,
                                                            const T* __restrict__ dq, const T* __restrict__ dk,
                                                            const float* __restrict__ dv, T* __restrict__ dx,
                                                            float* __restrict__ part, int B, int Tn, int C, int KD,
                                                            int DK, int REP, int tile, int tpb) {
  constexpr int V = Vec<T>::V;
  const int c = (blockIdx.x * kThreads + threadIdx.x) * V;
  if (c >= C) return;
  float tp[4][V];
  load_taps<TW, V>(w, c, tp);
  const Route rt = route(c, KD, DK, REP);
  const T* dqk = rt.isk ? dk : dq;
  const long long qrow = (long long)KD * REP, vrow = C - 2 * KD;
  const int ntiles = (Tn + tile - 1) / tile;
  const long long total = (long long)B * ntiles;
  float acc[4][V];
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int i = 0; i < V; ++i) acc[j][i] = 0.f;
  const long long q0 = (long long)blockIdx.y * tpb;
  const long long q1 = q0 + tpb < total ? q0 + tpb : total;
  for (long long qt = q0; qt < q1; ++qt) {
    const int b = (int)(qt / ntiles);
    const int t0 = (int)(qt % ntiles) * tile;
    const int tl = t0 + tile < Tn ? t0 + tile : Tn;  // this tile's outputs: [t0, tl)
    const T* xb = x + (size_t)b * Tn * C + c;
    T* dxb = dx + (size_t)b * Tn * C + c;
    float xm3[V], xm2[V], xm1[V], dm1[V], dm2[V], dm3[V];
#pragma unroll
    for (int i = 0; i < V; ++i) xm3[i] = xm2[i] = xm1[i] = dm1[i] = dm2[i] = dm3[i] = 0.f;
    if (t0 >= 3) ld(xb + (size_t)(t0 - 3) * C, xm3);
    if (t0 >= 2) ld(xb + (size_t)(t0 - 2) * C, xm2);
    if (t0 >= 1) ld(xb + (size_t)(t0 - 1) * C, xm1);
    // du[t] needs x[t - 3 .. t]; dx[t - 3] is complete once du[t] is known: walk t0 .. tl + 2, kBatchB steps' rows
    // of x and of the cotangents in flight before any is used; running pointers at row t0
    const long long bt0 = (long long)b * Tn + t0;
    const T* xp = xb + (size_t)t0 * C;
    const T* gp = (rt.isv || dqk == nullptr) ? nullptr : dqk + bt0 * qrow + rt.qcol;
    const float* gvp = (rt.isv && dv != nullptr) ? dv + bt0 * vrow + rt.cc : nullptr;
    T* dxp = dxb + (size_t)t0 * C;
    for (int tb = t0; tb < tl + 3; tb += kBatchB) {
      const int n = Tn - tb;  // rows of this batch inside the sequence
      float xr[kBatchB][V], g[kBatchB][V];
#pragma unroll
      for (int s = 0; s < kBatchB; ++s) {
#pragma unroll
        for (int i = 0; i < V; ++i) xr[s][i] = g[s][i] = 0.f;
        if (s < n) ld(xp + (size_t)s * C, xr[s]);
      }
      if (gvp) {
#pragma unroll
        for (int s = 0; s < kBatchB; ++s)
          if (s < n) ldf<V>(gvp + (long long)s * vrow, g[s]);
      } else if (gp) {
        const int nrep = RP > 0 ? RP : REP;
#pragma unroll
        for (int r = 0; r < (RP > 0 ? RP : 1); ++r) {  // the value heads' gradients, in order
#pragma unroll
          for (int s = 0; s < kBatchB; ++s) {
            if (s < n) {
              float gr[V];
              ld(gp + (long long)s * qrow + (long long)r * DK, gr);
#pragma unroll
              for (int i = 0; i < V; ++i) g[s][i] += gr[i];
            }
          }
        }
        for (int r = 1; RP == 0 && r < nrep; ++r) {
#pragma unroll
          for (int s = 0; s < kBatchB; ++s) {
            if (s < n) {
              float gr[V];
              ld(gp + (long long)s * qrow + (long long)r * DK, gr);
#pragma unroll
              for (int i = 0; i < V; ++i) g[s][i] += gr[i];
            }
          }
        }
      }
      xp += (size_t)kBatchB * C;
      if (gp) gp += (long long)kBatchB * qrow;
      if (gvp) gvp += (long long)kBatchB * vrow;
#pragma unroll
      for (int s = 0; s < kBatchB; ++s) {
        const int t = tb + s;
        if (t >= tl + 3) break;
        float du[V];
#pragma unroll
        for (int i = 0; i < V; ++i) {  // rows past Tn hold zeros: du = 0 there
          const float u =
              fmaf(tp[3][i], xr[s][i], fmaf(tp[2][i], xm1[i], fmaf(tp[1][i], xm2[i], tp[0][i] * xm3[i])));
          const float sg = sigmoid(u);
          du[i] = g[s][i] * sg * (1.f + u * (1.f - sg));
        }
        if (DW && t < tl) {
#pragma unroll
          for (int i = 0; i < V; ++i) {
            acc[0][i] = fmaf(du[i], xm3[i], acc[0][i]);
            acc[1][i] = fmaf(du[i], xm2[i], acc[1][i]);
            acc[2][i] = fmaf(du[i], xm1[i], acc[2][i]);
            acc[3][i] = fmaf(du[i], xr[s][i], acc[3][i]);
          }
        }
        if (t >= t0 + 3) {
          float o[V];
#pragma unroll
          for (int i = 0; i < V; ++i)
            o[i] = fmaf(tp[0][i], du[i], fmaf(tp[1][i], dm1[i], fmaf(tp[2][i], dm2[i], tp[3][i] * dm3[i])));
          st(dxp, o);  // row t - 3
          dxp += C;
        }
#pragma unroll
        for (int i = 0; i < V; ++i) {
          xm3[i] = xm2[i];
          xm2[i] = xm1[i];
          xm1[i] = xr[s][i];
          dm3[i] = dm2[i];
          dm2[i] = dm1[i];
          dm1[i] = du[i];
        }
      }
    }
  }
  if constexpr (DW) {
    float* pr = part + ((size_t)blockIdx.y * C + c) * 4;
#pragma unroll
    for (int i = 0; i < V; ++i)
      *reinterpret_cast<float4*>(pr + 4 * i) = make_float4(acc[0][i], acc[1][i], acc[2][i], acc[3][i]);
  }
}

// dw[n] (n = 4 c + j) = the sum of the P partial rows' element n: 32 elements a CTA, thread row y sums partials y,
// y + 32, ..., then a fixed tree over the 32 thread rows
template <typename TW>
__global__ void __launch_bounds__(1024) conv_dw_sum_kernel(const float* __restrict__ part, int P, int N,
                                                           TW* __restrict__ dw) {
  __shared__ float red[32][33];
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int n = blockIdx.x * 32 + tx;
  float s = 0.f;
  if (n < N)
    for (int p = ty; p < P; p += 32) s += part[(size_t)p * N + n];
  red[ty][tx] = s;
  __syncthreads();
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    if (ty < o) red[ty][tx] += red[ty + o][tx];
    __syncthreads();
  }
  if (ty == 0 && n < N) dw[n] = cvt<TW>(red[0][tx]);
}

// the backward's time steps a thread walks: 64 (its halo of 3 + 3 rows costs less per step) when that still gives two
// full waves of CTAs, else 32 or 16 (short sequences and few batch rows: more CTAs in flight)
int tile_for(int B, int Tn, int C) {
  const long long groups = (C / Vec<float>::V + kThreads - 1) / kThreads;
  for (int L = 64; L > 16; L /= 2)
    if (groups * B * ((Tn + L - 1) / L) >= kFillCTAs) return L;
  return 16;
}

// tiles per row block and the number of row blocks (at most kMaxPartials with dw, else at most the grid's y limit)
void plan(int B, int Tn, int tile, bool dw, int& tpb, int& P) {
  const long long total = (long long)B * ((Tn + tile - 1) / tile);
  const long long cap = dw ? kMaxPartials : kMaxGridY;
  tpb = (int)((total + cap - 1) / cap);
  if (tpb < 1) tpb = 1;
  P = (int)((total + tpb - 1) / tpb);
}

int status_of(cudaError_t e) { return e == cudaSuccess ? GD_OK : GD_ERR_LAUNCH; }
bool aligned16(const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <typename T, typename TW>
int fwd_t(const void* x, const void* w, void* q, void* k, float* v, int B, int Tn, int C, int KD, int DK, int REP,
          cudaStream_t st) {
  constexpr int V = Vec<T>::V;
  const int groups = C / V;
  dim3 grid((groups + kThreads - 1) / kThreads, (Tn + kTileF - 1) / kTileF, B);
  conv_fwd_kernel<T, TW><<<grid, kThreads, 0, st>>>(static_cast<const T*>(x), static_cast<const TW*>(w),
                                                    static_cast<T*>(q), static_cast<T*>(k), v, Tn, C, KD, DK, REP);
  return status_of(cudaGetLastError());
}

template <typename T, typename TW>
int bwd_t(const void* x, const void* w, const void* dq, const void* dk, const float* dv, void* dx, void* dw, int B,
          int Tn, int C, int KD, int DK, int REP, void* ws, cudaStream_t st) {
  constexpr int V = Vec<T>::V;
  const int groups = C / V;
  int tpb, P;
  const int tile = tile_for(B, Tn, C);
  plan(B, Tn, tile, dw != nullptr, tpb, P);
  dim3 grid((groups + kThreads - 1) / kThreads, P);
  float* part = static_cast<float*>(ws);
  auto launch = [&](auto kern) {
    kern<<<grid, kThreads, 0, st>>>(static_cast<const T*>(x), static_cast<const TW*>(w), static_cast<const T*>(dq),
                                    static_cast<const T*>(dk), dv, static_cast<T*>(dx), part, B, Tn, C, KD, DK, REP,
                                    tile, tpb);
  };
  if (dw == nullptr) {
    if (REP == 1) launch(conv_bwd_kernel<T, TW, false, 1>);
    else if (REP == 2) launch(conv_bwd_kernel<T, TW, false, 2>);
    else launch(conv_bwd_kernel<T, TW, false, 0>);
  } else {
    if (REP == 1) launch(conv_bwd_kernel<T, TW, true, 1>);
    else if (REP == 2) launch(conv_bwd_kernel<T, TW, true, 2>);
    else launch(conv_bwd_kernel<T, TW, true, 0>);
  }
  if (cudaGetLastError() != cudaSuccess) return GD_ERR_LAUNCH;
  if (dw == nullptr) return GD_OK;
  const int N = 4 * C;
  conv_dw_sum_kernel<TW><<<(N + 31) / 32, dim3(32, 32), 0, st>>>(part, P, N, static_cast<TW*>(dw));
  return status_of(cudaGetLastError());
}

// shapes the kernels take (the reference's supported(), _conv.py:178-185, with 16-byte channel groups): C = 2 KD + VD,
// KD a multiple of DK, VD of DV, (KD / DK) REP == VD / DV value heads, and C, KD, DK, DV multiples of the group
int check_args(int dtype, int wdtype, int B, int Tn, int C, int KD, int DK, int REP, int DV) {
  if (dtype < GD_FLOAT32 || dtype > GD_BFLOAT16 || wdtype < GD_FLOAT32 || wdtype > GD_BFLOAT16) return GD_ERR_ARG;
  if (wdtype != dtype && wdtype != GD_FLOAT32) return GD_ERR_ARG;
  const int V = dtype == GD_FLOAT32 ? 4 : 8;
  if (B < 0 || Tn < 0 || B > kMaxGridY || (Tn + kTileF - 1) / kTileF > kMaxGridY) return GD_ERR_SHAPE;
  if (KD <= 0 || DK <= 0 || REP <= 0 || DV <= 0) return GD_ERR_SHAPE;
  const int VD = C - 2 * KD;
  if (VD <= 0 || KD % DK != 0 || VD % DV != 0 || (KD / DK) * REP != VD / DV) return GD_ERR_SHAPE;
  if (C % V != 0 || KD % V != 0 || DK % V != 0 || DV % V != 0) return GD_ERR_SHAPE;
  if ((long long)B * Tn * C >= (1ll << 40)) return GD_ERR_SHAPE;
  return GD_OK;
}

}  // namespace

extern "C" {

size_t gd_conv_workspace_bytes(int B, int T, int C) {
  if (B < 0 || T < 0 || C <= 0) return 0;
  int tpb, P;
  plan(B, T, tile_for(B, T, C), true, tpb, P);
  return (size_t)P * C * 4 * sizeof(float);
}

int gd_conv_fwd(const void* x, const void* w, void* q, void* k, float* v, int dtype, int wdtype, int B, int T, int C,
                int KD, int DK, int REP, int DV, void* stream) {
  int s = check_args(dtype, wdtype, B, T, C, KD, DK, REP, DV);
  if (s) return s;
  if ((long long)B * T == 0) return GD_OK;
  if (!x || !w || !q || !k || !v) return GD_ERR_ARG;
  if (!aligned16(x) || !aligned16(q) || !aligned16(k) || !aligned16(v) ||
      (reinterpret_cast<uintptr_t>(w) & (wdtype == GD_FLOAT32 ? 3u : 1u)) != 0)
    return GD_ERR_ALIGN;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case GD_BFLOAT16:
      return wdtype == GD_FLOAT32 ? fwd_t<__nv_bfloat16, float>(x, w, q, k, v, B, T, C, KD, DK, REP, st)
                                  : fwd_t<__nv_bfloat16, __nv_bfloat16>(x, w, q, k, v, B, T, C, KD, DK, REP, st);
    case GD_FLOAT16:
      return wdtype == GD_FLOAT32 ? fwd_t<__half, float>(x, w, q, k, v, B, T, C, KD, DK, REP, st)
                                  : fwd_t<__half, __half>(x, w, q, k, v, B, T, C, KD, DK, REP, st);
    default: return fwd_t<float, float>(x, w, q, k, v, B, T, C, KD, DK, REP, st);
  }
}

int gd_conv_bwd(const void* x, const void* w, const void* dq, const void* dk, const float* dv, void* dx, void* dw,
                int dtype, int wdtype, int B, int T, int C, int KD, int DK, int REP, int DV, void* workspace,
                size_t workspace_bytes, void* stream) {
  int s = check_args(dtype, wdtype, B, T, C, KD, DK, REP, DV);
  if (s) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((long long)B * T == 0) {  // no tokens: the weight's gradient is zero
    if (dw && cudaMemsetAsync(dw, 0, (size_t)4 * C * (wdtype == GD_FLOAT32 ? 4 : 2), st) != cudaSuccess)
      return GD_ERR_LAUNCH;
    return GD_OK;
  }
  if (!x || !w || !dx) return GD_ERR_ARG;
  if (dw != nullptr && (workspace == nullptr || workspace_bytes < gd_conv_workspace_bytes(B, T, C)))
    return GD_ERR_WORKSPACE;
  if (!aligned16(x) || !aligned16(dq) || !aligned16(dk) || !aligned16(dv) || !aligned16(dx) || !aligned16(workspace) ||
      (reinterpret_cast<uintptr_t>(w) & (wdtype == GD_FLOAT32 ? 3u : 1u)) != 0)
    return GD_ERR_ALIGN;
  switch (dtype) {
    case GD_BFLOAT16:
      return wdtype == GD_FLOAT32
                 ? bwd_t<__nv_bfloat16, float>(x, w, dq, dk, dv, dx, dw, B, T, C, KD, DK, REP, workspace, st)
                 : bwd_t<__nv_bfloat16, __nv_bfloat16>(x, w, dq, dk, dv, dx, dw, B, T, C, KD, DK, REP, workspace, st);
    case GD_FLOAT16:
      return wdtype == GD_FLOAT32 ? bwd_t<__half, float>(x, w, dq, dk, dv, dx, dw, B, T, C, KD, DK, REP, workspace, st)
                                  : bwd_t<__half, __half>(x, w, dq, dk, dv, dx, dw, B, T, C, KD, DK, REP, workspace, st);
    default: return bwd_t<float, float>(x, w, dq, dk, dv, dx, dw, B, T, C, KD, DK, REP, workspace, st);
  }
}

}  // extern "C"
