// The gated RMSNorm on the rule's output (transformers' Qwen3_5RMSNormGated over rows of one value head), one pass
// each way. The reference's formulas (src/macai/layer/_gated_norm.py:1-16) and autograd contract (:154-197), with
// transformers' rounding points:
//   x_hat = x rsqrt(mean(x^2) + eps)                        (fp32)
//   h     = w x_hat.to(T)                                   (rounded to T again when w has x's dtype)
//   o     = (h silu(z)).to(T)
// backward in fp32, one rounding per gradient (s = silu(z), sig = sigmoid(z)):
//   dz = do h sig (1 + z (1 - sig)),  dx = r (dxh - x_hat <x_hat, dxh> / D) with dxh = do s w,
//   dw = sum over rows of do s x_hat.to(T)                  (only when asked: fixed-order partial rows, then a sum)
// x, z, o, dout, dx, dz: [rows, D] in T (fp32 / fp16 / bf16); w and dw: [D] in T or fp32.
//
// Every width runs on one design: a row belongs to a team of TEAM consecutive lanes of a warp (TEAM a power of two,
// 32 / TEAM rows a warp at once), lane i of a team holding the row's 16-byte (or, for 16-bit widths that are not a
// multiple of 8, 8-byte) chunks i, i + TEAM, ... in registers; the row's sums are xor shuffles inside the team.
// D = 128 at 16 bits (the Qwen3.5 value heads) has its own kernels: half a warp a row, two rows a lane in flight,
// streaming 16-byte loads and stores. HBM-bound: the forward reads x and z and writes o (3 x 2 B per element at
// bf16), the backward reads x, z, dout and writes dx, dz (5 x 2 B).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

#include "gated_delta_b200.h"

namespace {

constexpr int kThreads = 256;       // 8 warps
constexpr int kWarps = kThreads / 32;
constexpr int kMaxPartials = 1024;  // CTAs of the backward with dw (its fixed-order partial rows)
constexpr int kMaxD = 1024;

// x rounded to T and back (the .to(input_dtype) of the torch expression)
template <typename T>
__device__ __forceinline__ float rnd(float x);
template <>
__device__ __forceinline__ float rnd<float>(float x) { return x; }
template <>
__device__ __forceinline__ float rnd<__nv_bfloat16>(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
template <>
__device__ __forceinline__ float rnd<__half>(float x) { return __half2float(__float2half_rn(x)); }

template <typename T>
__device__ __forceinline__ T cvt(float x);
template <>
__device__ __forceinline__ float cvt<float>(float x) { return x; }
template <>
__device__ __forceinline__ __half cvt<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 cvt<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// sigmoid with the fast divide (2 ulp; a denominator past 2^126, z < -87, gives 0): the division's full-precision
// sequence made the kernels instruction-bound
__device__ __forceinline__ float sigmoid(float z) { return __fdividef(1.f, 1.f + expf(-z)); }

// 1 / sqrt(mean + eps) from a correctly rounded square root and division (PyTorch's rsqrt on the CPU rounds the same
// way to within an ulp)
__device__ __forceinline__ float inv_rms(float ss, int D, float eps) { return 1.f / sqrtf(ss / (float)D + eps); }

// ---- E consecutive elements of T <-> floats (E * sizeof(T) = 8 or 16 bytes, aligned to that)
template <typename T, int E>
struct Chunk {
  static_assert(E * sizeof(T) == 8 || E * sizeof(T) == 16, "8- or 16-byte chunks");
  using Raw = typename std::conditional<E * sizeof(T) == 16, uint4, uint2>::type;
  __device__ __forceinline__ static void load(const T* p, float (&f)[E]) {
    const Raw r = *reinterpret_cast<const Raw*>(p);
    const uint32_t* u = reinterpret_cast<const uint32_t*>(&r);
    if constexpr (std::is_same<T, float>::value) {
#pragma unroll
      for (int e = 0; e < E; ++e) f[e] = __uint_as_float(u[e]);
    } else {
#pragma unroll
      for (int i = 0; i < E / 2; ++i) {
        float2 v;
        if constexpr (std::is_same<T, __half>::value) {
          v = __half22float2(*reinterpret_cast<const __half2*>(u + i));
        } else {
          v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(u + i));
        }
        f[2 * i] = v.x;
        f[2 * i + 1] = v.y;
      }
    }
  }
  __device__ __forceinline__ static void store(T* p, const float (&f)[E]) {
    Raw r;
    uint32_t* u = reinterpret_cast<uint32_t*>(&r);
    if constexpr (std::is_same<T, float>::value) {
#pragma unroll
      for (int e = 0; e < E; ++e) u[e] = __float_as_uint(f[e]);
    } else {
#pragma unroll
      for (int i = 0; i < E / 2; ++i) {
        if constexpr (std::is_same<T, __half>::value) {
          const __half2 v = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
          u[i] = *reinterpret_cast<const uint32_t*>(&v);
        } else {
          const __nv_bfloat162 v = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
          u[i] = *reinterpret_cast<const uint32_t*>(&v);
        }
      }
    }
    *reinterpret_cast<Raw*>(p) = r;
  }
};

// the weight's E elements at p (w in T or fp32; element-wise loads: w is tiny and stays in L1)
template <typename TW, int E>
__device__ __forceinline__ void load_weights(const TW* p, float (&f)[E]) {
#pragma unroll
  for (int e = 0; e < E; ++e) {
    if constexpr (std::is_same<TW, float>::value) {
      f[e] = __ldg(p + e);
    } else if constexpr (std::is_same<TW, __half>::value) {
      f[e] = __half2float(p[e]);
    } else {
      f[e] = __bfloat162float(p[e]);
    }
  }
}

// sum over the team (lanes that differ only in the low team_log2 bits); every lane of the warp takes part
__device__ __forceinline__ float team_sum(float v, int team_log2) {
  for (int o = (1 << team_log2) >> 1; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// A team's view of the grid: the row it owns, its lane inside the team
struct Team {
  int log2, sub;
  long long row;
  __device__ __forceinline__ Team(int team_log2, long long first_row_of_warp) {
    const int lane = threadIdx.x & 31;
    log2 = team_log2;
    sub = lane & ((1 << team_log2) - 1);
    row = first_row_of_warp + (lane >> team_log2);
  }
  __device__ __forceinline__ int elem(int j, int E) const { return (sub + (j << log2)) * E; }  // chunk j's first element
};

// ---- forward, any width: warp w of CTA b owns rows (8 b + w) R .. + R - 1, R = 32 / TEAM
template <typename T, typename TW, int E, int NCH>
__global__ void __launch_bounds__(kThreads) gnorm_team_fwd(const T* __restrict__ x, const T* __restrict__ z,
                                                           const TW* __restrict__ w, T* __restrict__ o,
                                                           long long rows, int D, int team_log2, float eps,
                                                           bool round_h) {
  const long long warp_row0 = ((long long)blockIdx.x * kWarps + (threadIdx.x >> 5)) << (5 - team_log2);
  const Team tm(team_log2, warp_row0);
  const bool live = tm.row < rows;
  float xs[NCH][E], zs[NCH][E];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NCH; ++j) {  // all of the row's loads in flight before any arithmetic
    const int e0 = tm.elem(j, E);
    if (live && e0 < D) {
      Chunk<T, E>::load(x + tm.row * D + e0, xs[j]);
      Chunk<T, E>::load(z + tm.row * D + e0, zs[j]);
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e) xs[j][e] = zs[j][e] = 0.f;
    }
  }
#pragma unroll
  for (int j = 0; j < NCH; ++j)
#pragma unroll
    for (int e = 0; e < E; ++e) ss = fmaf(xs[j][e], xs[j][e], ss);
  const float r = inv_rms(team_sum(ss, team_log2), D, eps);
#pragma unroll
  for (int j = 0; j < NCH; ++j) {
    const int e0 = tm.elem(j, E);
    if (!live || e0 >= D) continue;
    float wv[E], out[E];
    load_weights<TW, E>(w + e0, wv);
#pragma unroll
    for (int e = 0; e < E; ++e) {
      float h = wv[e] * rnd<T>(xs[j][e] * r);
      if (round_h) h = rnd<T>(h);
      out[e] = h * (zs[j][e] * sigmoid(zs[j][e]));
    }
    Chunk<T, E>::store(o + tm.row * D + e0, out);
  }
}

// ---- backward, any width. No dw: rows as the forward. With dw: CTA p takes rows [p rpb, (p + 1) rpb) (rpb a
// multiple of 8 R), warp w the blocks of R rows w, w + 8, ...; a lane keeps its chunks' dw sums, the CTA's teams are
// added in team order into partial row p (dynamic shared memory [8 R][D] floats).
template <typename T, typename TW, int E, int NCH, bool DW>
__global__ void __launch_bounds__(kThreads) gnorm_team_bwd(const T* __restrict__ x, const T* __restrict__ z,
                                                           const TW* __restrict__ w, const T* __restrict__ dout,
                                                           T* __restrict__ dx, T* __restrict__ dz,
                                                           float* __restrict__ part, long long rows, int D,
                                                           int team_log2, float eps, bool round_h, long long rpb) {
  const int warp = threadIdx.x >> 5;
  const int R = 32 >> team_log2;
  float wsum[NCH][E];
#pragma unroll
  for (int j = 0; j < NCH; ++j)
#pragma unroll
    for (int e = 0; e < E; ++e) wsum[j][e] = 0.f;
  long long first, end, step;
  if constexpr (DW) {
    first = (long long)blockIdx.x * rpb + (long long)warp * R;
    end = (long long)blockIdx.x * rpb + rpb < rows ? (long long)blockIdx.x * rpb + rpb : rows;
    step = (long long)kWarps * R;
  } else {
    first = ((long long)blockIdx.x * kWarps + warp) * R;
    end = rows;
    step = rows;  // one block of rows
  }
  int sub = 0;
  for (long long base = first; base < end; base += step) {
    const Team tm(team_log2, base);
    sub = tm.sub;
    const bool live = tm.row < end;
    float xs[NCH][E], zs[NCH][E], gs[NCH][E];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const int e0 = tm.elem(j, E);
      if (live && e0 < D) {
        Chunk<T, E>::load(x + tm.row * D + e0, xs[j]);
        Chunk<T, E>::load(z + tm.row * D + e0, zs[j]);
        Chunk<T, E>::load(dout + tm.row * D + e0, gs[j]);
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) xs[j][e] = zs[j][e] = gs[j][e] = 0.f;
      }
    }
#pragma unroll
    for (int j = 0; j < NCH; ++j)
#pragma unroll
      for (int e = 0; e < E; ++e) ss = fmaf(xs[j][e], xs[j][e], ss);
    const float r = inv_rms(team_sum(ss, team_log2), D, eps);
    float dot = 0.f;  // <x_hat, dxh> over the lane's elements
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const int e0 = tm.elem(j, E);
      float wv[E];
      if (e0 < D) {
        load_weights<TW, E>(w + e0, wv);
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) wv[e] = 0.f;
      }
      float dzv[E];
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const float xn = xs[j][e] * r;
        const float xq = rnd<T>(xn);
        float h = wv[e] * xq;
        if (round_h) h = rnd<T>(h);
        const float zz = zs[j][e], sg = sigmoid(zz);
        dzv[e] = gs[j][e] * h * sg * (1.f + zz * (1.f - sg));
        const float gsl = gs[j][e] * (zz * sg);  // dout silu(z)
        if constexpr (DW) wsum[j][e] = fmaf(gsl, xq, wsum[j][e]);
        gs[j][e] = gsl * wv[e];                  // dxh
        dot = fmaf(xn, gs[j][e], dot);
        xs[j][e] = xn;
      }
      if (live && e0 < D) Chunk<T, E>::store(dz + tm.row * D + e0, dzv);
    }
    const float cmean = team_sum(dot, team_log2) / (float)D;
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const int e0 = tm.elem(j, E);
      if (!live || e0 >= D) continue;
      float out[E];
#pragma unroll
      for (int e = 0; e < E; ++e) out[e] = r * (gs[j][e] - xs[j][e] * cmean);
      Chunk<T, E>::store(dx + tm.row * D + e0, out);
    }
  }
  if constexpr (DW) {
    extern __shared__ __align__(16) float red[];  // [8 R teams][D]
    const int team = warp * R + ((threadIdx.x & 31) >> team_log2);
    if (first >= end) sub = (threadIdx.x & 31) & ((1 << team_log2) - 1);
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const int e0 = (sub + (j << team_log2)) * E;
      if (e0 < D)
#pragma unroll
        for (int e = 0; e < E; ++e) red[(size_t)team * D + e0 + e] = wsum[j][e];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < D; i += kThreads) {
      float s = 0.f;
      for (int k = 0; k < kWarps * R; ++k) s += red[(size_t)k * D + i];
      part[(size_t)blockIdx.x * D + i] = s;
    }
  }
}

// ---- D = 128 with 16-bit activations (the Qwen3.5 value heads): half a warp a row, 8 elements (16 bytes) a lane,
// two rows a warp per step and kRP steps' loads in flight at once
constexpr int kRP = 2;

__device__ __forceinline__ void unpack8(const uint4 u, float (&v)[8], const __nv_bfloat16*) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]));
    v[2 * j] = f.x;
    v[2 * j + 1] = f.y;
  }
}
__device__ __forceinline__ void unpack8(const uint4 u, float (&v)[8], const __half*) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
    v[2 * j] = f.x;
    v[2 * j + 1] = f.y;
  }
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
__device__ __forceinline__ uint4 pack8(const float (&v)[8]) {
  const T* tag = nullptr;
  return make_uint4(pack2(v[0], v[1], tag), pack2(v[2], v[3], tag), pack2(v[4], v[5], tag), pack2(v[6], v[7], tag));
}
// the lane's 8 weights
template <typename T>
__device__ __forceinline__ void load_w8(const T* w, float (&v)[8]) {
  unpack8(__ldg(reinterpret_cast<const uint4*>(w)), v, w);
}
__device__ __forceinline__ void load_w8(const float* w, float (&v)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(w)), b = __ldg(reinterpret_cast<const float4*>(w) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ float half_sum(float v) {  // over the 16 lanes of one half-warp
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// warp w of CTA b: rows 2 (kRP (8 b + w) + p) + half, p < kRP
template <typename T, typename TW>
__global__ void __launch_bounds__(kThreads) gnorm_fwd128_kernel(const T* __restrict__ x, const T* __restrict__ z,
                                                                const TW* __restrict__ w, T* __restrict__ o,
                                                                long long rows, float eps, bool round_h) {
  const int lane = threadIdx.x & 31, sub = lane & 15;
  const long long r0 = ((long long)blockIdx.x * kWarps + (threadIdx.x >> 5)) * 2 * kRP + (lane >> 4);
  uint4 xu[kRP], zu[kRP];
#pragma unroll
  for (int p = 0; p < kRP; ++p) {
    const long long row = r0 + 2 * p;
    if (row < rows) {
      xu[p] = __ldcs(reinterpret_cast<const uint4*>(x + row * 128) + sub);
      zu[p] = __ldcs(reinterpret_cast<const uint4*>(z + row * 128) + sub);
    } else {
      xu[p] = zu[p] = make_uint4(0, 0, 0, 0);
    }
  }
  float wv[8];
  load_w8(w + 8 * sub, wv);
#pragma unroll
  for (int p = 0; p < kRP; ++p) {
    const long long row = r0 + 2 * p;
    float xv[8], zv[8];
    unpack8(xu[p], xv, x);
    unpack8(zu[p], zv, z);
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) ss = fmaf(xv[e], xv[e], ss);
    const float r = inv_rms(half_sum(ss), 128, eps);
    float ov[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float h = wv[e] * rnd<T>(xv[e] * r);
      if (round_h) h = rnd<T>(h);
      ov[e] = h * (zv[e] * sigmoid(zv[e]));
    }
    if (row < rows) __stcs(reinterpret_cast<uint4*>(o + row * 128) + sub, pack8<T>(ov));
  }
}

// No dw: rows as the forward. With dw: CTA p takes rows [p rpb, (p + 1) rpb) (rpb a multiple of 16 kRP), warp k the
// steps k, k + 8, ... of it; each lane keeps its 8 columns' sums, and the CTA's 16 half-warp rows are summed in order
// into partial row p.
template <typename T, typename TW, bool DW>
__global__ void __launch_bounds__(kThreads) gnorm_bwd128_kernel(const T* __restrict__ x, const T* __restrict__ z,
                                                                const TW* __restrict__ w, const T* __restrict__ dout,
                                                                T* __restrict__ dx, T* __restrict__ dz,
                                                                float* __restrict__ part, long long rows, float eps,
                                                                bool round_h, long long rpb) {
  const int lane = threadIdx.x & 31, sub = lane & 15, warp = threadIdx.x >> 5;
  float wv[8], dwa[8];
  load_w8(w + 8 * sub, wv);
#pragma unroll
  for (int e = 0; e < 8; ++e) dwa[e] = 0.f;
  long long first, end, step;
  if constexpr (DW) {
    first = (long long)blockIdx.x * rpb + (long long)warp * 2 * kRP;
    end = (long long)blockIdx.x * rpb + rpb < rows ? (long long)blockIdx.x * rpb + rpb : rows;
    step = (long long)kWarps * 2 * kRP;
  } else {
    first = ((long long)blockIdx.x * kWarps + warp) * 2 * kRP;
    end = rows;
    step = end;  // one step
  }
  for (long long base = first; base < end; base += step) {
    const long long r0 = base + (lane >> 4);
    uint4 xu[kRP], zu[kRP], gu[kRP];
#pragma unroll
    for (int p = 0; p < kRP; ++p) {
      const long long row = r0 + 2 * p;
      if (row < end) {
        xu[p] = __ldcs(reinterpret_cast<const uint4*>(x + row * 128) + sub);
        zu[p] = __ldcs(reinterpret_cast<const uint4*>(z + row * 128) + sub);
        gu[p] = __ldcs(reinterpret_cast<const uint4*>(dout + row * 128) + sub);
      } else {
        xu[p] = zu[p] = gu[p] = make_uint4(0, 0, 0, 0);  // zeros: nothing added to dwa, nothing stored
      }
    }
#pragma unroll
    for (int p = 0; p < kRP; ++p) {
      const long long row = r0 + 2 * p;
      float xv[8], zv[8], gv[8];
      unpack8(xu[p], xv, x);
      unpack8(zu[p], zv, z);
      unpack8(gu[p], gv, dout);
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = fmaf(xv[e], xv[e], ss);
      const float r = inv_rms(half_sum(ss), 128, eps);
      float acc = 0.f, dzv[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float xn = xv[e] * r;
        const float xr = rnd<T>(xn);
        float h = wv[e] * xr;
        if (round_h) h = rnd<T>(h);
        const float sg = sigmoid(zv[e]);
        dzv[e] = gv[e] * h * sg * (1.f + zv[e] * (1.f - sg));
        const float gs = gv[e] * (zv[e] * sg);
        if constexpr (DW) dwa[e] = fmaf(gs, xr, dwa[e]);
        gv[e] = gs * wv[e];  // dxh
        acc = fmaf(xn, gv[e], acc);
        xv[e] = xn;
      }
      const float c = half_sum(acc) / 128.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) gv[e] = r * (gv[e] - xv[e] * c);
      if (row < end) {
        __stcs(reinterpret_cast<uint4*>(dz + row * 128) + sub, pack8<T>(dzv));
        __stcs(reinterpret_cast<uint4*>(dx + row * 128) + sub, pack8<T>(gv));
      }
    }
  }
  if constexpr (DW) {
    __shared__ __align__(16) float red[2 * kWarps][128];
#pragma unroll
    for (int e = 0; e < 8; ++e) red[2 * warp + (lane >> 4)][8 * sub + e] = dwa[e];
    __syncthreads();
    if (threadIdx.x < 128) {
      float s = 0.f;
#pragma unroll
      for (int k = 0; k < 2 * kWarps; ++k) s += red[k][threadIdx.x];
      part[(size_t)blockIdx.x * 128 + threadIdx.x] = s;
    }
  }
}

// dw[c] = the sum of the P partial rows' column c: 32 columns a CTA, thread row y sums the partials y, y + 32, ...,
// then a fixed tree over the 32 thread rows (the error grows with P / 32 + 5 additions, not P)
template <typename TW>
__global__ void __launch_bounds__(1024) gnorm_dw_sum_kernel(const float* __restrict__ part, int P, int D,
                                                            TW* __restrict__ dw) {
  __shared__ float red[32][33];
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int c = blockIdx.x * 32 + tx;
  float s = 0.f;
  if (c < D)
    for (int p = ty; p < P; p += 32) s += part[(size_t)p * D + c];
  red[ty][tx] = s;
  __syncthreads();
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    if (ty < o) red[ty][tx] += red[ty + o][tx];
    __syncthreads();
  }
  if (ty == 0 && c < D) dw[c] = cvt<TW>(red[0][tx]);
}

// rows per partial row of dw: a multiple of `unit` (a CTA's rows per step), at least ceil(rows / kMaxPartials)
void partition(long long rows, long long unit, long long& rpb, int& P) {
  rpb = (rows + kMaxPartials - 1) / kMaxPartials;
  rpb = (rpb + unit - 1) / unit * unit;
  if (rpb < unit) rpb = unit;
  P = (int)((rows + rpb - 1) / rpb);
  if (P < 1) P = 1;
}

int status_of(cudaError_t e) { return e == cudaSuccess ? GD_OK : GD_ERR_LAUNCH; }
bool aligned16(const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// The team shape for width D: chunk E elements (16 bytes, or 8 when a 16-bit width is not a multiple of 8), D / E
// chunks a row; up to 32 chunks: a team of the next power of two lanes, one chunk each; more: 32 lanes, NCH chunks each
struct Shape {
  int E, nch, team_log2;
};
template <typename T>
Shape shape_for(int D) {
  Shape s;
  s.E = (sizeof(T) == 2 && D % 8 == 0) ? 8 : 4;
  const int chunks = D / s.E;
  if (chunks <= 32) {
    s.nch = 1;
    s.team_log2 = 0;
    while ((1 << s.team_log2) < chunks) ++s.team_log2;
  } else {
    s.team_log2 = 5;
    s.nch = chunks <= 64 ? 2 : (chunks <= 128 ? 4 : 8);
  }
  return s;
}

template <typename T, typename TW, int E, int NCH>
int team_fwd(const void* x, const void* z, const void* w, void* o, long long rows, int D, int tl, float eps,
             bool round_h, cudaStream_t st) {
  const long long per = (long long)kWarps << (5 - tl);  // rows a CTA
  gnorm_team_fwd<T, TW, E, NCH><<<(unsigned)((rows + per - 1) / per), kThreads, 0, st>>>(
      static_cast<const T*>(x), static_cast<const T*>(z), static_cast<const TW*>(w), static_cast<T*>(o), rows, D, tl,
      eps, round_h);
  return status_of(cudaGetLastError());
}

template <typename T, typename TW, int E, int NCH>
int team_bwd(const void* x, const void* z, const void* w, const void* dout, void* dx, void* dz, void* dw,
             long long rows, int D, int tl, float eps, bool round_h, void* ws, cudaStream_t st) {
  const T* xp = static_cast<const T*>(x);
  const T* zp = static_cast<const T*>(z);
  const TW* wp = static_cast<const TW*>(w);
  const T* gp = static_cast<const T*>(dout);
  const long long per = (long long)kWarps << (5 - tl);
  if (dw == nullptr) {
    gnorm_team_bwd<T, TW, E, NCH, false><<<(unsigned)((rows + per - 1) / per), kThreads, 0, st>>>(
        xp, zp, wp, gp, static_cast<T*>(dx), static_cast<T*>(dz), nullptr, rows, D, tl, eps, round_h, 0);
    return status_of(cudaGetLastError());
  }
  long long rpb;
  int P;
  partition(rows, per, rpb, P);
  const size_t smem = (size_t)per * D * sizeof(float);
  gnorm_team_bwd<T, TW, E, NCH, true><<<P, kThreads, smem, st>>>(xp, zp, wp, gp, static_cast<T*>(dx),
                                                                   static_cast<T*>(dz), static_cast<float*>(ws), rows,
                                                                   D, tl, eps, round_h, rpb);
  if (cudaGetLastError() != cudaSuccess) return GD_ERR_LAUNCH;
  gnorm_dw_sum_kernel<TW><<<(D + 31) / 32, dim3(32, 32), 0, st>>>(static_cast<float*>(ws), P, D,
                                                                   static_cast<TW*>(dw));
  return status_of(cudaGetLastError());
}

// the chunk width E and chunks a lane NCH as template arguments
template <typename T, typename TW, int E>
int fwd_e(const Shape& s, const void* x, const void* z, const void* w, void* o, long long rows, int D, float eps,
          bool round_h, cudaStream_t st) {
  switch (s.nch) {
    case 1: return team_fwd<T, TW, E, 1>(x, z, w, o, rows, D, s.team_log2, eps, round_h, st);
    case 2: return team_fwd<T, TW, E, 2>(x, z, w, o, rows, D, s.team_log2, eps, round_h, st);
    case 4: return team_fwd<T, TW, E, 4>(x, z, w, o, rows, D, s.team_log2, eps, round_h, st);
    default: return team_fwd<T, TW, E, 8>(x, z, w, o, rows, D, s.team_log2, eps, round_h, st);
  }
}
template <typename T, typename TW, int E>
int bwd_e(const Shape& s, const void* x, const void* z, const void* w, const void* dout, void* dx, void* dz, void* dw,
          long long rows, int D, float eps, bool round_h, void* ws, cudaStream_t st) {
  switch (s.nch) {
    case 1: return team_bwd<T, TW, E, 1>(x, z, w, dout, dx, dz, dw, rows, D, s.team_log2, eps, round_h, ws, st);
    case 2: return team_bwd<T, TW, E, 2>(x, z, w, dout, dx, dz, dw, rows, D, s.team_log2, eps, round_h, ws, st);
    case 4: return team_bwd<T, TW, E, 4>(x, z, w, dout, dx, dz, dw, rows, D, s.team_log2, eps, round_h, ws, st);
    default: return team_bwd<T, TW, E, 8>(x, z, w, dout, dx, dz, dw, rows, D, s.team_log2, eps, round_h, ws, st);
  }
}

template <typename T, typename TW>
int fwd_t(const void* x, const void* z, const void* w, void* o, long long rows, int D, float eps, cudaStream_t st) {
  const bool round_h = sizeof(T) == sizeof(TW);
  if constexpr (sizeof(T) == 2) {
    if (D == 128) {
      const long long per = (long long)kWarps * 2 * kRP;
      gnorm_fwd128_kernel<T, TW><<<(unsigned)((rows + per - 1) / per), kThreads, 0, st>>>(
          static_cast<const T*>(x), static_cast<const T*>(z), static_cast<const TW*>(w), static_cast<T*>(o), rows,
          eps, round_h);
      return status_of(cudaGetLastError());
    }
  }
  const Shape s = shape_for<T>(D);
  if constexpr (sizeof(T) == 2) {
    if (s.E == 8) return fwd_e<T, TW, 8>(s, x, z, w, o, rows, D, eps, round_h, st);
  }
  return fwd_e<T, TW, 4>(s, x, z, w, o, rows, D, eps, round_h, st);
}

template <typename T, typename TW>
int bwd_t(const void* x, const void* z, const void* w, const void* dout, void* dx, void* dz, void* dw, long long rows,
          int D, float eps, void* ws, cudaStream_t st) {
  const bool round_h = sizeof(T) == sizeof(TW);
  if constexpr (sizeof(T) == 2) {
    if (D == 128) {
      const T* xp = static_cast<const T*>(x);
      const T* zp = static_cast<const T*>(z);
      const TW* wp = static_cast<const TW*>(w);
      const T* gp = static_cast<const T*>(dout);
      const long long per = (long long)kWarps * 2 * kRP;
      if (dw == nullptr) {
        gnorm_bwd128_kernel<T, TW, false><<<(unsigned)((rows + per - 1) / per), kThreads, 0, st>>>(
            xp, zp, wp, gp, static_cast<T*>(dx), static_cast<T*>(dz), nullptr, rows, eps, round_h, 0);
        return status_of(cudaGetLastError());
      }
      long long rpb;
      int P;
      partition(rows, per, rpb, P);
      gnorm_bwd128_kernel<T, TW, true><<<P, kThreads, 0, st>>>(xp, zp, wp, gp, static_cast<T*>(dx),
                                                               static_cast<T*>(dz), static_cast<float*>(ws), rows, eps,
                                                               round_h, rpb);
      if (cudaGetLastError() != cudaSuccess) return GD_ERR_LAUNCH;
      gnorm_dw_sum_kernel<TW><<<(D + 31) / 32, dim3(32, 32), 0, st>>>(static_cast<float*>(ws), P, D,
                                                                       static_cast<TW*>(dw));
      return status_of(cudaGetLastError());
    }
  }
  const Shape s = shape_for<T>(D);
  if constexpr (sizeof(T) == 2) {
    if (s.E == 8) return bwd_e<T, TW, 8>(s, x, z, w, dout, dx, dz, dw, rows, D, eps, round_h, ws, st);
  }
  return bwd_e<T, TW, 4>(s, x, z, w, dout, dx, dz, dw, rows, D, eps, round_h, ws, st);
}

// w has x's dtype or is fp32 (the reference's supported(), _gated_norm.py:148-151)
int check_args(int dtype, int wdtype, long long rows, int D) {
  if (dtype < GD_FLOAT32 || dtype > GD_BFLOAT16) return GD_ERR_ARG;
  if (wdtype != dtype && wdtype != GD_FLOAT32) return GD_ERR_ARG;
  if (D <= 0 || D > kMaxD || D % 4 != 0 || rows < 0 || rows >= (1ll << 34)) return GD_ERR_SHAPE;  // grid.x < 2^31
  return GD_OK;
}

}  // namespace

extern "C" {

size_t gd_gnorm_workspace_bytes(long long rows, int D) {
  if (rows < 0 || D <= 0 || D > kMaxD) return 0;
  long long rpb;
  int P;
  partition(rows, kWarps, rpb, P);  // the smallest unit: enough partial rows for every path
  return (size_t)P * D * sizeof(float);
}

int gd_gnorm_fwd(const void* x, const void* z, const void* w, void* o, int dtype, int wdtype, long long rows, int D,
                 float eps, void* stream) {
  int s = check_args(dtype, wdtype, rows, D);
  if (s) return s;
  if (rows == 0) return GD_OK;
  if (!x || !z || !w || !o) return GD_ERR_ARG;
  if (!aligned16(x) || !aligned16(z) || !aligned16(w) || !aligned16(o)) return GD_ERR_ALIGN;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case GD_BFLOAT16:
      return wdtype == GD_FLOAT32 ? fwd_t<__nv_bfloat16, float>(x, z, w, o, rows, D, eps, st)
                                  : fwd_t<__nv_bfloat16, __nv_bfloat16>(x, z, w, o, rows, D, eps, st);
    case GD_FLOAT16:
      return wdtype == GD_FLOAT32 ? fwd_t<__half, float>(x, z, w, o, rows, D, eps, st)
                                  : fwd_t<__half, __half>(x, z, w, o, rows, D, eps, st);
    default: return fwd_t<float, float>(x, z, w, o, rows, D, eps, st);
  }
}

int gd_gnorm_bwd(const void* x, const void* z, const void* w, const void* dout, void* dx, void* dz, void* dw,
                 int dtype, int wdtype, long long rows, int D, float eps, void* workspace, size_t workspace_bytes,
                 void* stream) {
  int s = check_args(dtype, wdtype, rows, D);
  if (s) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (rows == 0) {  // no rows (the row pointers of empty tensors may be NULL): the weight's gradient is zero
    if (dw && cudaMemsetAsync(dw, 0, (size_t)D * (wdtype == GD_FLOAT32 ? 4 : 2), st) != cudaSuccess)
      return GD_ERR_LAUNCH;
    return GD_OK;
  }
  if (!x || !z || !w || !dout || !dx || !dz) return GD_ERR_ARG;
  if (dw != nullptr && (workspace == nullptr || workspace_bytes < gd_gnorm_workspace_bytes(rows, D)))
    return GD_ERR_WORKSPACE;
  if (!aligned16(x) || !aligned16(z) || !aligned16(w) || !aligned16(dout) || !aligned16(dx) || !aligned16(dz) ||
      !aligned16(workspace))
    return GD_ERR_ALIGN;
  switch (dtype) {
    case GD_BFLOAT16:
      return wdtype == GD_FLOAT32
                 ? bwd_t<__nv_bfloat16, float>(x, z, w, dout, dx, dz, dw, rows, D, eps, workspace, st)
                 : bwd_t<__nv_bfloat16, __nv_bfloat16>(x, z, w, dout, dx, dz, dw, rows, D, eps, workspace, st);
    case GD_FLOAT16:
      return wdtype == GD_FLOAT32 ? bwd_t<__half, float>(x, z, w, dout, dx, dz, dw, rows, D, eps, workspace, st)
                                  : bwd_t<__half, __half>(x, z, w, dout, dx, dz, dw, rows, D, eps, workspace, st);
    default: return bwd_t<float, float>(x, z, w, dout, dx, dz, dw, rows, D, eps, workspace, st);
  }
}

}  // extern "C"
