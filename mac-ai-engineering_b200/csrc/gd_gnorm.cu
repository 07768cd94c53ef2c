// The gated RMSNorm on the rule's output (transformers' Qwen3_5RMSNormGated over rows of one value head), one pass
// each way, mirroring the reference's gnorm_fwd / gnorm_bwd kernels (src/macai/layer/_gated_norm.py:1-16 formulas,
// :28-104 kernels, :127-137 column sum) and its autograd function (:154-197), with transformers' rounding points:
//   x_hat = x rsqrt(mean(x^2) + eps)                        (fp32)
//   h     = w x_hat.to(T)                                   (rounded to T again when w has x's dtype)
//   o     = (h silu(z)).to(T)
// backward in fp32, one rounding per gradient (s = silu(z), sig = sigmoid(z)):
//   dz = do h sig (1 + z (1 - sig)),  dx = r (dxh - x_hat <x_hat, dxh> / D) with dxh = do s w,
//   dw = sum over rows of do s x_hat.to(T)                  (only when asked: fixed-order partial rows, then a sum)
// x, z, o, dout, dx, dz: [rows, D] in T (fp32 / fp16 / bf16); w and dw: [D] in T or fp32. Any width: one warp a row,
// 4 adjacent elements a lane per 128 columns. D = 128 at 16 bits (the Qwen3.5 value heads): half a warp a row, 16-byte
// loads and stores, 4 rows a warp in flight. The row sums are warp shuffles. HBM-bound: the forward reads x
// and z and writes o (3 x 2 B per element at bf16), the backward reads x, z, dout and writes dx, dz (5 x 2 B).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "gated_delta_b200.h"

namespace {

constexpr int kThreads = 256;       // 8 warps, one row each at a time
constexpr int kWarps = kThreads / 32;
constexpr int kMaxPartials = 1024;  // CTAs of the backward with dw (its fixed-order partial rows)
constexpr int kMaxD = 1024;

// 4 consecutive elements <-> float4 (8-byte aligned start for 16-bit types, 16-byte for fp32)
__device__ __forceinline__ float4 ld4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ float4 ld4(const __nv_bfloat16* p) {
  const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ float4 ld4(const __half* p) {
  const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ void st4(__nv_bfloat16* p, float4 v) {
  const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<const uint32_t*>(&a);
  u.y = *reinterpret_cast<const uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}
__device__ __forceinline__ void st4(__half* p, float4 v) {
  const __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<const uint32_t*>(&a);
  u.y = *reinterpret_cast<const uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}

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
__device__ __forceinline__ float4 rnd4(float4 v) {
  return make_float4(rnd<T>(v.x), rnd<T>(v.y), rnd<T>(v.z), rnd<T>(v.w));
}

template <typename T>
__device__ __forceinline__ T cvt(float x);
template <>
__device__ __forceinline__ float cvt<float>(float x) { return x; }
template <>
__device__ __forceinline__ __half cvt<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 cvt<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float dot4(float4 a, float4 b) { return a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w; }
__device__ __forceinline__ float4 mul4(float4 a, float4 b) { return make_float4(a.x * b.x, a.y * b.y, a.z * b.z, a.w * b.w); }
__device__ __forceinline__ float4 scale4(float4 a, float s) { return make_float4(a.x * s, a.y * s, a.z * s, a.w * s); }
// sigmoid with the fast divide (2 ulp; a denominator past 2^126, z < -87, gives 0): the division's full-precision
// sequence made the kernels instruction-bound
__device__ __forceinline__ float sigmoid(float z) { return __fdividef(1.f, 1.f + expf(-z)); }

// 1 / sqrt(mean + eps) from a correctly rounded square root and division (PyTorch's rsqrt on the CPU rounds the same
// way to within an ulp)
__device__ __forceinline__ float inv_rms(float ss, int D, float eps) { return 1.f / sqrtf(ss / (float)D + eps); }

// the CH column groups (128 elements each) of one row: element offset of this lane's 4 in group j
__device__ __forceinline__ int col(int j, int lane) { return j * 128 + lane * 4; }

// ---- any width (D % 4 == 0, D <= 1024): one warp a row
template <typename T, typename TW, int CH>
__global__ void __launch_bounds__(kThreads) gnorm_fwd_kernel(const T* __restrict__ x, const T* __restrict__ z,
                                                             const TW* __restrict__ w, T* __restrict__ o,
                                                             long long rows, int D, float eps, bool round_h) {
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const T* xr = x + row * D;
  const T* zr = z + row * D;
  float4 xv[CH], zv[CH];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < CH; ++j) {  // every load in flight before any arithmetic
    const int i = col(j, lane);
    const bool in = i < D;
    xv[j] = in ? ld4(xr + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    zv[j] = in ? ld4(zr + i) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int j = 0; j < CH; ++j) ss += dot4(xv[j], xv[j]);
  const float r = inv_rms(warp_sum(ss), D, eps);
  T* orow = o + row * D;
#pragma unroll
  for (int j = 0; j < CH; ++j) {
    const int i = col(j, lane);
    if (i < D) {
      float4 h = mul4(ld4(w + i), rnd4<T>(scale4(xv[j], r)));
      if (round_h) h = rnd4<T>(h);
      const float4 zf = zv[j];
      const float4 s = make_float4(zf.x * sigmoid(zf.x), zf.y * sigmoid(zf.y), zf.z * sigmoid(zf.z), zf.w * sigmoid(zf.w));
      st4(orow + i, mul4(h, s));
    }
  }
}

// One row's backward; accumulates do s x_hat.to(T) into dwa when DW.
template <typename T, typename TW, int CH, bool DW>
__device__ __forceinline__ void gnorm_bwd_row(const T* __restrict__ x, const T* __restrict__ z,
                                              const TW* __restrict__ w, const T* __restrict__ dout,
                                              T* __restrict__ dx, T* __restrict__ dz, long long row, int D, float eps,
                                              bool round_h, int lane, float4 (&dwa)[CH]) {
  const size_t base = (size_t)row * D;
  float4 xv[CH], zv[CH], gv[CH];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < CH; ++j) {
    const int i = col(j, lane);
    const bool in = i < D;
    xv[j] = in ? ld4(x + base + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    zv[j] = in ? ld4(z + base + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    gv[j] = in ? ld4(dout + base + i) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int j = 0; j < CH; ++j) ss += dot4(xv[j], xv[j]);
  const float r = inv_rms(warp_sum(ss), D, eps);
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < CH; ++j) {
    const int i = col(j, lane);
    if (i < D) {
      const float4 wv = ld4(w + i);
      const float4 xn = scale4(xv[j], r);  // x_hat (fp32)
      const float4 xr4 = rnd4<T>(xn);      // x_hat.to(T)
      float4 h = mul4(wv, xr4);
      if (round_h) h = rnd4<T>(h);
      const float zz[4] = {zv[j].x, zv[j].y, zv[j].z, zv[j].w};
      const float hh[4] = {h.x, h.y, h.z, h.w};
      const float gg[4] = {gv[j].x, gv[j].y, gv[j].z, gv[j].w};
      float dzv[4], gs[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float sg = sigmoid(zz[e]);
        dzv[e] = gg[e] * hh[e] * sg * (1.f + zz[e] * (1.f - sg));
        gs[e] = gg[e] * (zz[e] * sg);  // do silu(z)
      }
      st4(dz + base + i, make_float4(dzv[0], dzv[1], dzv[2], dzv[3]));
      const float4 g4 = make_float4(gs[0], gs[1], gs[2], gs[3]);
      gv[j] = mul4(g4, wv);  // dxh, kept in gv
      acc += dot4(xn, gv[j]);
      if constexpr (DW) {
        const float4 t = mul4(g4, xr4);
        dwa[j].x += t.x;
        dwa[j].y += t.y;
        dwa[j].z += t.z;
        dwa[j].w += t.w;
      }
    }
  }
  const float c = warp_sum(acc) / (float)D;
#pragma unroll
  for (int j = 0; j < CH; ++j) {
    const int i = col(j, lane);
    if (i < D) {
      const float4 xn = scale4(xv[j], r);
      st4(dx + base + i, make_float4(r * (gv[j].x - xn.x * c), r * (gv[j].y - xn.y * c), r * (gv[j].z - xn.z * c),
                                     r * (gv[j].w - xn.w * c)));
    }
  }
}

// No dw: one row a warp. With dw: CTA p takes rows [p rpb, (p + 1) rpb), warp k rows k, k + 8, ...; the CTA's column
// sums (warps in order) go to partial row p.
template <typename T, typename TW, int CH, bool DW>
__global__ void __launch_bounds__(kThreads) gnorm_bwd_kernel(const T* __restrict__ x, const T* __restrict__ z,
                                                             const TW* __restrict__ w, const T* __restrict__ dout,
                                                             T* __restrict__ dx, T* __restrict__ dz,
                                                             float* __restrict__ part, long long rows, int D,
                                                             float eps, bool round_h, long long rpb) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float4 dwa[CH];
#pragma unroll
  for (int j = 0; j < CH; ++j) dwa[j] = make_float4(0.f, 0.f, 0.f, 0.f);
  if constexpr (!DW) {
    const long long row = (long long)blockIdx.x * kWarps + warp;
    if (row < rows) gnorm_bwd_row<T, TW, CH, false>(x, z, w, dout, dx, dz, row, D, eps, round_h, lane, dwa);
  } else {
    __shared__ __align__(16) float red[kWarps][kMaxD];
    const long long r0 = (long long)blockIdx.x * rpb;
    const long long r1 = r0 + rpb < rows ? r0 + rpb : rows;
    for (long long row = r0 + warp; row < r1; row += kWarps)
      gnorm_bwd_row<T, TW, CH, true>(x, z, w, dout, dx, dz, row, D, eps, round_h, lane, dwa);
#pragma unroll
    for (int j = 0; j < CH; ++j) {
      const int i = col(j, lane);
      if (i < D) *reinterpret_cast<float4*>(&red[warp][i]) = dwa[j];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < D; i += kThreads) {
      float s = 0.f;
#pragma unroll
      for (int k = 0; k < kWarps; ++k) s += red[k][i];
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

template <typename T, typename TW, int CH>
int fwd_c(const void* x, const void* z, const void* w, void* o, long long rows, int D, float eps, bool round_h,
          cudaStream_t st) {
  if constexpr (sizeof(T) == 2 && CH == 1) {
    if (D == 128) {
      const long long per = (long long)kWarps * 2 * kRP;
      gnorm_fwd128_kernel<T, TW><<<(unsigned)((rows + per - 1) / per), kThreads, 0, st>>>(
          static_cast<const T*>(x), static_cast<const T*>(z), static_cast<const TW*>(w), static_cast<T*>(o), rows,
          eps, round_h);
      return status_of(cudaGetLastError());
    }
  }
  const long long blocks = (rows + kWarps - 1) / kWarps;
  gnorm_fwd_kernel<T, TW, CH><<<(unsigned)blocks, kThreads, 0, st>>>(
      static_cast<const T*>(x), static_cast<const T*>(z), static_cast<const TW*>(w), static_cast<T*>(o), rows, D, eps,
      round_h);
  return status_of(cudaGetLastError());
}

template <typename T, typename TW, int CH>
int bwd_c(const void* x, const void* z, const void* w, const void* dout, void* dx, void* dz, void* dw, long long rows,
          int D, float eps, bool round_h, void* ws, cudaStream_t st) {
  const T* xp = static_cast<const T*>(x);
  const T* zp = static_cast<const T*>(z);
  const TW* wp = static_cast<const TW*>(w);
  const T* gp = static_cast<const T*>(dout);
  T* dxp = static_cast<T*>(dx);
  T* dzp = static_cast<T*>(dz);
  float* part = static_cast<float*>(ws);
  long long rpb = 0;
  int P = 0;
  if (dw) partition(rows, sizeof(T) == 2 && D == 128 ? (long long)kWarps * 2 * kRP : kWarps, rpb, P);
  bool done = false;
  if constexpr (sizeof(T) == 2 && CH == 1) {
    if (D == 128) {
      const long long per = (long long)kWarps * 2 * kRP;
      if (dw == nullptr)
        gnorm_bwd128_kernel<T, TW, false><<<(unsigned)((rows + per - 1) / per), kThreads, 0, st>>>(
            xp, zp, wp, gp, dxp, dzp, nullptr, rows, eps, round_h, 0);
      else
        gnorm_bwd128_kernel<T, TW, true><<<P, kThreads, 0, st>>>(xp, zp, wp, gp, dxp, dzp, part, rows, eps, round_h,
                                                                 rpb);
      done = true;
    }
  }
  if (!done) {
    if (dw == nullptr)
      gnorm_bwd_kernel<T, TW, CH, false><<<(unsigned)((rows + kWarps - 1) / kWarps), kThreads, 0, st>>>(
          xp, zp, wp, gp, dxp, dzp, nullptr, rows, D, eps, round_h, 0);
    else
      gnorm_bwd_kernel<T, TW, CH, true><<<P, kThreads, 0, st>>>(xp, zp, wp, gp, dxp, dzp, part, rows, D, eps,
                                                                round_h, rpb);
  }
  if (cudaGetLastError() != cudaSuccess) return GD_ERR_LAUNCH;
  if (dw == nullptr) return GD_OK;
  gnorm_dw_sum_kernel<TW><<<(D + 31) / 32, dim3(32, 32), 0, st>>>(part, P, D, static_cast<TW*>(dw));
  return status_of(cudaGetLastError());
}

// CH = ceil(D / 128) column groups: 1, 2, 4 or 8 (D <= 1024)
template <typename T, typename TW>
int fwd_t(const void* x, const void* z, const void* w, void* o, long long rows, int D, float eps, cudaStream_t st) {
  const bool round_h = sizeof(T) == sizeof(TW);
  if (D <= 128) return fwd_c<T, TW, 1>(x, z, w, o, rows, D, eps, round_h, st);
  if (D <= 256) return fwd_c<T, TW, 2>(x, z, w, o, rows, D, eps, round_h, st);
  if (D <= 512) return fwd_c<T, TW, 4>(x, z, w, o, rows, D, eps, round_h, st);
  return fwd_c<T, TW, 8>(x, z, w, o, rows, D, eps, round_h, st);
}

template <typename T, typename TW>
int bwd_t(const void* x, const void* z, const void* w, const void* dout, void* dx, void* dz, void* dw, long long rows,
          int D, float eps, void* ws, cudaStream_t st) {
  const bool round_h = sizeof(T) == sizeof(TW);
  if (D <= 128) return bwd_c<T, TW, 1>(x, z, w, dout, dx, dz, dw, rows, D, eps, round_h, ws, st);
  if (D <= 256) return bwd_c<T, TW, 2>(x, z, w, dout, dx, dz, dw, rows, D, eps, round_h, ws, st);
  if (D <= 512) return bwd_c<T, TW, 4>(x, z, w, dout, dx, dz, dw, rows, D, eps, round_h, ws, st);
  return bwd_c<T, TW, 8>(x, z, w, dout, dx, dz, dw, rows, D, eps, round_h, ws, st);
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
