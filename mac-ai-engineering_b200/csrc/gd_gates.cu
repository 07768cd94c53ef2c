// The linear-attention layer's gates in one pass each way (the reference's gates_fwd / gates_bwd Metal kernels,
// src/macai/layer/_gates.py:27-63, and its autograd function :82-117):
//   beta = sigmoid(b),  g = -exp(A_log) softplus(a + dt_bias)     (softplus(x) = x above 20, PyTorch's threshold)
//   db = dbeta beta (1 - beta),  da = dg (-exp(A_log)) sigmoid(x)   (1 above the threshold), x = a + dt_bias
//   dA_log = sum over tokens of dg g,  ddt_bias = sum over tokens of da (before its cast)
// b, a, db, da: [rows, H] in the input dtype (bf16 / fp16 / fp32); A_log, dt_bias and their gradients: [H] in the weight
// dtype; beta, g, dbeta, dg: fp32. Elementwise work is HBM-bound: one read of b and a, one write of beta and g (the
// backward: reads b, a, dbeta, dg; writes db, da). The per-head sums are deterministic: every CTA sums a fixed block of
// rows per head in a fixed order into a partial row, and a second kernel sums the partial rows in order.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "gated_delta_b200.h"

namespace {

constexpr float kThreshold = 20.f;
constexpr int kThreads = 256;
constexpr int kMaxPartials = 1024;  // CTAs of the backward with per-head sums (rows split into this many blocks at most)
constexpr int kSmemHeads = 1024;    // heads whose per-head constants are staged in shared memory (8 KB)

template <typename T>
__device__ __forceinline__ float ld(const T* p, size_t i);
template <>
__device__ __forceinline__ float ld<float>(const float* p, size_t i) { return __ldg(p + i); }
template <>
__device__ __forceinline__ float ld<__half>(const __half* p, size_t i) { return __half2float(p[i]); }
template <>
__device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p, size_t i) {
  return __bfloat162float(p[i]);
}

template <typename T>
__device__ __forceinline__ T cvt(float x);
template <>
__device__ __forceinline__ float cvt<float>(float x) { return x; }
template <>
__device__ __forceinline__ __half cvt<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 cvt<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// 8 consecutive elements (16-byte aligned start) to / from float
__device__ __forceinline__ float2 unpack2(uint32_t w, const __nv_bfloat16*) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
}
__device__ __forceinline__ float2 unpack2(uint32_t w, const __half*) {
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}
__device__ __forceinline__ uint32_t pack2(float x, float y, const __nv_bfloat16*) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(x, y);
  return *reinterpret_cast<const uint32_t*>(&v);
}
__device__ __forceinline__ uint32_t pack2(float x, float y, const __half*) {
  const __half2 v = __floats2half2_rn(x, y);
  return *reinterpret_cast<const uint32_t*>(&v);
}
template <typename T>
__device__ __forceinline__ void ld8(const T* p, float (&v)[8]) {
  if constexpr (sizeof(T) == 4) {
    const float4 x = __ldg(reinterpret_cast<const float4*>(p)), y = __ldg(reinterpret_cast<const float4*>(p) + 1);
    v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w; v[4] = y.x; v[5] = y.y; v[6] = y.z; v[7] = y.w;
  } else {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack2(w[j], p);
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
  }
}
template <typename T>
__device__ __forceinline__ void st8(T* p, const float (&v)[8]) {
  if constexpr (sizeof(T) == 4) {
    reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    *reinterpret_cast<uint4*>(p) = make_uint4(pack2(v[0], v[1], p), pack2(v[2], v[3], p), pack2(v[4], v[5], p),
                                              pack2(v[6], v[7], p));
  }
}
__device__ __forceinline__ void ld8f(const float* p, float (&v)[8]) {
  if (p == nullptr) {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = 0.f;
    return;
  }
  const float4 x = __ldg(reinterpret_cast<const float4*>(p)), y = __ldg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w; v[4] = y.x; v[5] = y.y; v[6] = y.z; v[7] = y.w;
}

// the fast divide (2 ulp; a denominator past 2^126, x < -87, gives 0)
__device__ __forceinline__ float sigmoid(float x) { return __fdividef(1.f, 1.f + expf(-x)); }
// Both arms are computed before the select (the expensive one on x clamped at the threshold, so it stays finite; a NaN
// still propagates): a select with an expensive arm is compiled into per-element branches that serialise the chains
// of a vector group.
__device__ __forceinline__ float softplus(float x) {
  const float s = log1pf(expf(x > kThreshold ? kThreshold : x));
  return x > kThreshold ? x : s;
}
__device__ __forceinline__ float dsoftplus(float x) {  // PyTorch's softplus backward: 1 above the threshold
  const float s = sigmoid(x > kThreshold ? kThreshold : x);
  return x > kThreshold ? 1.f : s;
}

// per-head constants -exp(A_log) and dt_bias, staged once per CTA (heads beyond kSmemHeads read from global)
template <typename TW>
__device__ __forceinline__ void stage_heads(const TW* alog, const TW* dtb, int H, float* s_na, float* s_dt) {
  const int hs = H < kSmemHeads ? H : kSmemHeads;
  for (int h = threadIdx.x; h < hs; h += blockDim.x) {
    s_na[h] = -expf(ld(alog, h));
    s_dt[h] = ld(dtb, h);
  }
  __syncthreads();
}

template <typename TW>
__device__ __forceinline__ void head_consts(const TW* alog, const TW* dtb, const float* s_na, const float* s_dt, int h,
                                            float& na, float& dt) {
  if (h < kSmemHeads) {
    na = s_na[h];
    dt = s_dt[h];
  } else {
    na = -expf(ld(alog, h));
    dt = ld(dtb, h);
  }
}

// Each thread takes groups of 8 consecutive elements; vec: every pointer 16-byte aligned, so whole groups move as
// 16-byte pieces (the tail group, and every group when vec is false, element by element).
template <typename T, typename TW>
__global__ void __launch_bounds__(kThreads) gates_fwd_kernel(const T* __restrict__ b, const T* __restrict__ a,
                                                             const TW* __restrict__ alog, const TW* __restrict__ dtb,
                                                             float* __restrict__ beta, float* __restrict__ g,
                                                             int n, int H, bool vec) {
  __shared__ float s_na[kSmemHeads], s_dt[kSmemHeads];
  stage_heads(alog, dtb, H, s_na, s_dt);
  const int groups = (n + 7) / 8, stride = gridDim.x * blockDim.x;
  // group i0 .. i0 + 7 from its loaded b, a
  auto out8 = [&](int i0, const float (&vb)[8], const float (&va)[8]) {
    float ob[8], og[8];
    int h = i0 % H;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float na, dt;
      head_consts(alog, dtb, s_na, s_dt, h, na, dt);
      ob[j] = sigmoid(vb[j]);
      og[j] = na * softplus(va[j] + dt);
      h = h + 1 == H ? 0 : h + 1;
    }
    st8(beta + i0, ob);
    st8(g + i0, og);
  };
  auto scalar = [&](int i0) {  // the tail group, or any group when the pointers are not 16-byte aligned
    int h = i0 % H;
    for (int i = i0; i < n && i < i0 + 8; ++i) {
      float na, dt;
      head_consts(alog, dtb, s_na, s_dt, h, na, dt);
      beta[i] = sigmoid(ld(b, i));
      g[i] = na * softplus(ld(a, i) + dt);
      h = h + 1 == H ? 0 : h + 1;
    }
  };
  // two groups a step (gi and gi + stride), their four 16-byte loads in flight before either is computed
  for (int gi = blockIdx.x * blockDim.x + threadIdx.x; gi < groups; gi += 2 * stride) {
    const int gj = gi + stride;
    if (vec && 8 * gj + 8 <= n) {
      float vb0[8], va0[8], vb1[8], va1[8];
      ld8(b + 8 * gi, vb0);
      ld8(a + 8 * gi, va0);
      ld8(b + 8 * gj, vb1);
      ld8(a + 8 * gj, va1);
      out8(8 * gi, vb0, va0);
      out8(8 * gj, vb1, va1);
    } else {
      for (int gk = gi; gk < groups && gk <= gj; gk += stride) {
        if (vec && 8 * gk + 8 <= n) {
          float vb[8], va[8];
          ld8(b + 8 * gk, vb);
          ld8(a + 8 * gk, va);
          out8(8 * gk, vb, va);
        } else {
          scalar(8 * gk);
        }
      }
    }
  }
}

// Elementwise db, da; with sums, CTA p also owns rows [p * rpb, (p + 1) * rpb) and writes its per-head totals of
// dg * g and of da to partial rows p of pa / pd ([P][H] fp32). Thread t covers head t % H of rows t / H, t / H + K, ...
// (K = blockDim / H rows at a time, so consecutive threads read consecutive elements); the CTA's totals per head are
// then summed over its K row lanes in order.
template <typename T, typename TW>
__global__ void __launch_bounds__(kThreads) gates_bwd_kernel(const T* __restrict__ b, const T* __restrict__ a,
                                                             const TW* __restrict__ alog, const TW* __restrict__ dtb,
                                                             const float* __restrict__ dbeta,
                                                             const float* __restrict__ dg, T* __restrict__ db,
                                                             T* __restrict__ da, long long rows, int H, long long rpb,
                                                             float* __restrict__ pa, float* __restrict__ pd, bool vec) {
  __shared__ float s_na[kSmemHeads], s_dt[kSmemHeads];
  __shared__ float s_sa[kThreads], s_sd[kThreads];
  stage_heads(alog, dtb, H, s_na, s_dt);
  const bool sums = pa != nullptr;
  if (!sums) {  // plain elementwise pass in groups of 8 (as the forward)
    const int n = (int)(rows * H), groups = (n + 7) / 8, stride = gridDim.x * blockDim.x;
    for (int gi = blockIdx.x * blockDim.x + threadIdx.x; gi < groups; gi += stride) {
      const int i0 = 8 * gi;
      int h = i0 % H;
      if (vec && i0 + 8 <= n) {
        float vb[8], va[8], vdb[8], vdg[8], ob[8], oa[8];
        ld8(b + i0, vb);
        ld8(a + i0, va);
        ld8f(dbeta ? dbeta + i0 : nullptr, vdb);
        ld8f(dg ? dg + i0 : nullptr, vdg);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float na, dt;
          head_consts(alog, dtb, s_na, s_dt, h, na, dt);
          const float sb = sigmoid(vb[j]);
          ob[j] = vdb[j] * sb * (1.f - sb);
          const float x = va[j] + dt;
          oa[j] = vdg[j] * na * dsoftplus(x);
          h = h + 1 == H ? 0 : h + 1;
        }
        st8(db + i0, ob);
        st8(da + i0, oa);
      } else {
        for (int i = i0; i < n && i < i0 + 8; ++i) {
          float na, dt;
          head_consts(alog, dtb, s_na, s_dt, h, na, dt);
          const float sb = sigmoid(ld(b, i));
          db[i] = cvt<T>((dbeta ? dbeta[i] : 0.f) * sb * (1.f - sb));
          const float x = ld(a, i) + dt;
          const float sx = dsoftplus(x);
          da[i] = cvt<T>((dg ? dg[i] : 0.f) * na * sx);
          h = h + 1 == H ? 0 : h + 1;
        }
      }
    }
    return;
  }
  const long long r0 = (long long)blockIdx.x * rpb;
  const long long r1 = r0 + rpb < rows ? r0 + rpb : rows;
  for (int h0 = 0; h0 < H; h0 += kThreads) {  // head blocks of up to kThreads
    const int hn = H - h0 < kThreads ? H - h0 : kThreads;
    const int K = kThreads / hn;  // row lanes
    const int t = threadIdx.x, h = h0 + t % hn, lane_r = t / hn;
    float sa = 0.f, sd = 0.f;
    if (lane_r < K) {
      float na, dt;
      head_consts(alog, dtb, s_na, s_dt, h, na, dt);
      for (long long r = r0 + lane_r; r < r1; r += K) {
        const size_t i = (size_t)r * H + h;
        const float sb = sigmoid(ld(b, i));
        db[i] = cvt<T>((dbeta ? dbeta[i] : 0.f) * sb * (1.f - sb));
        const float x = ld(a, i) + dt;
        const float sx = dsoftplus(x);
        const float dgi = dg ? dg[i] : 0.f;
        const float dai = dgi * na * sx;
        da[i] = cvt<T>(dai);
        sa = fmaf(dgi, na * softplus(x), sa);  // dg * g
        sd += dai;
      }
    }
    s_sa[t] = sa;
    s_sd[t] = sd;
    __syncthreads();
    if (t < hn) {
      float ta = 0.f, td = 0.f;
      for (int k = 0; k < K; ++k) {
        ta += s_sa[k * hn + t];
        td += s_sd[k * hn + t];
      }
      pa[(size_t)blockIdx.x * H + h0 + t] = ta;
      pd[(size_t)blockIdx.x * H + h0 + t] = td;
    }
    __syncthreads();
  }
}

// dA_log[h] = sum_p pa[p][h], ddt_bias[h] = sum_p pd[p][h], in partial order
template <typename TW>
__global__ void __launch_bounds__(kThreads) gates_sum_kernel(const float* __restrict__ pa,
                                                             const float* __restrict__ pd, int P, int H,
                                                             TW* __restrict__ dalog, TW* __restrict__ ddtb) {
  const int h = blockIdx.x * blockDim.x + threadIdx.x;
  if (h >= H) return;
  float ta = 0.f, td = 0.f;
  for (int p = 0; p < P; ++p) {
    ta += pa[(size_t)p * H + h];
    td += pd[(size_t)p * H + h];
  }
  if (dalog) dalog[h] = cvt<TW>(ta);
  if (ddtb) ddtb[h] = cvt<TW>(td);
}

int blocks_for(long long n) {  // n = work items (groups of 8 elements)
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long want = (n + kThreads - 1) / kThreads;
  const long long cap = (long long)sms * 8;
  return (int)(want < cap ? (want > 0 ? want : 1) : cap);
}

// rows per partial block and the number of partial rows for the per-head sums
void partition(long long rows, long long& rpb, int& P) {
  rpb = (rows + kMaxPartials - 1) / kMaxPartials;
  if (rpb < 16) rpb = 16;
  P = (int)((rows + rpb - 1) / rpb);
  if (P < 1) P = 1;
}

bool aligned4(const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }
bool aligned16(const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int status_of(cudaError_t e) { return e == cudaSuccess ? GD_OK : GD_ERR_LAUNCH; }

template <typename T, typename TW>
int fwd_t(const void* b, const void* a, const void* alog, const void* dtb, float* beta, float* g, long long n, int H,
          cudaStream_t st) {
  const bool vec = aligned16(b) && aligned16(a) && aligned16(beta) && aligned16(g);
  gates_fwd_kernel<T, TW><<<blocks_for((n + 7) / 8), kThreads, 0, st>>>(
      static_cast<const T*>(b), static_cast<const T*>(a), static_cast<const TW*>(alog), static_cast<const TW*>(dtb),
      beta, g, (int)n, H, vec);
  return status_of(cudaGetLastError());
}

template <typename T, typename TW>
int bwd_t(const void* b, const void* a, const void* alog, const void* dtb, const float* dbeta, const float* dg,
          void* db, void* da, void* dalog, void* ddtb, long long n, int H, void* ws, cudaStream_t st) {
  const long long rows = n / H;
  if (dalog == nullptr && ddtb == nullptr) {
    const bool vec = aligned16(b) && aligned16(a) && aligned16(dbeta) && aligned16(dg) && aligned16(db) &&
                     aligned16(da);
    gates_bwd_kernel<T, TW><<<blocks_for((n + 7) / 8), kThreads, 0, st>>>(
        static_cast<const T*>(b), static_cast<const T*>(a), static_cast<const TW*>(alog), static_cast<const TW*>(dtb),
        dbeta, dg, static_cast<T*>(db), static_cast<T*>(da), rows, H, 0, nullptr, nullptr, vec);
    return status_of(cudaGetLastError());
  }
  long long rpb;
  int P;
  partition(rows, rpb, P);
  float* pa = static_cast<float*>(ws);
  float* pd = pa + (size_t)P * H;
  gates_bwd_kernel<T, TW><<<P, kThreads, 0, st>>>(
      static_cast<const T*>(b), static_cast<const T*>(a), static_cast<const TW*>(alog), static_cast<const TW*>(dtb),
      dbeta, dg, static_cast<T*>(db), static_cast<T*>(da), rows, H, rpb, pa, pd, false);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return GD_ERR_LAUNCH;
  gates_sum_kernel<TW><<<(H + kThreads - 1) / kThreads, kThreads, 0, st>>>(pa, pd, P, H, static_cast<TW*>(dalog),
                                                                            static_cast<TW*>(ddtb));
  return status_of(cudaGetLastError());
}

template <typename T>
int fwd_w(int wdtype, const void* b, const void* a, const void* alog, const void* dtb, float* beta, float* g,
          long long n, int H, cudaStream_t st) {
  switch (wdtype) {
    case GD_BFLOAT16: return fwd_t<T, __nv_bfloat16>(b, a, alog, dtb, beta, g, n, H, st);
    case GD_FLOAT16: return fwd_t<T, __half>(b, a, alog, dtb, beta, g, n, H, st);
    default: return fwd_t<T, float>(b, a, alog, dtb, beta, g, n, H, st);
  }
}

template <typename T>
int bwd_w(int wdtype, const void* b, const void* a, const void* alog, const void* dtb, const float* dbeta,
          const float* dg, void* db, void* da, void* dalog, void* ddtb, long long n, int H, void* ws, cudaStream_t st) {
  switch (wdtype) {
    case GD_BFLOAT16: return bwd_t<T, __nv_bfloat16>(b, a, alog, dtb, dbeta, dg, db, da, dalog, ddtb, n, H, ws, st);
    case GD_FLOAT16: return bwd_t<T, __half>(b, a, alog, dtb, dbeta, dg, db, da, dalog, ddtb, n, H, ws, st);
    default: return bwd_t<T, float>(b, a, alog, dtb, dbeta, dg, db, da, dalog, ddtb, n, H, ws, st);
  }
}

int check_args(int dtype, int wdtype, long long n, int H) {
  if (dtype < GD_FLOAT32 || dtype > GD_BFLOAT16 || wdtype < GD_FLOAT32 || wdtype > GD_BFLOAT16) return GD_ERR_ARG;
  if (H <= 0 || n < 0 || n % H != 0 || n >= (1ll << 31)) return GD_ERR_SHAPE;
  return GD_OK;
}

}  // namespace

extern "C" {

size_t gd_gates_workspace_bytes(long long n, int H) {
  if (H <= 0 || n < 0 || n % H != 0) return 0;
  long long rpb;
  int P;
  partition(n / H, rpb, P);
  return (size_t)2 * P * H * sizeof(float);
}

int gd_gates_fwd(const void* b, const void* a, const void* A_log, const void* dt_bias, float* beta, float* g,
                 int dtype, int wdtype, long long n, int H, void* stream) {
  int s = check_args(dtype, wdtype, n, H);
  if (s) return s;
  if (n == 0) return GD_OK;
  if (!b || !a || !A_log || !dt_bias || !beta || !g) return GD_ERR_ARG;
  if (!aligned4(beta) || !aligned4(g)) return GD_ERR_ALIGN;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case GD_BFLOAT16: return fwd_w<__nv_bfloat16>(wdtype, b, a, A_log, dt_bias, beta, g, n, H, st);
    case GD_FLOAT16: return fwd_w<__half>(wdtype, b, a, A_log, dt_bias, beta, g, n, H, st);
    default: return fwd_w<float>(wdtype, b, a, A_log, dt_bias, beta, g, n, H, st);
  }
}

int gd_gates_bwd(const void* b, const void* a, const void* A_log, const void* dt_bias, const float* dbeta,
                 const float* dg, void* db, void* da, void* dA_log, void* ddt_bias, int dtype, int wdtype, long long n,
                 int H, void* workspace, size_t workspace_bytes, void* stream) {
  int s = check_args(dtype, wdtype, n, H);
  if (s) return s;
  if (!b || !a || !A_log || !dt_bias || !db || !da) return GD_ERR_ARG;
  const bool sums = dA_log != nullptr || ddt_bias != nullptr;
  if (sums && (workspace == nullptr || workspace_bytes < gd_gates_workspace_bytes(n, H))) return GD_ERR_WORKSPACE;
  if (!aligned4(workspace) || !aligned4(dbeta) || !aligned4(dg)) return GD_ERR_ALIGN;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n == 0) {  // no tokens: the per-head sums are zero
    if (!sums) return GD_OK;
    const size_t wb = wdtype == GD_FLOAT32 ? 4 : 2;
    if (dA_log && cudaMemsetAsync(dA_log, 0, wb * H, st) != cudaSuccess) return GD_ERR_LAUNCH;
    if (ddt_bias && cudaMemsetAsync(ddt_bias, 0, wb * H, st) != cudaSuccess) return GD_ERR_LAUNCH;
    return GD_OK;
  }
  switch (dtype) {
    case GD_BFLOAT16:
      return bwd_w<__nv_bfloat16>(wdtype, b, a, A_log, dt_bias, dbeta, dg, db, da, dA_log, ddt_bias, n, H, workspace, st);
    case GD_FLOAT16:
      return bwd_w<__half>(wdtype, b, a, A_log, dt_bias, dbeta, dg, db, da, dA_log, ddt_bias, n, H, workspace, st);
    default:
      return bwd_w<float>(wdtype, b, a, A_log, dt_bias, dbeta, dg, db, da, dA_log, ddt_bias, n, H, workspace, st);
  }
}

}  // extern "C"
