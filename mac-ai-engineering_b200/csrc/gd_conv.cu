// The linear-attention layer's convolution path (the step that produces the rule's q, k, v), one pass each way.
//
// What it computes (the reference's formulas, src/macai/layer/_conv.py:1-21, and its autograd contract, :188-237):
//   u[t, c] = sum_j w[c, j] x[t - 3 + j, c]        kernel 4, no bias, zero before the sequence start; fp32
//   y = u sigmoid(u)                               on the fp32 u, rounded once
//   q, k = y's channel blocks [0, KD) and [KD, 2 KD) as [B, T, H_v, DK] in x's dtype, key head h written to value
//          heads h REP .. h REP + REP - 1 (the repeat_interleave of the Qwen3.5 layer, without a copy)
//   v    = y's channels [2 KD, C) as [B, T, H_v, DV] in fp32
// and backward (x saved, u recomputed):
//   du = dy sigmoid(u) (1 + u (1 - sigmoid(u)))    dy of a q / k channel = the sum of its REP copies' cotangents
//   dx[t, c] = sum_j w[c, j] du[t + 3 - j, c]      du = 0 past the sequence end; [B, T, C] in x's dtype
//   dw[c, j] = sum_{b, t} du[t, c] x[t - 3 + j, c] only when asked: fixed-order partial rows, then a tree sum
//
// How (B200): the work is cut into windows of CW channels (one 256-byte span of x's rows) by 64 (forward) or 32
// (backward) time steps of one batch row. A CTA owns one channel window and walks a run of consecutive (batch row, time tile) windows. Each
// window's x rows, with the 3 rows of history before it (and in the backward the 3 rows after it), arrive in shared
// memory by one TMA tensor copy (a ring of three stages forward, two backward: later windows' copies are in flight
// while this one is computed; rows before the sequence start arrive as zeros, which is the causal padding). A thread owns one 16-byte channel
// group and every 16th row of the window, and forms each output from the 4 staged rows it needs: no state carried
// from one time step to the next. The backward first writes du for the window's rows (and the 3 after it) into a
// shared fp32 tile, then forms dx from that tile; its cotangents (each read once) are staged a window ahead by
// per-thread asynchronous 16-byte copies. Outputs are written once each with 16-byte streaming stores. HBM-bound
// elementwise work: no tensor cores.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

#include "gd_common.cuh"

namespace {

using gd::mbar_arrive_expect_tx;
using gd::mbar_init;
using gd::mbar_try_wait;
using gd::smem_u32;

constexpr int kThreads = 256;
constexpr int kTT = 64;              // time steps a window holds
constexpr int kMaxPartials = 256;    // partial rows of dw at most (the CTAs' runs of windows)
constexpr int kMaxGridY = 65535;
constexpr long long kWaitBudget = 4000000000ll;  // SM clocks a copy wait may take (~2 s) before the CTA gives up

// channels a 16-byte group holds, channel groups a 256-byte window row holds
template <typename T>
struct Geo {
  static constexpr int G = 16 / (int)sizeof(T);
  static constexpr int CW = 256 / (int)sizeof(T);
  static constexpr int NG = CW / G;              // 16
  static constexpr int RSTEP = kThreads / NG;    // rows a pass of the CTA covers (16)
};

// ---- 16-byte groups <-> floats
template <typename T>
__device__ __forceinline__ void unpack(uint4 u, float (&f)[16 / sizeof(T)]);
template <>
__device__ __forceinline__ void unpack<float>(uint4 u, float (&f)[4]) {
  f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y); f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
}
template <>
__device__ __forceinline__ void unpack<__nv_bfloat16>(uint4 u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
template <>
__device__ __forceinline__ void unpack<__half>(uint4 u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 p = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    f[2 * i] = p.x;
    f[2 * i + 1] = p.y;
  }
}
template <typename T>
__device__ __forceinline__ uint4 pack(const float (&f)[16 / sizeof(T)]);
template <>
__device__ __forceinline__ uint4 pack<float>(const float (&f)[4]) {
  return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
}
template <>
__device__ __forceinline__ uint4 pack<__nv_bfloat16>(const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 p = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&p);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}
template <>
__device__ __forceinline__ uint4 pack<__half>(const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2 p = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&p);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

template <typename TW>
__device__ __forceinline__ float weight_at(const TW* p) {
  if constexpr (std::is_same<TW, float>::value) {
    return __ldg(p);
  } else if constexpr (std::is_same<TW, __half>::value) {
    return __half2float(p[0]);
  } else {
    return __bfloat162float(p[0]);
  }
}

__device__ __forceinline__ float sigm(float u) { return __fdividef(1.f, 1.f + expf(-u)); }

// Where a channel group's results go. Channels c < KD are q (key head c / DK), KD <= c < 2 KD are k, the rest v
// (value head (c - 2 KD) / DV). `col` is the element offset of the group's first channel inside one token's row of
// its output ([H_v * DK] for q / k, copy r at col + r * DK; [H_v * DV] for v); row_len is that row's length.
struct Dest {
  int kind;  // 0 q, 1 k, 2 v, -1 past C
  long long col, row_len;
};
__device__ __forceinline__ Dest dest_of(int c, int C, int KD, int DK, int REP, int DV) {
  Dest d;
  if (c >= C) {
    d.kind = -1;
    d.col = d.row_len = 0;
  } else if (c < 2 * KD) {
    d.kind = c < KD ? 0 : 1;
    const int cq = c - d.kind * KD;
    d.col = (long long)(cq / DK) * REP * DK + cq % DK;
    d.row_len = (long long)KD * REP;
  } else {
    d.kind = 2;
    const int cv = c - 2 * KD;
    d.col = (long long)(cv / DV) * DV + cv % DV;
    d.row_len = C - 2 * KD;
  }
  return d;
}

// 3-D tiled copy of x [B, T, C] (C innermost) into shared memory: box {CW channels, rows, 1 batch row} at (c0, t, b)
__device__ __forceinline__ void tma_x(void* dst, const CUtensorMap* map, int c0, int t, int b, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(t), "r"(b), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ bool wait_copy(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity))
    if (clock64() - t0 > kWaitBudget) return false;
  return true;
}

// the run of windows of grid row blockIdx.y: windows [first, last) of the (batch row, time tile) order
struct Run {
  long long first, last;
  int ntile;  // time tiles a batch row has
  __device__ __forceinline__ void window(long long i, int& b, int& t0) const {
    b = (int)(i / ntile);
    t0 = (int)(i % ntile) * kTT;
  }
};

// ------------------------------------------------------------------------------------------------------------------
// forward: a three-stage ring of x windows, kTT + 3 staged rows each (row 0 = time t0 - 3)

constexpr int kStagesF = 3;

template <typename T, typename TW>
__global__ void __launch_bounds__(kThreads, 4) conv_window_fwd(const __grid_constant__ CUtensorMap xmap,
                                                               const TW* __restrict__ w, T* __restrict__ qo,
                                                               T* __restrict__ ko, float* __restrict__ vo, int B,
                                                               int Tn, int C, int KD, int DK, int REP, int DV,
                                                               long long per_run) {
  using Gm = Geo<T>;
  constexpr int G = Gm::G, CW = Gm::CW, ROWS = kTT + 3;
  constexpr int STAGE = ROWS * 256;  // bytes
  extern __shared__ __align__(128) unsigned char sm[];
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + kStagesF * STAGE);
  const int tid = threadIdx.x, grp = tid % Gm::NG, row0 = tid / Gm::NG;
  const int c0 = blockIdx.x * CW, c = c0 + grp * G;
  Run run;
  run.ntile = (Tn + kTT - 1) / kTT;
  run.first = (long long)blockIdx.y * per_run;
  const long long total = (long long)B * run.ntile;
  run.last = run.first + per_run < total ? run.first + per_run : total;
  const long long n = run.last - run.first;
  if (n <= 0) return;
  if (tid == 0) {
    for (int s = 0; s < kStagesF; ++s) mbar_init(full + s, 1);
    gd::fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](long long i) {  // window first + i into stage i % kStagesF
    int b, t0;
    run.window(run.first + i, b, t0);
    const int s = (int)(i % kStagesF);
    mbar_arrive_expect_tx(full + s, (uint32_t)STAGE);
    tma_x(sm + s * STAGE, &xmap, c0, t0 - 3, b, full + s);
  };
  if (tid == 0)
    for (long long i = 0; i < kStagesF && i < n; ++i) issue(i);
  // the group's 4 taps (tap j multiplies x[t - 3 + j]) and its destination
  float tap[4][G];
#pragma unroll
  for (int i = 0; i < G; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) tap[j][i] = c + i < C ? weight_at(w + (size_t)(c + i) * 4 + j) : 0.f;
  const Dest d = dest_of(c, C, KD, DK, REP, DV);
  for (long long i = 0; i < n; ++i) {
    const int s = (int)(i % kStagesF);
    const unsigned char* st = sm + s * STAGE;
    const bool landed = wait_copy(full + s, (uint32_t)((i / kStagesF) & 1));
    if (!__syncthreads_and(landed)) return;
    int b, t0;
    run.window(run.first + i, b, t0);
    if (d.kind >= 0) {
#pragma unroll 2
      for (int r = row0; r < kTT; r += Gm::RSTEP) {
        const int t = t0 + r;
        if (t >= Tn) break;
        float y[G];
        {
          float xv[4][G];  // staged rows r .. r + 3 = times t - 3 .. t
#pragma unroll
          for (int j = 0; j < 4; ++j)
            unpack<T>(*reinterpret_cast<const uint4*>(st + (r + j) * 256 + grp * 16), xv[j]);
#pragma unroll
          for (int e = 0; e < G; ++e) {
            float u = tap[3][e] * xv[3][e];
            u = fmaf(tap[2][e], xv[2][e], u);
            u = fmaf(tap[1][e], xv[1][e], u);
            u = fmaf(tap[0][e], xv[0][e], u);
            y[e] = u * sigm(u);
          }
        }
        const long long tok = (long long)b * Tn + t;
        if (d.kind == 2) {
          float* p = vo + tok * d.row_len + d.col;
#pragma unroll
          for (int e = 0; e < G; e += 4)
            __stcs(reinterpret_cast<float4*>(p + e), make_float4(y[e], y[e + 1], y[e + 2], y[e + 3]));
        } else {
          T* p = (d.kind == 0 ? qo : ko) + tok * d.row_len + d.col;
          const uint4 u = pack<T>(y);
          for (int rr = 0; rr < REP; ++rr) __stcs(reinterpret_cast<uint4*>(p + (long long)rr * DK), u);
        }
      }
    }
    __syncthreads();  // every thread is done with this stage: it may be refilled
    if (tid == 0 && i + kStagesF < n) issue(i + kStagesF);
  }
}

// ------------------------------------------------------------------------------------------------------------------
// backward: windows of kTB time steps. Per window, in shared memory:
//   x    [kTB + 6 rows][256 B]          by TMA, row 0 = time t0 - 3 (kStagesB stages)
//   cot  [kTB + 3 rows][NG groups][SLOT] the cotangents of times t0 .. t0 + kTB + 2, copied by each thread for its
//                                        own (row, group) slots with cp.async (kStagesB stages; rows past T
//                                        zero-filled):
//                                        a q / k group's REP copies (16 B each), or a v group's fp32 values
//   du   [kTB + 3 rows][CW] fp32         du of those times
// The next window's copies are in flight while this window is computed; the thread that copies a cotangent slot
// is the one that reads it, so only its own async-group wait orders those copies.

constexpr int kTB = 32;
constexpr int kStagesB = 2;

__device__ __forceinline__ void cp16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait_all_but() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <typename T>
__host__ __device__ constexpr int slot_bytes(int rep) {
  return rep * 16 > 4 * Geo<T>::G ? rep * 16 : 4 * Geo<T>::G;
}

template <typename T, typename TW, bool DW>
__global__ void __launch_bounds__(kThreads, DW ? 2 : 3) conv_window_bwd(const __grid_constant__ CUtensorMap xmap,
                                                               const TW* __restrict__ w, const T* __restrict__ dq,
                                                               const T* __restrict__ dk, const float* __restrict__ dv,
                                                               T* __restrict__ dx, float* __restrict__ part, int B,
                                                               int Tn, int C, int KD, int DK, int REP, int DV,
                                                               long long per_run) {
  using Gm = Geo<T>;
  constexpr int G = Gm::G, CW = Gm::CW, XROWS = kTB + 6, UROWS = kTB + 3;
  constexpr int XSTAGE = XROWS * 256;
  const int SLOT = slot_bytes<T>(REP);
  const int CSTAGE = UROWS * Gm::NG * SLOT;
  extern __shared__ __align__(128) unsigned char sm[];
  float* du = reinterpret_cast<float*>(sm + kStagesB * XSTAGE);                 // [UROWS][CW]
  unsigned char* cot = sm + kStagesB * XSTAGE + UROWS * CW * 4;                  // [kStagesB][UROWS][NG][SLOT]
  uint64_t* full = reinterpret_cast<uint64_t*>(cot + kStagesB * CSTAGE);
  const int tid = threadIdx.x, grp = tid % Gm::NG, row0 = tid / Gm::NG;
  const int c0 = blockIdx.x * CW, c = c0 + grp * G;
  Run run;
  run.ntile = (Tn + kTB - 1) / kTB;
  run.first = (long long)blockIdx.y * per_run;
  const long long total = (long long)B * run.ntile;
  run.last = run.first + per_run < total ? run.first + per_run : total;
  const long long n = run.last - run.first;
  if (tid == 0) {
    for (int k = 0; k < kStagesB; ++k) mbar_init(full + k, 1);
    gd::fence_mbar_init();
  }
  __syncthreads();
  auto window_of = [&](long long i, int& b, int& t0) {
    const long long q = run.first + i;
    b = (int)(q / run.ntile);
    t0 = (int)(q % run.ntile) * kTB;
  };
  auto issue_x = [&](long long i) {
    int b, t0;
    window_of(i, b, t0);
    const int k = (int)(i % kStagesB);
    mbar_arrive_expect_tx(full + k, (uint32_t)XSTAGE);
    tma_x(sm + k * XSTAGE, &xmap, c0, t0 - 3, b, full + k);
  };
  const Dest d = dest_of(c, C, KD, DK, REP, DV);
  const T* dqk = d.kind == 0 ? dq : (d.kind == 1 ? dk : nullptr);
  // this thread's cotangent slots of window i (always one commit group, possibly empty)
  auto issue_cot = [&](long long i) {
    if (i < n && d.kind >= 0 && (d.kind == 2 ? dv != nullptr : dqk != nullptr)) {
      int b, t0;
      window_of(i, b, t0);
      unsigned char* base = cot + (int)(i % kStagesB) * CSTAGE;
      for (int r = row0; r < UROWS; r += Gm::RSTEP) {
        const int t = t0 + r;
        const bool valid = t < Tn;
        const long long tok = (long long)b * Tn + (valid ? t : 0);
        unsigned char* slot = base + (r * Gm::NG + grp) * SLOT;
        if (d.kind == 2) {
          const float* src = dv + tok * d.row_len + d.col;
          for (int e = 0; e < G; e += 4) cp16(slot + e * 4, src + e, valid);
        } else {
          const T* src = dqk + tok * d.row_len + d.col;
          for (int rr = 0; rr < REP; ++rr) cp16(slot + rr * 16, src + (long long)rr * DK, valid);
        }
      }
    }
    cp_commit();
  };
  if (tid == 0)
    for (long long i = 0; i < kStagesB && i < n; ++i) issue_x(i);
  for (int i = 0; i < kStagesB - 1; ++i) issue_cot(i);
  float tap[4][G];
#pragma unroll
  for (int i = 0; i < G; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) tap[j][i] = c + i < C ? weight_at(w + (size_t)(c + i) * 4 + j) : 0.f;
  const bool has_cot = d.kind >= 0 && (d.kind == 2 ? dv != nullptr : dqk != nullptr);
  float wsum[4][G];  // this thread's share of dw for its channels (taps j = 0 .. 3)
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int e = 0; e < G; ++e) wsum[j][e] = 0.f;
  for (long long i = 0; i < n; ++i) {
    // window i + 1's cotangents, into the slots window i - 1 read; then wait for window i's (one group may remain)
    issue_cot(i + kStagesB - 1);
    cp_wait_all_but<kStagesB - 1>();
    const int k = (int)(i % kStagesB);
    const unsigned char* st = sm + k * XSTAGE;
    const bool landed = wait_copy(full + k, (uint32_t)((i / kStagesB) & 1));
    if (!__syncthreads_and(landed)) return;
    int b, t0;
    window_of(i, b, t0);
    const unsigned char* cs = cot + k * CSTAGE;
    // du for times t0 .. t0 + kTB + 2 (zero past the sequence end, past C and for a missing cotangent)
    for (int r = row0; r < UROWS; r += Gm::RSTEP) {
      float g[G];
#pragma unroll
      for (int e = 0; e < G; ++e) g[e] = 0.f;
      if (has_cot) {
        const unsigned char* slot = cs + (r * Gm::NG + grp) * SLOT;
        if (d.kind == 2) {
#pragma unroll
          for (int e = 0; e < G; e += 4) {
            const float4 a = *reinterpret_cast<const float4*>(slot + e * 4);
            g[e] = a.x; g[e + 1] = a.y; g[e + 2] = a.z; g[e + 3] = a.w;
          }
        } else {
          for (int rr = 0; rr < REP; ++rr) {  // the value heads' cotangents, summed in order
            float a[G];
            unpack<T>(*reinterpret_cast<const uint4*>(slot + rr * 16), a);
#pragma unroll
            for (int e = 0; e < G; ++e) g[e] += a[e];
          }
        }
      }
      float xv[4][G];  // staged rows r .. r + 3 = times t - 3 .. t
#pragma unroll
      for (int j = 0; j < 4; ++j) unpack<T>(*reinterpret_cast<const uint4*>(st + (r + j) * 256 + grp * 16), xv[j]);
      float dd[G];
#pragma unroll
      for (int e = 0; e < G; ++e) {
        float u = tap[3][e] * xv[3][e];
        u = fmaf(tap[2][e], xv[2][e], u);
        u = fmaf(tap[1][e], xv[1][e], u);
        u = fmaf(tap[0][e], xv[0][e], u);
        const float sg = sigm(u);
        dd[e] = g[e] * sg * fmaf(u, 1.f - sg, 1.f);
      }
      if (DW && r < kTB && t0 + r < Tn) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int e = 0; e < G; ++e) wsum[j][e] = fmaf(dd[e], xv[j][e], wsum[j][e]);
      }
      float* q = du + r * CW + grp * G;
#pragma unroll
      for (int e = 0; e < G; e += 4) *reinterpret_cast<float4*>(q + e) = make_float4(dd[e], dd[e + 1], dd[e + 2], dd[e + 3]);
    }
    __syncthreads();  // the window's du complete
    // dx for times t0 .. t0 + kTB - 1: du rows r .. r + 3 (times t .. t + 3) against taps 3 .. 0
    if (d.kind >= 0) {
#pragma unroll 2
      for (int r = row0; r < kTB; r += Gm::RSTEP) {
        const int t = t0 + r;
        if (t >= Tn) break;
        float o[G];
#pragma unroll
        for (int e = 0; e < G; ++e) o[e] = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float* q = du + (r + j) * CW + grp * G;
#pragma unroll
          for (int e = 0; e < G; e += 4) {
            const float4 a = *reinterpret_cast<const float4*>(q + e);
            o[e] = fmaf(tap[3 - j][e], a.x, o[e]);
            o[e + 1] = fmaf(tap[3 - j][e + 1], a.y, o[e + 1]);
            o[e + 2] = fmaf(tap[3 - j][e + 2], a.z, o[e + 2]);
            o[e + 3] = fmaf(tap[3 - j][e + 3], a.w, o[e + 3]);
          }
        }
        __stcs(reinterpret_cast<uint4*>(dx + ((long long)b * Tn + t) * C + c), pack<T>(o));
      }
    }
    __syncthreads();  // the x stage and the du tile are free
    if (tid == 0 && i + kStagesB < n) issue_x(i + kStagesB);
  }
  asm volatile("cp.async.wait_all;" ::: "memory");  // no copy of this CTA's left in flight
  if constexpr (DW) {
    // the CTA's sums: thread rows of one channel group added in row order, then partial row blockIdx.y
    float* red = du;  // [RSTEP][CW * 4] over the du tile and the cotangent slots after it (free after the last window)
    static_assert(Gm::RSTEP * CW * 4 * 4 <= UROWS * CW * 4 + kStagesB * UROWS * Gm::NG * 16,
                  "the reduction fits in the du tile and the (smallest) cotangent slots");
#pragma unroll
    for (int e = 0; e < G; ++e)
      *reinterpret_cast<float4*>(red + (size_t)row0 * CW * 4 + (grp * G + e) * 4) =
          make_float4(wsum[0][e], wsum[1][e], wsum[2][e], wsum[3][e]);
    __syncthreads();
    for (int idx = tid; idx < CW * 4; idx += kThreads) {
      const int cc = c0 + idx / 4;
      float s = 0.f;
      for (int rr = 0; rr < Gm::RSTEP; ++rr) s += red[(size_t)rr * CW * 4 + idx];
      if (cc < C) part[((size_t)blockIdx.y * C + cc) * 4 + idx % 4] = s;
    }
  }
}

// dw[k] (k = 4 c + j) = the sum over the P partial rows of element k: 32 consecutive elements a CTA (one per lane, so
// every row's read is one coalesced 128-byte line), thread row y adding rows y, y + 8, ... in order, then the 8 row
// sums added pairwise in a fixed tree (the same bits every run)
template <typename TW>
__global__ void __launch_bounds__(256) conv_dw_total(const float* __restrict__ part, int P, int N, TW* __restrict__ dw) {
  __shared__ float acc[8][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int k = blockIdx.x * 32 + tx;
  float s = 0.f;
  if (k < N)
    for (int p = ty; p < P; p += 8) s += part[(size_t)p * N + k];
  acc[ty][tx] = s;
  __syncthreads();
  for (int h = 4; h > 0; h >>= 1) {
    if (ty < h) acc[ty][tx] += acc[ty + h][tx];
    __syncthreads();
  }
  if (ty == 0 && k < N) {
    const float t = acc[0][tx];
    if constexpr (std::is_same<TW, float>::value) {
      dw[k] = t;
    } else if constexpr (std::is_same<TW, __half>::value) {
      dw[k] = __float2half_rn(t);
    } else {
      dw[k] = __float2bfloat16_rn(t);
    }
  }
}

// ------------------------------------------------------------------------------------------------------------------
// host

template <typename T>
constexpr CUtensorMapDataType tmap_type() {
  return std::is_same<T, float>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                       : (std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                                         : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16);
}

// x [B, T, C] as a 3-D tensor map with a {CW, rows, 1} box; rows outside [0, T) and channels past C read as zeros
template <typename T>
bool x_map(CUtensorMap* m, const void* x, int B, int Tn, int C, int rows) {
  gd::EncodeTiled enc = gd::encode_tiled();
  if (enc == nullptr) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)C, (cuuint64_t)Tn, (cuuint64_t)B};
  const cuuint64_t strides[2] = {(cuuint64_t)C * sizeof(T), (cuuint64_t)Tn * C * sizeof(T)};
  const cuuint32_t box[3] = {(cuuint32_t)Geo<T>::CW, (cuuint32_t)rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, tmap_type<T>(), 3, const_cast<void*>(x), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// windows per CTA run when the weight's gradient is formed: at most kMaxPartials runs (one partial row of dw each)
void runs(long long windows, bool dw, long long& per_run, int& P) {
  const long long want = dw ? kMaxPartials : kMaxGridY;
  per_run = (windows + want - 1) / want;
  if (per_run < 1) per_run = 1;
  P = (int)((windows + per_run - 1) / per_run);
  if (P < 1) P = 1;
}

int status_of(cudaError_t e) { return e == cudaSuccess ? GD_OK : GD_ERR_LAUNCH; }
bool aligned16(const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// The dynamic shared-memory opt-in, once per device, at the largest size any launch of the kernel may ask for (the
// backward's size grows with REP), so that one setting serves every later call, inside a stream capture too.
template <typename K>
cudaError_t smem_opt_in(K kern, bool (&done)[gd::kMaxDevices]) {
  return gd::set_smem_once(kern, 227 * 1024, done);
}

// The grid: channel windows (x) times runs of time windows (y). A run is about kRunWindows windows (measured on the
// B200: many short runs, whose CTAs start while others drain, beat one resident wave of long runs by 15-25 % at
// config 4's size), but the grid is never smaller than one wave of resident CTAs (this kernel's occupancy at this
// shared-memory size times the SM count), which matters for short sequences.
constexpr int kRunWindows = 8;

template <typename K>
void plan_runs(K kern, size_t smem, long long groups, long long windows, long long& per_run, int& P) {
  int dev = 0, sms = 148, per_sm = 1;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem) != cudaSuccess || per_sm < 1) {
    sms = 148;
    per_sm = 1;
  }
  long long want = (long long)sms * per_sm / groups;  // runs a channel window for one wave
  const long long by_len = (windows + kRunWindows - 1) / kRunWindows;
  if (want < by_len) want = by_len;
  if (want < 1) want = 1;
  if (want > kMaxGridY) want = kMaxGridY;
  per_run = (windows + want - 1) / want;
  if (per_run < 1) per_run = 1;
  P = (int)((windows + per_run - 1) / per_run);
  if (P < 1) P = 1;
}

template <typename T, typename TW>
int fwd_t(const void* x, const void* w, void* q, void* k, float* v, int B, int Tn, int C, int KD, int DK, int REP,
          int DV, cudaStream_t st) {
  CUtensorMap m{};
  if (!x_map<T>(&m, x, B, Tn, C, kTT + 3)) return GD_ERR_LAUNCH;
  const long long groups = (C + Geo<T>::CW - 1) / Geo<T>::CW;
  const long long windows = (long long)B * ((Tn + kTT - 1) / kTT);
  const size_t smem = kStagesF * (kTT + 3) * 256 + 8 * kStagesF;
  static bool done[gd::kMaxDevices] = {};
  if (smem_opt_in(conv_window_fwd<T, TW>, done) != cudaSuccess) return GD_ERR_LAUNCH;
  long long per_run;
  int P;
  plan_runs(conv_window_fwd<T, TW>, smem, groups, windows, per_run, P);
  conv_window_fwd<T, TW><<<dim3((unsigned)groups, (unsigned)P), kThreads, smem, st>>>(
      m, static_cast<const TW*>(w), static_cast<T*>(q), static_cast<T*>(k), v, B, Tn, C, KD, DK, REP, DV, per_run);
  return status_of(cudaGetLastError());
}

template <typename T, typename TW>
int bwd_t(const void* x, const void* w, const void* dq, const void* dk, const float* dv, void* dx, void* dw, int B,
          int Tn, int C, int KD, int DK, int REP, int DV, void* ws, cudaStream_t st) {
  CUtensorMap m{};
  if (!x_map<T>(&m, x, B, Tn, C, kTB + 6)) return GD_ERR_LAUNCH;
  const long long groups = (C + Geo<T>::CW - 1) / Geo<T>::CW;
  const long long windows = (long long)B * ((Tn + kTB - 1) / kTB);
  const size_t smem = kStagesB * (kTB + 6) * 256 + (size_t)(kTB + 3) * Geo<T>::CW * 4 +
                      kStagesB * (size_t)(kTB + 3) * Geo<T>::NG * slot_bytes<T>(REP) + 8 * kStagesB;
  if (smem > 227 * 1024) return GD_ERR_SHAPE;
  long long per_run;
  int P;
  float* part = static_cast<float*>(ws);
  if (dw == nullptr) {
    static bool done[gd::kMaxDevices] = {};
    if (smem_opt_in(conv_window_bwd<T, TW, false>, done) != cudaSuccess) return GD_ERR_LAUNCH;
    plan_runs(conv_window_bwd<T, TW, false>, smem, groups, windows, per_run, P);
    const dim3 grid((unsigned)groups, (unsigned)P);
    conv_window_bwd<T, TW, false><<<grid, kThreads, smem, st>>>(
        m, static_cast<const TW*>(w), static_cast<const T*>(dq), static_cast<const T*>(dk), dv, static_cast<T*>(dx),
        nullptr, B, Tn, C, KD, DK, REP, DV, per_run);
    return status_of(cudaGetLastError());
  }
  static bool done[gd::kMaxDevices] = {};
  if (smem_opt_in(conv_window_bwd<T, TW, true>, done) != cudaSuccess) return GD_ERR_LAUNCH;
  runs(windows, dw != nullptr, per_run, P);  // the partial rows gd_conv_workspace_bytes counts
  const dim3 grid((unsigned)groups, (unsigned)P);
  conv_window_bwd<T, TW, true><<<grid, kThreads, smem, st>>>(
      m, static_cast<const TW*>(w), static_cast<const T*>(dq), static_cast<const T*>(dk), dv, static_cast<T*>(dx),
      part, B, Tn, C, KD, DK, REP, DV, per_run);
  if (cudaGetLastError() != cudaSuccess) return GD_ERR_LAUNCH;
  const int N = 4 * C;
  conv_dw_total<TW><<<(N + 31) / 32, 256, 0, st>>>(part, P, N, static_cast<TW*>(dw));
  return status_of(cudaGetLastError());
}

// shapes the kernels take (the reference's supported(), src/macai/layer/_conv.py:178-185, with 16-byte channel
// groups): C = 2 KD + VD, KD a multiple of DK, VD of DV, (KD / DK) REP == VD / DV value heads, and C, KD, DK, DV
// multiples of a group (8 channels at 16 bits, 4 at fp32), so that a group never straddles a head
int check_args(int dtype, int wdtype, int B, int Tn, int C, int KD, int DK, int REP, int DV) {
  if (dtype < GD_FLOAT32 || dtype > GD_BFLOAT16 || wdtype < GD_FLOAT32 || wdtype > GD_BFLOAT16) return GD_ERR_ARG;
  if (wdtype != dtype && wdtype != GD_FLOAT32) return GD_ERR_ARG;
  const int V = dtype == GD_FLOAT32 ? 4 : 8;
  if (B < 0 || Tn < 0 || B > (1 << 20)) return GD_ERR_SHAPE;
  if (KD <= 0 || DK <= 0 || REP <= 0 || DV <= 0) return GD_ERR_SHAPE;
  const int VD = C - 2 * KD;
  if (VD <= 0 || KD % DK != 0 || VD % DV != 0 || (KD / DK) * REP != VD / DV) return GD_ERR_SHAPE;
  if (C % V != 0 || KD % V != 0 || DK % V != 0 || DV % V != 0) return GD_ERR_SHAPE;
  if ((long long)B * Tn * C >= (1ll << 40) || (C + 127) / 128 > kMaxGridY * 2) return GD_ERR_SHAPE;
  return GD_OK;
}

}  // namespace

extern "C" {

size_t gd_conv_workspace_bytes(int B, int T, int C) {
  if (B < 0 || T < 0 || C <= 0) return 0;
  long long per_run;
  int P;
  runs((long long)B * ((T + kTB - 1) / kTB), true, per_run, P);
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
      return wdtype == GD_FLOAT32 ? fwd_t<__nv_bfloat16, float>(x, w, q, k, v, B, T, C, KD, DK, REP, DV, st)
                                  : fwd_t<__nv_bfloat16, __nv_bfloat16>(x, w, q, k, v, B, T, C, KD, DK, REP, DV, st);
    case GD_FLOAT16:
      return wdtype == GD_FLOAT32 ? fwd_t<__half, float>(x, w, q, k, v, B, T, C, KD, DK, REP, DV, st)
                                  : fwd_t<__half, __half>(x, w, q, k, v, B, T, C, KD, DK, REP, DV, st);
    default: return fwd_t<float, float>(x, w, q, k, v, B, T, C, KD, DK, REP, DV, st);
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
                 ? bwd_t<__nv_bfloat16, float>(x, w, dq, dk, dv, dx, dw, B, T, C, KD, DK, REP, DV, workspace, st)
                 : bwd_t<__nv_bfloat16, __nv_bfloat16>(x, w, dq, dk, dv, dx, dw, B, T, C, KD, DK, REP, DV, workspace,
                                                       st);
    case GD_FLOAT16:
      return wdtype == GD_FLOAT32
                 ? bwd_t<__half, float>(x, w, dq, dk, dv, dx, dw, B, T, C, KD, DK, REP, DV, workspace, st)
                 : bwd_t<__half, __half>(x, w, dq, dk, dv, dx, dw, B, T, C, KD, DK, REP, DV, workspace, st);
    default: return bwd_t<float, float>(x, w, dq, dk, dv, dx, dw, B, T, C, KD, DK, REP, DV, workspace, st);
  }
}

}  // extern "C"
