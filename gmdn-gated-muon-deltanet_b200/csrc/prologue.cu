// Mixer prologue: train_ablation.py:124-140 after the two projections,
//   qkv = silu(conv(u)),  u = self.qkv(x) (B, T, 3D), conv depthwise causal k=4
//   q, k = L2-normalised per head (F.normalize, eps 1e-12), v as is, (B, H, T, dh)
//   g = sigmoid(self.gates(x)) (B, T, nG*H) -> (nG, B, H, T)
// forward and backward (the projections stay plain GEMMs in the caller).
//
// The conv is causal: out[t] = bias + sum_j w[j] u[t + j - 3] (Conv1d with
// padding 3, truncated to the first T outputs).  Each warp walks one strip
// (b, part, heads) over kTB consecutive time steps with the four-tap window in
// registers, so u is read once and the outputs are written as contiguous
// (b, h) rows.  The wide kernels (below) give a lane 16 or 8 bytes of a row
// and a warp as many heads as that covers; the one-head-a-warp kernels (lanes
// hold dh / 32 channels) take the shapes whose head count does not divide.
// All arithmetic is fp32; outputs are rounded to the I/O dtype.
//
// Backward per strip: dz[t] = ds[t] silu'(z[t]) with ds the cotangent of the
// SiLU output (through the L2 norm for q and k:
// ds = (dq - qn <qn, dq>) / max(|s|, eps), or dq / eps below eps);
// du[t] = sum_j w[j] dz[t + 3 - j]; dw[j] = sum_t dz[t] u[t + j - 3];
// dbias = sum_t dz[t].  A strip recomputes dz for the three steps after it
// (for du) and adds dw and dbias for its own steps only, per lane into fp32
// atomics (one per channel and tap per strip).

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <type_traits>

#include "cp_async.cuh"
#include "fast_path.h"

namespace gmdn {
namespace {

constexpr int kTB = 64;          // time steps per strip
constexpr int kWarpsP = 8;       // warps per block (forward)
constexpr int kWarpsB = 2;       // warps per block (backward: ~160 registers a thread, so
                                 // small blocks let six of them share an SM)
constexpr float kNormEps = 1e-12f;
constexpr int kPF = 2;           // rows a forward warp loads ahead of its arithmetic
constexpr int kPB = 2;           // rows (and cotangent rows) a backward warp loads ahead

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

template <int VEC, typename T>
struct VecP {
  static constexpr int kBytes = VEC * static_cast<int>(sizeof(T));
  using Raw = typename std::conditional<
      kBytes == 16, uint4,
      typename std::conditional<kBytes == 8, uint2,
                                typename std::conditional<kBytes == 4, uint32_t,
                                                          uint16_t>::type>::type>::type;
  __device__ __forceinline__ static void load(const T* p, float* x) {
    union {
      Raw r;
      T e[VEC];
    } u;
    u.r = *reinterpret_cast<const Raw*>(p);
#pragma unroll
    for (int v = 0; v < VEC; ++v) x[v] = to_f(u.e[v]);
  }
  __device__ __forceinline__ static void store(T* p, const float* x) {
    union {
      Raw r;
      T e[VEC];
    } u;
#pragma unroll
    for (int v = 0; v < VEC; ++v) u.e[v] = from_f<T>(x[v]);
    *reinterpret_cast<Raw*>(p) = u.r;
  }
};

__device__ __forceinline__ float wsum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Per-thread prefetch rings (cp_async.cuh): each lane copies its own VEC
// elements of a row (4-16 bytes) into shared memory and reads them back itself.
constexpr int kRingP = 8;    // forward: 8 warps a block, one array
constexpr int kRingB = 8;    // backward: 2 warps a block, u and the cotangent (16 measured the same)
// fast exp and divide: ~1e-6 relative, and these kernels are issue-bound
__device__ __forceinline__ float sigm(float z) { return __fdividef(1.f, 1.f + __expf(-z)); }

struct Strip {
  int b, part, h, t0, t1;
};

__device__ __forceinline__ Strip strip_of(int w, int H, int T) {
  const int ntb = (T + kTB - 1) / kTB;
  Strip s;
  const int tb = w % ntb;
  int rest = w / ntb;
  s.h = rest % H;
  rest /= H;
  s.part = rest % 3;
  s.b = rest / 3;
  s.t0 = tb * kTB;
  s.t1 = min(s.t0 + kTB, T);
  return s;
}

template <int VEC, typename TT>
__global__ void __launch_bounds__(kWarpsP * 32, 4)   // 64 registers: 32 warps an SM
prologue_fwd_kernel(const TT* __restrict__ u, const float* __restrict__ cw,
                    const float* __restrict__ cb, TT* __restrict__ q, TT* __restrict__ k,
                    TT* __restrict__ v, int B, int T, int H, int strips) {
  constexpr int DH = VEC * 32;
  const int w = blockIdx.x * kWarpsP + (threadIdx.x >> 5);
  if (w >= strips) return;
  const int lane = threadIdx.x & 31;
  const Strip s = strip_of(w, H, T);
  const int D = H * DH;
  const int c0 = s.part * D + s.h * DH + lane * VEC;   // channel of this lane's first element
  const size_t row = static_cast<size_t>(3) * D;        // u row stride
  const TT* ub = u + static_cast<size_t>(s.b) * T * row + c0;
  TT* out = (s.part == 0 ? q : s.part == 1 ? k : v) +
            (static_cast<size_t>(s.b) * H + s.h) * static_cast<size_t>(T) * DH + lane * VEC;
  float wt[4][VEC], bias[VEC], win[3][VEC];
#pragma unroll
  for (int e = 0; e < VEC; ++e) {
#pragma unroll
    for (int j = 0; j < 4; ++j) wt[j][e] = cw[(c0 + e) * 4 + j];
    bias[e] = cb[c0 + e];
  }
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int t = s.t0 - 3 + j;
    if (t >= 0) {
      VecP<VEC, TT>::load(ub + static_cast<size_t>(t) * row, win[j]);
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e) win[j][e] = 0.f;
    }
  }
  for (int tb = s.t0; tb < s.t1; tb += kPF) {
    // the rows of kPF steps are loaded before any is used, so a warp keeps
    // kPF loads in flight instead of one
    float xs[kPF][VEC];
#pragma unroll
    for (int i = 0; i < kPF; ++i)
      if (tb + i < s.t1) VecP<VEC, TT>::load(ub + static_cast<size_t>(tb + i) * row, xs[i]);
#pragma unroll
    for (int i = 0; i < kPF; ++i) {
    const int t = tb + i;
    if (t >= s.t1) break;
    const float* x = xs[i];
    float o[VEC];
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const float z = bias[e] + wt[0][e] * win[0][e] + wt[1][e] * win[1][e] +
                      wt[2][e] * win[2][e] + wt[3][e] * x[e];
      o[e] = z * sigm(z);
      ss = fmaf(o[e], o[e], ss);
      win[0][e] = win[1][e];
      win[1][e] = win[2][e];
      win[2][e] = x[e];
    }
    if (s.part < 2) {
      const float inv = 1.f / fmaxf(sqrtf(wsum(ss)), kNormEps);
#pragma unroll
      for (int e = 0; e < VEC; ++e) o[e] *= inv;
    }
    VecP<VEC, TT>::store(out + static_cast<size_t>(t) * DH, o);
    }
  }
}

// dz at step t (zero outside [0, T)): recomputes z from the window
// (u[t-3], u[t-2], u[t-1] in win, u[t] in x) and reads the cotangent of the
// strip's output at t.
template <int VEC>
__device__ __forceinline__ void dz_at(int t, int T, int part, const float (&win)[3][VEC],
                                      const float* x, const float (&wt)[4][VEC],
                                      const float* bias, const float* gin, float* dz) {
  if (t >= T) {
#pragma unroll
    for (int e = 0; e < VEC; ++e) dz[e] = 0.f;
    return;
  }
  float z[VEC], sg[VEC], sv[VEC], g[VEC];
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < VEC; ++e) {
    z[e] = bias[e] + wt[0][e] * win[0][e] + wt[1][e] * win[1][e] + wt[2][e] * win[2][e] +
           wt[3][e] * x[e];
    sg[e] = sigm(z[e]);
    sv[e] = z[e] * sg[e];
    ss = fmaf(sv[e], sv[e], ss);
  }
#pragma unroll
  for (int e = 0; e < VEC; ++e) g[e] = gin[e];
  if (part < 2) {
    const float nrm = sqrtf(wsum(ss));
    if (nrm > kNormEps) {
      const float inv = 1.f / nrm;
      float dot = 0.f;
#pragma unroll
      for (int e = 0; e < VEC; ++e) dot = fmaf(sv[e] * inv, g[e], dot);
      dot = wsum(dot);
#pragma unroll
      for (int e = 0; e < VEC; ++e) g[e] = (g[e] - sv[e] * inv * dot) * inv;
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e) g[e] *= 1.f / kNormEps;
    }
  }
#pragma unroll
  for (int e = 0; e < VEC; ++e) dz[e] = g[e] * sg[e] * (1.f + z[e] * (1.f - sg[e]));
}

template <int VEC, typename TT>
__global__ void __launch_bounds__(kWarpsB * 32)
prologue_bwd_kernel(const TT* __restrict__ u, const float* __restrict__ cw,
                    const float* __restrict__ cb, const TT* __restrict__ dq,
                    const TT* __restrict__ dk, const TT* __restrict__ dv, TT* __restrict__ du,
                    float* __restrict__ dcw, float* __restrict__ dcb, int B, int T, int H,
                    int strips) {
  constexpr int DH = VEC * 32;
  const int w = blockIdx.x * kWarpsB + (threadIdx.x >> 5);
  if (w >= strips) return;
  const int lane = threadIdx.x & 31;
  const Strip s = strip_of(w, H, T);
  const int D = H * DH;
  const int c0 = s.part * D + s.h * DH + lane * VEC;
  const size_t row = static_cast<size_t>(3) * D;
  const TT* ub = u + static_cast<size_t>(s.b) * T * row + c0;
  TT* dub = du + static_cast<size_t>(s.b) * T * row + c0;
  const TT* dout = (s.part == 0 ? dq : s.part == 1 ? dk : dv) +
                   (static_cast<size_t>(s.b) * H + s.h) * static_cast<size_t>(T) * DH + lane * VEC;
  float wt[4][VEC], bias[VEC], win[3][VEC], dzw[3][VEC];   // dzw: dz[t-3], dz[t-2], dz[t-1]
  float aw[4][VEC], ab[VEC];
#pragma unroll
  for (int e = 0; e < VEC; ++e) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      wt[j][e] = cw[(c0 + e) * 4 + j];
      aw[j][e] = 0.f;
    }
#pragma unroll
    for (int j = 0; j < 3; ++j) dzw[j][e] = 0.f;   // dz before t0 is never read
    bias[e] = cb[c0 + e];
    ab[e] = 0.f;
  }
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int t = s.t0 - 3 + j;
    if (t >= 0) {
      VecP<VEC, TT>::load(ub + static_cast<size_t>(t) * row, win[j]);
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e) win[j][e] = 0.f;
    }
  }
  // steps t0 .. t1+2: dz[t]; du[t-3] once dz[t-3 .. t] are known (t-3 >= t0)
  const int tend = min(s.t1 + 3, T);   // steps whose dz this strip needs
  for (int tb = s.t0; tb < s.t1 + 3; tb += kPB) {
    float xs[kPB][VEC], gs[kPB][VEC];
#pragma unroll
    for (int i = 0; i < kPB; ++i) {
      const int t = tb + i;
      if (t < tend) {
        VecP<VEC, TT>::load(ub + static_cast<size_t>(t) * row, xs[i]);
        VecP<VEC, TT>::load(dout + static_cast<size_t>(t) * DH, gs[i]);
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) xs[i][e] = gs[i][e] = 0.f;
      }
    }
#pragma unroll
    for (int i = 0; i < kPB; ++i) {
    const int t = tb + i;
    if (t >= s.t1 + 3) break;
    const float* x = xs[i];
    float dz[VEC];
    dz_at<VEC>(t, T, s.part, win, x, wt, bias, gs[i], dz);
    if (t < s.t1) {   // this strip's own steps: weight and bias gradients
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        aw[0][e] = fmaf(dz[e], win[0][e], aw[0][e]);
        aw[1][e] = fmaf(dz[e], win[1][e], aw[1][e]);
        aw[2][e] = fmaf(dz[e], win[2][e], aw[2][e]);
        aw[3][e] = fmaf(dz[e], x[e], aw[3][e]);
        ab[e] += dz[e];
      }
    }
    const int tp = t - 3;   // du[tp] = w0 dz[tp+3] + w1 dz[tp+2] + w2 dz[tp+1] + w3 dz[tp]
    if (tp >= s.t0) {
      float g[VEC];
#pragma unroll
      for (int e = 0; e < VEC; ++e)
        g[e] = wt[0][e] * dz[e] + wt[1][e] * dzw[2][e] + wt[2][e] * dzw[1][e] +
               wt[3][e] * dzw[0][e];
      VecP<VEC, TT>::store(dub + static_cast<size_t>(tp) * row, g);
    }
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      win[0][e] = win[1][e];
      win[1][e] = win[2][e];
      win[2][e] = x[e];
      dzw[0][e] = dzw[1][e];
      dzw[1][e] = dzw[2][e];
      dzw[2][e] = dz[e];
    }
    }
  }
#pragma unroll
  for (int e = 0; e < VEC; ++e) {
#pragma unroll
    for (int j = 0; j < 4; ++j) atomicAdd(dcw + (c0 + e) * 4 + j, aw[j][e]);
    atomicAdd(dcb + c0 + e, ab[e]);
  }
}

// The same strip walks with the rows of u (and of the output cotangent) coming
// through a per-lane cp.async ring (kRingP / kRingB rows deep) instead of
// loads kPF / kPB rows ahead into registers: a warp keeps 8 rows in flight at
// the register cost of none (the backward dropped from ~141 registers and 12
// warps an SM to 124 and 16, and from 1.03 to 0.60 ms at config-1 size; the
// forward from 0.36 to 0.29 ms).  Used where a lane holds at least 4 bytes of
// a row (VEC * sizeof(TT) >= 4: every head dim but bf16 dh 32).
template <int VEC, typename TT>
__global__ void __launch_bounds__(kWarpsP * 32, 4)
prologue_fwd_ring_kernel(const TT* __restrict__ u, const float* __restrict__ cw,
                         const float* __restrict__ cb, TT* __restrict__ q, TT* __restrict__ k,
                         TT* __restrict__ v, int B, int T, int H, int strips) {
  constexpr int DH = VEC * 32;
  constexpr int VB = VEC * static_cast<int>(sizeof(TT));
  static_assert(VB == 4 || VB == 8 || VB == 16, "cp.async size");
  __shared__ __align__(16) uint8_t ring[kWarpsP][kRingP][32 * VB];
  const int wl = threadIdx.x >> 5;
  const int w = blockIdx.x * kWarpsP + wl;
  if (w >= strips) return;
  const int lane = threadIdx.x & 31;
  const Strip s = strip_of(w, H, T);
  const int D = H * DH;
  const int c0 = s.part * D + s.h * DH + lane * VEC;
  const size_t row = static_cast<size_t>(3) * D;
  const TT* ub = u + static_cast<size_t>(s.b) * T * row + c0;
  TT* out = (s.part == 0 ? q : s.part == 1 ? k : v) +
            (static_cast<size_t>(s.b) * H + s.h) * static_cast<size_t>(T) * DH + lane * VEC;
  float wt[4][VEC], bias[VEC], win[3][VEC];
#pragma unroll
  for (int e = 0; e < VEC; ++e) {
#pragma unroll
    for (int j = 0; j < 4; ++j) wt[j][e] = cw[(c0 + e) * 4 + j];
#pragma unroll
    for (int j = 0; j < 3; ++j) win[j][e] = 0.f;
    bias[e] = cb[c0 + e];
  }
  // steps t0 - 3 .. t1 - 1 through the ring: the first three fill the window
  const int first = s.t0 - 3, n = s.t1 - first;
  auto slot = [&](int i) { return &ring[wl][i % kRingP][lane * VB]; };
  auto issue = [&](int i) {
    const int t = first + i;
    if (i < n && t >= 0) cp_async<VB>(slot(i), ub + static_cast<size_t>(t) * row);
    cp_async_commit();
  };
#pragma unroll
  for (int i = 0; i < kRingP - 1; ++i) issue(i);
  for (int i = 0; i < n; ++i) {
    issue(i + kRingP - 1);   // refills the slot read in step i - 1
    cp_async_wait<kRingP - 1>();
    const int t = first + i;
    float x[VEC];
    if (t >= 0) {
      VecP<VEC, TT>::load(reinterpret_cast<const TT*>(slot(i)), x);
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e) x[e] = 0.f;
    }
    if (i < 3) {   // fill the window (shifted, so that no index is dynamic)
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        win[0][e] = win[1][e];
        win[1][e] = win[2][e];
        win[2][e] = x[e];
      }
      continue;
    }
    float o[VEC];
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const float z = bias[e] + wt[0][e] * win[0][e] + wt[1][e] * win[1][e] +
                      wt[2][e] * win[2][e] + wt[3][e] * x[e];
      o[e] = z * sigm(z);
      ss = fmaf(o[e], o[e], ss);
      win[0][e] = win[1][e];
      win[1][e] = win[2][e];
      win[2][e] = x[e];
    }
    if (s.part < 2) {
      const float inv = 1.f / fmaxf(sqrtf(wsum(ss)), kNormEps);
#pragma unroll
      for (int e = 0; e < VEC; ++e) o[e] *= inv;
    }
    VecP<VEC, TT>::store(out + static_cast<size_t>(t) * DH, o);
  }
  cp_async_wait<0>();
}

template <int VEC, typename TT>
__global__ void __launch_bounds__(kWarpsB * 32)
prologue_bwd_ring_kernel(const TT* __restrict__ u, const float* __restrict__ cw,
                         const float* __restrict__ cb, const TT* __restrict__ dq,
                         const TT* __restrict__ dk, const TT* __restrict__ dv, TT* __restrict__ du,
                         float* __restrict__ dcw, float* __restrict__ dcb, int B, int T, int H,
                         int strips) {
  constexpr int DH = VEC * 32;
  constexpr int VB = VEC * static_cast<int>(sizeof(TT));
  static_assert(VB == 4 || VB == 8 || VB == 16, "cp.async size");
  __shared__ __align__(16) uint8_t ring[kWarpsB][kRingB][2][32 * VB];
  const int wl = threadIdx.x >> 5;
  const int w = blockIdx.x * kWarpsB + wl;
  if (w >= strips) return;
  const int lane = threadIdx.x & 31;
  const Strip s = strip_of(w, H, T);
  const int D = H * DH;
  const int c0 = s.part * D + s.h * DH + lane * VEC;
  const size_t row = static_cast<size_t>(3) * D;
  const TT* ub = u + static_cast<size_t>(s.b) * T * row + c0;
  TT* dub = du + static_cast<size_t>(s.b) * T * row + c0;
  const TT* dout = (s.part == 0 ? dq : s.part == 1 ? dk : dv) +
                   (static_cast<size_t>(s.b) * H + s.h) * static_cast<size_t>(T) * DH + lane * VEC;
  float wt[4][VEC], bias[VEC], win[3][VEC], dzw[3][VEC];   // dzw: dz[t-3], dz[t-2], dz[t-1]
  float aw[4][VEC], ab[VEC];
#pragma unroll
  for (int e = 0; e < VEC; ++e) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      wt[j][e] = cw[(c0 + e) * 4 + j];
      aw[j][e] = 0.f;
    }
#pragma unroll
    for (int j = 0; j < 3; ++j) dzw[j][e] = win[j][e] = 0.f;   // dz before t0 is never read
    bias[e] = cb[c0 + e];
    ab[e] = 0.f;
  }
  // steps t0 - 3 .. t1 + 2: u through the ring from t0 - 3 (the window), the
  // cotangent from t0; dz[t] for t >= t0, du[t-3] once dz[t-3 .. t] are known
  const int first = s.t0 - 3, n = s.t1 + 3 - first;
  const int tend = min(s.t1 + 3, T);   // steps whose dz this strip needs
  auto slot = [&](int i, int a) { return &ring[wl][i % kRingB][a][lane * VB]; };
  auto issue = [&](int i) {
    const int t = first + i;
    if (i < n && t >= 0 && t < tend) {
      cp_async<VB>(slot(i, 0), ub + static_cast<size_t>(t) * row);
      if (t >= s.t0) cp_async<VB>(slot(i, 1), dout + static_cast<size_t>(t) * DH);
    }
    cp_async_commit();
  };
#pragma unroll
  for (int i = 0; i < kRingB - 1; ++i) issue(i);
  for (int i = 0; i < n; ++i) {
    issue(i + kRingB - 1);   // refills the slot read in step i - 1
    cp_async_wait<kRingB - 1>();
    const int t = first + i;
    float x[VEC], gs[VEC];
    if (t >= 0 && t < tend) {
      VecP<VEC, TT>::load(reinterpret_cast<const TT*>(slot(i, 0)), x);
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e) x[e] = 0.f;
    }
    if (i < 3) {   // fill the window (shifted, so that no index is dynamic)
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        win[0][e] = win[1][e];
        win[1][e] = win[2][e];
        win[2][e] = x[e];
      }
      continue;
    }
    if (t < tend) {
      VecP<VEC, TT>::load(reinterpret_cast<const TT*>(slot(i, 1)), gs);
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e) gs[e] = 0.f;
    }
    float dz[VEC];
    dz_at<VEC>(t, T, s.part, win, x, wt, bias, gs, dz);
    if (t < s.t1) {   // this strip's own steps: weight and bias gradients
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        aw[0][e] = fmaf(dz[e], win[0][e], aw[0][e]);
        aw[1][e] = fmaf(dz[e], win[1][e], aw[1][e]);
        aw[2][e] = fmaf(dz[e], win[2][e], aw[2][e]);
        aw[3][e] = fmaf(dz[e], x[e], aw[3][e]);
        ab[e] += dz[e];
      }
    }
    const int tp = t - 3;   // du[tp] = w0 dz[tp+3] + w1 dz[tp+2] + w2 dz[tp+1] + w3 dz[tp]
    if (tp >= s.t0) {
      float g[VEC];
#pragma unroll
      for (int e = 0; e < VEC; ++e)
        g[e] = wt[0][e] * dz[e] + wt[1][e] * dzw[2][e] + wt[2][e] * dzw[1][e] +
               wt[3][e] * dzw[0][e];
      VecP<VEC, TT>::store(dub + static_cast<size_t>(tp) * row, g);
    }
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      win[0][e] = win[1][e];
      win[1][e] = win[2][e];
      win[2][e] = x[e];
      dzw[0][e] = dzw[1][e];
      dzw[1][e] = dzw[2][e];
      dzw[2][e] = dz[e];
    }
  }
  cp_async_wait<0>();
#pragma unroll
  for (int e = 0; e < VEC; ++e) {
#pragma unroll
    for (int j = 0; j < 4; ++j) atomicAdd(dcw + (c0 + e) * 4 + j, aw[j][e]);
    atomicAdd(dcb + c0 + e, ab[e]);
  }
}

// Wide strips: each lane holds 16 bytes of a row (8 bf16 or 4 fp32 channels),
// so a warp covers HPW = 32 * VEC / DH heads of one part at once (2 at bf16
// dh 128, 4 at dh 64), and the per-row work that does not grow with the
// channels (the ring's copy issue, commit and wait, the loop, the norm's
// shuffle reduction over the LPH lanes of a head) is shared by more channels.
// The channel arithmetic runs on channel pairs with the packed fp32x2 FMA,
// multiply and add of sm_100 (each half rounded exactly as the scalar
// instruction), the sigmoid as 1 / (1 + 2^(-z log2 e)) on the approximate
// exp2 and reciprocal instructions.  The conv window is a 4-slot register
// ring rotated by the unrolled step index (no shifts), its first three rows
// are loaded before the loop, and the norm takes one reciprocal square root:
//   1 / max(|s|, eps) = rsqrt(|s|^2) for |s|^2 > eps^2, else 1 / eps.
// Used where H is a multiple of HPW.
template <int DH, typename TT, int LB>
struct Wide {
  static constexpr int VEC = LB / static_cast<int>(sizeof(TT));
  static constexpr int NP = VEC / 2;     // channel pairs a lane
  static constexpr int LPH = DH / VEC;   // lanes per head
  static constexpr int HPW = 32 / LPH;   // heads per warp
  static_assert(NP >= 1 && LPH >= 1 && LPH <= 32 && 32 % LPH == 0, "head width");
};
// lane bytes: the forward takes 16; the backward holds about twice the
// forward's state a channel, so it takes 8 where a head fits a warp (twice the
// warps an SM at half the channels a lane)
template <int DH, typename TT>
constexpr int kLaneBytesB = (DH / (8 / static_cast<int>(sizeof(TT)))) <= 32 ? 8 : 16;

template <int LPH>
__device__ __forceinline__ float head_sum(float v) {
#pragma unroll
  for (int o = LPH / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float inv_norm(float ss) {
  return ss > kNormEps * kNormEps ? rsqrtf(ss) : 1.f / kNormEps;
}

template <int I>
using Ix = std::integral_constant<int, I>;

__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
constexpr float kLog2e = 1.4426950408889634f;   // log2(e)
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// sigmoid of a channel pair.  fp32 I/O: 1 / (1 + e^-z), e^-z = 2^(-z log2 e)
// (two special-function ops an element, ~1e-6 relative); bf16 I/O:
// (1 + tanh(z / 2)) / 2, one op an element (absolute error ~5e-4, below the
// bf16 rounding of the outputs).
template <typename TT>
__device__ __forceinline__ float2 sigm2(float2 z) {
  if constexpr (std::is_same<TT, float>::value) {
    const float2 t = mul2(z, f2(-kLog2e));
    const float2 d = add2(make_float2(ex2_approx(t.x), ex2_approx(t.y)), f2(1.f));
    return make_float2(rcp_approx(d.x), rcp_approx(d.y));
  } else {
    const float2 h = mul2(z, f2(0.5f));
    return fma2(make_float2(tanh_approx(h.x), tanh_approx(h.y)), f2(0.5f), f2(0.5f));
  }
}

// a lane's 16 bytes of a row as NP channel pairs, and back
template <typename TT, int NP>
__device__ __forceinline__ void load2(const TT* p, float2 (&x)[NP]) {
  float f[2 * NP];
  VecP<2 * NP, TT>::load(p, f);
#pragma unroll
  for (int c = 0; c < NP; ++c) x[c] = make_float2(f[2 * c], f[2 * c + 1]);
}
template <typename TT, int NP>
__device__ __forceinline__ void store2(TT* p, const float2 (&x)[NP]) {
  float f[2 * NP];
#pragma unroll
  for (int c = 0; c < NP; ++c) {
    f[2 * c] = x[c].x;
    f[2 * c + 1] = x[c].y;
  }
  VecP<2 * NP, TT>::store(p, f);
}

template <int DH, typename TT>
__global__ void __launch_bounds__(kWarpsP * 32, 2)
prologue_fwd_wide_kernel(const TT* __restrict__ u, const float* __restrict__ cw,
                         const float* __restrict__ cb, TT* __restrict__ q, TT* __restrict__ k,
                         TT* __restrict__ v, int B, int T, int H, int strips) {
  using W = Wide<DH, TT, 16>;
  constexpr int VEC = W::VEC, NP = W::NP, LPH = W::LPH, HPW = W::HPW;
  __shared__ __align__(16) uint8_t ring[kWarpsP][kRingP][32 * 16];
  const int wl = threadIdx.x >> 5;
  const int w = blockIdx.x * kWarpsP + wl;
  if (w >= strips) return;
  const int lane = threadIdx.x & 31;
  const Strip s = strip_of(w, H / HPW, T);   // s.h: group of HPW heads
  const int D = H * DH;
  const int h = s.h * HPW + lane / LPH;
  const int c0 = s.part * D + s.h * HPW * DH + lane * VEC;
  const size_t row = static_cast<size_t>(3) * D;
  const TT* ub = u + static_cast<size_t>(s.b) * T * row + c0;
  TT* out = (s.part == 0 ? q : s.part == 1 ? k : v) +
            (static_cast<size_t>(s.b) * H + h) * static_cast<size_t>(T) * DH + (lane % LPH) * VEC;
  float2 wt[4][NP], bias[NP], wr[4][NP];
#pragma unroll
  for (int c = 0; c < NP; ++c) {
#pragma unroll
    for (int j = 0; j < 4; ++j)
      wt[j][c] = make_float2(cw[(c0 + 2 * c) * 4 + j], cw[(c0 + 2 * c + 1) * 4 + j]);
    bias[c] = make_float2(cb[c0 + 2 * c], cb[c0 + 2 * c + 1]);
  }
#pragma unroll
  for (int j = 0; j < 3; ++j) {   // u[t0 - 3 .. t0 - 1]
    const int t = s.t0 - 3 + j;
    if (t >= 0) {
      load2<TT, NP>(ub + static_cast<size_t>(t) * row, wr[j]);
    } else {
#pragma unroll
      for (int c = 0; c < NP; ++c) wr[j][c] = f2(0.f);
    }
  }
  const int n = s.t1 - s.t0;
  auto slot = [&](int i) { return &ring[wl][i % kRingP][lane * 16]; };
  auto issue = [&](int i) {
    if (i < n) cp_async_cg16(slot(i), ub + static_cast<size_t>(s.t0 + i) * row);
    cp_async_commit();
  };
#pragma unroll
  for (int i = 0; i < kRingP - 1; ++i) issue(i);
  // step i of the strip, i = R (mod 4): wr[R], wr[R+1], wr[R+2] hold
  // u[t-3], u[t-2], u[t-1]; u[t] goes into wr[R+3] (indices mod 4)
  auto step = [&](int i, auto r) {
    constexpr int R = decltype(r)::value;
    constexpr int A0 = R, A1 = (R + 1) & 3, A2 = (R + 2) & 3, A3 = (R + 3) & 3;
    issue(i + kRingP - 1);   // refills the slot read in step i - 1
    cp_async_wait<kRingP - 1>();
    load2<TT, NP>(reinterpret_cast<const TT*>(slot(i)), wr[A3]);
    float2 o[NP];
    float2 ss2 = f2(0.f);
#pragma unroll
    for (int c = 0; c < NP; ++c) {
      float2 z = fma2(wt[0][c], wr[A0][c], bias[c]);
      z = fma2(wt[1][c], wr[A1][c], z);
      z = fma2(wt[2][c], wr[A2][c], z);
      z = fma2(wt[3][c], wr[A3][c], z);
      o[c] = mul2(z, sigm2<TT>(z));
      ss2 = fma2(o[c], o[c], ss2);
    }
    if (s.part < 2) {
      const float2 inv = f2(inv_norm(head_sum<LPH>(ss2.x + ss2.y)));
#pragma unroll
      for (int c = 0; c < NP; ++c) o[c] = mul2(o[c], inv);
    }
    store2<TT, NP>(out + static_cast<size_t>(s.t0 + i) * DH, o);
  };
  for (int i = 0; i < n; i += 4) {   // n is the same for every lane of the warp
    step(i, Ix<0>{});
    if (i + 1 < n) step(i + 1, Ix<1>{});
    if (i + 2 < n) step(i + 2, Ix<2>{});
    if (i + 3 < n) step(i + 3, Ix<3>{});
  }
  cp_async_wait<0>();
}

template <int DH, typename TT>
__global__ void __launch_bounds__(kWarpsB * 32)
prologue_bwd_wide_kernel(const TT* __restrict__ u, const float* __restrict__ cw,
                         const float* __restrict__ cb, const TT* __restrict__ dq,
                         const TT* __restrict__ dk, const TT* __restrict__ dv, TT* __restrict__ du,
                         float* __restrict__ dcw, float* __restrict__ dcb, int B, int T, int H,
                         int strips) {
  constexpr int LB = kLaneBytesB<DH, TT>;
  using W = Wide<DH, TT, LB>;
  constexpr int VEC = W::VEC, NP = W::NP, LPH = W::LPH, HPW = W::HPW;
  __shared__ __align__(16) uint8_t ring[kWarpsB][kRingB][2][32 * LB];
  const int wl = threadIdx.x >> 5;
  const int w = blockIdx.x * kWarpsB + wl;
  if (w >= strips) return;
  const int lane = threadIdx.x & 31;
  const Strip s = strip_of(w, H / HPW, T);
  const int D = H * DH;
  const int h = s.h * HPW + lane / LPH;
  const int c0 = s.part * D + s.h * HPW * DH + lane * VEC;
  const size_t row = static_cast<size_t>(3) * D;
  const TT* ub = u + static_cast<size_t>(s.b) * T * row + c0;
  TT* dub = du + static_cast<size_t>(s.b) * T * row + c0;
  const TT* dout = (s.part == 0 ? dq : s.part == 1 ? dk : dv) +
                   (static_cast<size_t>(s.b) * H + h) * static_cast<size_t>(T) * DH +
                   (lane % LPH) * VEC;
  // wr: u window, dzr: dz window, both rotated like the forward's
  float2 wt[4][NP], bias[NP], wr[4][NP], dzr[4][NP], aw[4][NP], ab[NP];
#pragma unroll
  for (int c = 0; c < NP; ++c) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      wt[j][c] = make_float2(cw[(c0 + 2 * c) * 4 + j], cw[(c0 + 2 * c + 1) * 4 + j]);
      aw[j][c] = f2(0.f);
      dzr[j][c] = f2(0.f);   // dz before t0 is never read
    }
    bias[c] = make_float2(cb[c0 + 2 * c], cb[c0 + 2 * c + 1]);
    ab[c] = f2(0.f);
  }
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int t = s.t0 - 3 + j;
    if (t >= 0) {
      load2<TT, NP>(ub + static_cast<size_t>(t) * row, wr[j]);
    } else {
#pragma unroll
      for (int c = 0; c < NP; ++c) wr[j][c] = f2(0.f);
    }
  }
  // steps t0 .. t1 + 2: dz[t] for each (zero from T on), du[t - 3] once
  // dz[t - 3 .. t] are known, dw and dbias for the strip's own steps
  const int n = s.t1 + 3 - s.t0;
  const int tend = min(s.t1 + 3, T);   // steps whose u and cotangent rows exist
  auto slot = [&](int i, int a) { return &ring[wl][i % kRingB][a][lane * LB]; };
  auto issue = [&](int i) {
    const int t = s.t0 + i;
    if (i < n && t < tend) {
      cp_async<LB>(slot(i, 0), ub + static_cast<size_t>(t) * row);
      cp_async<LB>(slot(i, 1), dout + static_cast<size_t>(t) * DH);
    }
    cp_async_commit();
  };
#pragma unroll
  for (int i = 0; i < kRingB - 1; ++i) issue(i);
  auto step = [&](int i, auto r) {
    constexpr int R = decltype(r)::value;
    constexpr int A0 = R, A1 = (R + 1) & 3, A2 = (R + 2) & 3, A3 = (R + 3) & 3;
    issue(i + kRingB - 1);
    cp_async_wait<kRingB - 1>();
    const int t = s.t0 + i;
    float2 g[NP];
    if (t < tend) {   // warp-uniform
      load2<TT, NP>(reinterpret_cast<const TT*>(slot(i, 0)), wr[A3]);
      load2<TT, NP>(reinterpret_cast<const TT*>(slot(i, 1)), g);
    } else {
#pragma unroll
      for (int c = 0; c < NP; ++c) wr[A3][c] = g[c] = f2(0.f);
    }
    // dz[t] (zero from T on: t >= tend there)
    float2 z[NP], sg[NP], sv[NP];
    float2 ss2 = f2(0.f), dot2 = f2(0.f);
#pragma unroll
    for (int c = 0; c < NP; ++c) {
      z[c] = fma2(wt[0][c], wr[A0][c], bias[c]);
      z[c] = fma2(wt[1][c], wr[A1][c], z[c]);
      z[c] = fma2(wt[2][c], wr[A2][c], z[c]);
      z[c] = fma2(wt[3][c], wr[A3][c], z[c]);
      sg[c] = sigm2<TT>(z[c]);
      sv[c] = mul2(z[c], sg[c]);
      ss2 = fma2(sv[c], sv[c], ss2);
      dot2 = fma2(sv[c], g[c], dot2);
    }
    if (s.part < 2) {   // warp-uniform; the heads of a warp may differ in the branch
                        // below, so both reductions run before it
      const float ss_h = head_sum<LPH>(ss2.x + ss2.y);
      const float dot = head_sum<LPH>(dot2.x + dot2.y);
      if (ss_h > kNormEps * kNormEps) {
        const float inv = rsqrtf(ss_h);
        const float2 nc = f2(-dot * inv * inv), iv = f2(inv);   // -<s, g> / |s|^2, 1 / |s|
#pragma unroll
        for (int c = 0; c < NP; ++c) g[c] = mul2(fma2(sv[c], nc, g[c]), iv);
      } else {
#pragma unroll
        for (int c = 0; c < NP; ++c) g[c] = mul2(g[c], f2(1.f / kNormEps));
      }
    }
    const bool own = t < s.t1;   // this strip's own steps: weight and bias gradients
#pragma unroll
    for (int c = 0; c < NP; ++c) {
      // silu'(z) = sg (1 + z (1 - sg))
      const float2 dsl = fma2(z[c], fma2(sg[c], f2(-1.f), f2(1.f)), f2(1.f));
      const float2 d = t < tend ? mul2(mul2(g[c], sg[c]), dsl) : f2(0.f);
      dzr[A3][c] = d;
      if (own) {
        aw[0][c] = fma2(d, wr[A0][c], aw[0][c]);
        aw[1][c] = fma2(d, wr[A1][c], aw[1][c]);
        aw[2][c] = fma2(d, wr[A2][c], aw[2][c]);
        aw[3][c] = fma2(d, wr[A3][c], aw[3][c]);
        ab[c] = add2(ab[c], d);
      }
    }
    if (t - 3 >= s.t0) {   // du[t-3] = w0 dz[t] + w1 dz[t-1] + w2 dz[t-2] + w3 dz[t-3]
      float2 o[NP];
#pragma unroll
      for (int c = 0; c < NP; ++c) {
        float2 a = mul2(wt[0][c], dzr[A3][c]);
        a = fma2(wt[1][c], dzr[A2][c], a);
        a = fma2(wt[2][c], dzr[A1][c], a);
        o[c] = fma2(wt[3][c], dzr[A0][c], a);
      }
      store2<TT, NP>(dub + static_cast<size_t>(t - 3) * row, o);
    }
  };
  for (int i = 0; i < n; i += 4) {
    step(i, Ix<0>{});
    if (i + 1 < n) step(i + 1, Ix<1>{});
    if (i + 2 < n) step(i + 2, Ix<2>{});
    if (i + 3 < n) step(i + 3, Ix<3>{});
  }
  cp_async_wait<0>();
#pragma unroll
  for (int c = 0; c < NP; ++c) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      atomicAdd(dcw + (c0 + 2 * c) * 4 + j, aw[j][c].x);
      atomicAdd(dcw + (c0 + 2 * c + 1) * 4 + j, aw[j][c].y);
    }
    atomicAdd(dcb + c0 + 2 * c, ab[c].x);
    atomicAdd(dcb + c0 + 2 * c + 1, ab[c].y);
  }
}

// gates: gl (B, T, nG*H) -> g (nG, B, H, T) = sigmoid; backward dgl = dg s (1 - s).
// One block a (b, tt-step tile): the tile's rows of gl are read whole and
// each gate's tt steps written as one contiguous run (the transposition goes
// through shared memory, so neither side is strided).  tt = 32 (64-byte runs
// at bf16), fewer where nG*H is so large that 48 KB would not hold the tile.
// Each thread has its kGateB loads in flight before it uses them, and splits
// flat indices with a float reciprocal (exact here: the quotients are small
// and the remainder keeps a margin of half a divisor).
constexpr int kGateT = 32;
constexpr int kGateB = 8;   // loads in flight a thread
inline int gate_tile(int GH) {
  return std::max(1, std::min(kGateT, (48 * 1024) / ((GH + 1) * static_cast<int>(sizeof(float)))));
}

__device__ __forceinline__ float sigmoid_ieee(float z) { return 1.f / (1.f + expf(-z)); }
// i / d for 0 <= i < 2^20, d >= 1 (inv = 1 / d)
__device__ __forceinline__ int quot(int i, float inv) {
  return static_cast<int>((static_cast<float>(i) + 0.5f) * inv);
}

template <typename TT>
__global__ void __launch_bounds__(256)
gates_fwd_kernel(const TT* __restrict__ gl, TT* __restrict__ g, int B, int T, int GH, int H,
                 int tt) {
  extern __shared__ float tile[];   // [tt][GH + 1]
  const int ntt = (T + tt - 1) / tt;
  const int b = blockIdx.x / ntt, t0 = (blockIdx.x % ntt) * tt;
  const int nt = min(tt, T - t0);
  const int ld = GH + 1;
  const float ig = 1.f / GH, it = 1.f / tt, ih = 1.f / H;
  const TT* src = gl + (static_cast<size_t>(b) * T + t0) * GH;
  for (int i0 = threadIdx.x; i0 < nt * GH; i0 += kGateB * 256) {
    float x[kGateB];
#pragma unroll
    for (int j = 0; j < kGateB; ++j) {
      const int i = i0 + j * 256;
      x[j] = i < nt * GH ? to_f(src[i]) : 0.f;
    }
#pragma unroll
    for (int j = 0; j < kGateB; ++j) {
      const int i = i0 + j * 256, r = quot(i, ig);
      if (i < nt * GH) tile[r * ld + (i - r * GH)] = sigmoid_ieee(x[j]);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < GH * tt; i += 256) {
    const int c = quot(i, it), r = i - c * tt;
    if (r < nt) {
      const int gi = quot(c, ih), h = c - gi * H;
      g[((static_cast<size_t>(gi) * B + b) * H + h) * T + t0 + r] = from_f<TT>(tile[r * ld + c]);
    }
  }
}

template <typename TT>
__global__ void __launch_bounds__(256)
gates_bwd_kernel(const TT* __restrict__ gl, const TT* __restrict__ dg, TT* __restrict__ dgl,
                 int B, int T, int GH, int H, int tt) {
  extern __shared__ float tile[];   // [tt][GH + 1]
  const int ntt = (T + tt - 1) / tt;
  const int b = blockIdx.x / ntt, t0 = (blockIdx.x % ntt) * tt;
  const int nt = min(tt, T - t0);
  const int ld = GH + 1;
  const float ig = 1.f / GH, it = 1.f / tt, ih = 1.f / H;
  for (int i0 = threadIdx.x; i0 < GH * tt; i0 += kGateB * 256) {
    float x[kGateB];
#pragma unroll
    for (int j = 0; j < kGateB; ++j) {
      const int i = i0 + j * 256, c = quot(i, it), r = i - c * tt, gi = quot(c, ih);
      x[j] = i < GH * tt && r < nt
                 ? to_f(dg[((static_cast<size_t>(gi) * B + b) * H + (c - gi * H)) * T + t0 + r])
                 : 0.f;
    }
#pragma unroll
    for (int j = 0; j < kGateB; ++j) {
      const int i = i0 + j * 256, c = quot(i, it);
      if (i < GH * tt) tile[(i - c * tt) * ld + c] = x[j];
    }
  }
  __syncthreads();
  const size_t base = (static_cast<size_t>(b) * T + t0) * GH;
  for (int i0 = threadIdx.x; i0 < nt * GH; i0 += kGateB * 256) {
    float x[kGateB];
#pragma unroll
    for (int j = 0; j < kGateB; ++j) {
      const int i = i0 + j * 256;
      x[j] = i < nt * GH ? to_f(gl[base + i]) : 0.f;
    }
#pragma unroll
    for (int j = 0; j < kGateB; ++j) {
      const int i = i0 + j * 256, r = quot(i, ig);
      if (i < nt * GH) {
        const float sgm = sigmoid_ieee(x[j]);
        dgl[base + i] = from_f<TT>(tile[r * ld + (i - r * GH)] * sgm * (1.f - sgm));
      }
    }
  }
}

template <int VEC, typename TT>
cudaError_t fwd_t(const void* u, const float* cw, const float* cb, const void* gl, void* q,
                  void* k, void* v, void* g, int B, int T, int H, int nG, cudaStream_t st) {
  constexpr int DH = VEC * 32;
  constexpr int HPW = Wide<DH, TT, 16>::HPW;
  if (H % HPW == 0) {
    const int strips = B * 3 * (H / HPW) * ((T + kTB - 1) / kTB);
    prologue_fwd_wide_kernel<DH, TT><<<(strips + kWarpsP - 1) / kWarpsP, kWarpsP * 32, 0, st>>>(
        static_cast<const TT*>(u), cw, cb, static_cast<TT*>(q), static_cast<TT*>(k),
        static_cast<TT*>(v), B, T, H, strips);
  } else {
  const int strips = B * 3 * H * ((T + kTB - 1) / kTB);
  const int blocks = (strips + kWarpsP - 1) / kWarpsP;
  if constexpr (VEC * sizeof(TT) >= 4)
    prologue_fwd_ring_kernel<VEC, TT><<<blocks, kWarpsP * 32, 0, st>>>(
        static_cast<const TT*>(u), cw, cb, static_cast<TT*>(q), static_cast<TT*>(k),
        static_cast<TT*>(v), B, T, H, strips);
  else
    prologue_fwd_kernel<VEC, TT><<<blocks, kWarpsP * 32, 0, st>>>(
        static_cast<const TT*>(u), cw, cb, static_cast<TT*>(q), static_cast<TT*>(k),
        static_cast<TT*>(v), B, T, H, strips);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int GH = nG * H, tt = gate_tile(GH);
  gates_fwd_kernel<TT><<<B * ((T + tt - 1) / tt), 256, tt * (GH + 1) * sizeof(float), st>>>(
      static_cast<const TT*>(gl), static_cast<TT*>(g), B, T, GH, H, tt);
  return cudaGetLastError();
}

template <int VEC, typename TT>
cudaError_t bwd_t(const void* u, const float* cw, const float* cb, const void* gl,
                  const void* dq, const void* dk, const void* dv, const void* dg, void* du,
                  float* dcw, float* dcb, void* dgl, int B, int T, int H, int nG,
                  cudaStream_t st) {
  const int D = H * VEC * 32;
  cudaError_t e = cudaMemsetAsync(dcw, 0, sizeof(float) * 3 * D * 4, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(dcb, 0, sizeof(float) * 3 * D, st);
  if (e != cudaSuccess) return e;
  constexpr int DH = VEC * 32;
  constexpr int HPW = Wide<DH, TT, kLaneBytesB<DH, TT>>::HPW;
  if (H % HPW == 0) {
    const int strips = B * 3 * (H / HPW) * ((T + kTB - 1) / kTB);
    prologue_bwd_wide_kernel<DH, TT><<<(strips + kWarpsB - 1) / kWarpsB, kWarpsB * 32, 0, st>>>(
        static_cast<const TT*>(u), cw, cb, static_cast<const TT*>(dq), static_cast<const TT*>(dk),
        static_cast<const TT*>(dv), static_cast<TT*>(du), dcw, dcb, B, T, H, strips);
  } else {
  const int strips = B * 3 * H * ((T + kTB - 1) / kTB);
  const int blocks = (strips + kWarpsB - 1) / kWarpsB;
  if constexpr (VEC * sizeof(TT) >= 4)
    prologue_bwd_ring_kernel<VEC, TT><<<blocks, kWarpsB * 32, 0, st>>>(
        static_cast<const TT*>(u), cw, cb, static_cast<const TT*>(dq), static_cast<const TT*>(dk),
        static_cast<const TT*>(dv), static_cast<TT*>(du), dcw, dcb, B, T, H, strips);
  else
    prologue_bwd_kernel<VEC, TT><<<blocks, kWarpsB * 32, 0, st>>>(
        static_cast<const TT*>(u), cw, cb, static_cast<const TT*>(dq), static_cast<const TT*>(dk),
        static_cast<const TT*>(dv), static_cast<TT*>(du), dcw, dcb, B, T, H, strips);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int GH = nG * H, tt = gate_tile(GH);
  gates_bwd_kernel<TT><<<B * ((T + tt - 1) / tt), 256, tt * (GH + 1) * sizeof(float), st>>>(
      static_cast<const TT*>(gl), static_cast<const TT*>(dg), static_cast<TT*>(dgl), B, T, GH, H,
      tt);
  return cudaGetLastError();
}

}  // namespace

cudaError_t mixer_prologue_fwd(const void* u, const float* cw, const float* cb, const void* gl,
                               void* q, void* k, void* v, void* g, int B, int T, int H, int dh,
                               int n_gates, bool io_f32, cudaStream_t st) {
  using bf = __nv_bfloat16;
  switch (dh) {
    case 32: return io_f32 ? fwd_t<1, float>(u, cw, cb, gl, q, k, v, g, B, T, H, n_gates, st)
                           : fwd_t<1, bf>(u, cw, cb, gl, q, k, v, g, B, T, H, n_gates, st);
    case 64: return io_f32 ? fwd_t<2, float>(u, cw, cb, gl, q, k, v, g, B, T, H, n_gates, st)
                           : fwd_t<2, bf>(u, cw, cb, gl, q, k, v, g, B, T, H, n_gates, st);
    case 128: return io_f32 ? fwd_t<4, float>(u, cw, cb, gl, q, k, v, g, B, T, H, n_gates, st)
                            : fwd_t<4, bf>(u, cw, cb, gl, q, k, v, g, B, T, H, n_gates, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t mixer_prologue_bwd(const void* u, const float* cw, const float* cb, const void* gl,
                               const void* dq, const void* dk, const void* dv, const void* dg,
                               void* du, float* dcw, float* dcb, void* dgl, int B, int T, int H,
                               int dh, int n_gates, bool io_f32, cudaStream_t st) {
  using bf = __nv_bfloat16;
#define GMDN_PRO_BWD(V, TT) \
  bwd_t<V, TT>(u, cw, cb, gl, dq, dk, dv, dg, du, dcw, dcb, dgl, B, T, H, n_gates, st)
  switch (dh) {
    case 32: return io_f32 ? GMDN_PRO_BWD(1, float) : GMDN_PRO_BWD(1, bf);
    case 64: return io_f32 ? GMDN_PRO_BWD(2, float) : GMDN_PRO_BWD(2, bf);
    case 128: return io_f32 ? GMDN_PRO_BWD(4, float) : GMDN_PRO_BWD(4, bf);
    default: return cudaErrorInvalidValue;
  }
#undef GMDN_PRO_BWD
}

}  // namespace gmdn
