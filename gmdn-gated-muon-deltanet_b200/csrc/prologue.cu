// Mixer prologue: train_ablation.py:124-140 after the two projections,
//   qkv = silu(conv(u)),  u = self.qkv(x) (B, T, 3D), conv depthwise causal k=4
//   q, k = L2-normalised per head (F.normalize, eps 1e-12), v as is, (B, H, T, dh)
//   g = sigmoid(self.gates(x)) (B, T, nG*H) -> (nG, B, H, T)
// forward and backward (the projections stay plain GEMMs in the caller).
//
// The conv is causal: out[t] = bias + sum_j w[j] u[t + j - 3] (Conv1d with
// padding 3, truncated to the first T outputs).  Each warp walks one strip
// (b, part, head) over kTB consecutive time steps with the four-tap window in
// registers, so u is read once and the outputs are written as contiguous
// (b, h) rows; lanes hold dh / 32 channels.  All arithmetic is fp32; outputs
// are rounded to the I/O dtype.
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

// gates: gl (B, T, nG*H) -> g (nG, B, H, T) = sigmoid; backward dgl = dg s (1 - s)
template <typename TT>
__global__ void gates_fwd_kernel(const TT* __restrict__ gl, TT* __restrict__ g, int B, int T,
                                 int GH, int H, long long n) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const uint32_t iu = static_cast<uint32_t>(i);
    const uint32_t gh = iu % static_cast<uint32_t>(GH);
    const uint32_t bt = iu / static_cast<uint32_t>(GH);
    const uint32_t t = bt % static_cast<uint32_t>(T), b = bt / static_cast<uint32_t>(T);
    const uint32_t gi = gh / static_cast<uint32_t>(H), h = gh % static_cast<uint32_t>(H);
    const float z = to_f(gl[i]);
    g[((static_cast<size_t>(gi) * B + b) * H + h) * T + t] = from_f<TT>(1.f / (1.f + expf(-z)));
  }
}

template <typename TT>
__global__ void gates_bwd_kernel(const TT* __restrict__ gl, const TT* __restrict__ dg,
                                 TT* __restrict__ dgl, int B, int T, int GH, int H, long long n) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const uint32_t iu = static_cast<uint32_t>(i);
    const uint32_t gh = iu % static_cast<uint32_t>(GH);
    const uint32_t bt = iu / static_cast<uint32_t>(GH);
    const uint32_t t = bt % static_cast<uint32_t>(T), b = bt / static_cast<uint32_t>(T);
    const uint32_t gi = gh / static_cast<uint32_t>(H), h = gh % static_cast<uint32_t>(H);
    const float sgm = 1.f / (1.f + expf(-to_f(gl[i])));
    const float d = to_f(dg[((static_cast<size_t>(gi) * B + b) * H + h) * T + t]);
    dgl[i] = from_f<TT>(d * sgm * (1.f - sgm));
  }
}

int sms_x(int k) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms * k;
}

template <int VEC, typename TT>
cudaError_t fwd_t(const void* u, const float* cw, const float* cb, const void* gl, void* q,
                  void* k, void* v, void* g, int B, int T, int H, int nG, cudaStream_t st) {
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
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const long long n = static_cast<long long>(B) * T * nG * H;
  gates_fwd_kernel<TT><<<sms_x(4), 256, 0, st>>>(static_cast<const TT*>(gl), static_cast<TT*>(g),
                                                B, T, nG * H, H, n);
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
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const long long n = static_cast<long long>(B) * T * nG * H;
  gates_bwd_kernel<TT><<<sms_x(4), 256, 0, st>>>(static_cast<const TT*>(gl),
                                                static_cast<const TT*>(dg), static_cast<TT*>(dgl),
                                                B, T, nG * H, H, n);
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
