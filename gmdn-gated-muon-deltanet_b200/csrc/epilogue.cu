// Mixer epilogue: the per-head RMSNorm of train_ablation.py:188-189
// (`self.norm(o).to(x.dtype)` with norm = nn.RMSNorm(dh), then the (B, T, D)
// view the output projection reads), forward and backward.
//
// Semantics follow torch's rms_norm for bf16 / fp32 input (the function the
// reference's nn.RMSNorm calls): the row is upcast to fp32,
// y = x * rsqrt(mean(x^2) + eps) * w with eps = FLT_EPSILON unless given,
// rounded to the input dtype, then converted to the output dtype (the
// `.to(x.dtype)` of the reference).  Backward (the cotangent first rounded to
// the input dtype, as autograd of that conversion does):
//   x_hat = x rstd,  g = dy w,  dx = (g - x_hat <x_hat, g> / dh) rstd,
//   dw = sum over rows of dy x_hat.
//
// Both kernels stream HBM once: one warp per (b, h, t) row, dh / 32 elements
// per lane, the input row read contiguously from o (B, H, T, dh) and the
// output row written contiguously at (b, t, h * dh) of y (B, T, H * dh), so
// the head transpose costs nothing.  dw is reduced per block in shared memory
// and added with one atomic per column per block.  A warp walks rows r, r +
// W, r + 2W, ... (W warps in the grid); where a lane holds at least 4 bytes
// of a row, the rows come through a per-lane cp.async ring (kRingF / kRingB
// rows ahead) instead of two rows loaded ahead into registers.

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <type_traits>

#include "cp_async.cuh"
#include "fast_path.h"

namespace gmdn {
namespace {

constexpr int kWarps = 8;   // warps per block
constexpr int kRows = 2;    // rows a warp has in flight (loads issued before any reduction)
constexpr int kRingF = 8;   // ring depth, forward (one array)
constexpr int kRingB = 4;   // ring depth, backward (o and dy; fp32 at 16 bytes a lane fits 48 KB)

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

// VEC consecutive elements of a row: one vector access per lane.
template <int VEC, typename T>
struct Vec {
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

__device__ __forceinline__ float warp_sum32(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int VEC, typename TI, typename TO>
__global__ void __launch_bounds__(kWarps * 32)
head_rmsnorm_fwd_kernel(const TI* __restrict__ o, const float* __restrict__ w, TO* __restrict__ y,
                        int H, int T, float eps, long long rows) {
  constexpr int D = VEC * 32;
  const int lane = threadIdx.x & 31;
  const long long nw = static_cast<long long>(gridDim.x) * kWarps;
  float wr[VEC];
#pragma unroll
  for (int v = 0; v < VEC; ++v) wr[v] = w[lane * VEC + v];
  for (long long r0 = static_cast<long long>(blockIdx.x) * kWarps + (threadIdx.x >> 5); r0 < rows;
       r0 += nw * kRows) {
    float x[kRows][VEC];
#pragma unroll
    for (int k = 0; k < kRows; ++k) {
      const long long r = r0 + k * nw;
      if (r < rows) Vec<VEC, TI>::load(o + r * D + lane * VEC, x[k]);
    }
#pragma unroll
    for (int k = 0; k < kRows; ++k) {
      const long long r = r0 + k * nw;
      if (r >= rows) break;
      // 32-bit divisions (B*H*T < 2^31 is checked by the caller): 64-bit ones are
      // long software sequences and made this kernel issue-bound
      const uint32_t ru = static_cast<uint32_t>(r);
      const uint32_t bh = ru / static_cast<uint32_t>(T);
      const long long t = ru - bh * static_cast<uint32_t>(T);
      const long long b = bh / static_cast<uint32_t>(H);
      const long long h = bh - static_cast<uint32_t>(b) * static_cast<uint32_t>(H);
      float ss = 0.f;
#pragma unroll
      for (int v = 0; v < VEC; ++v) ss = fmaf(x[k][v], x[k][v], ss);
      const float rs = rsqrtf(warp_sum32(ss) * (1.f / D) + eps);
      float out[VEC];
#pragma unroll
      for (int v = 0; v < VEC; ++v) out[v] = to_f(from_f<TI>(x[k][v] * rs * wr[v]));   // input dtype
      Vec<VEC, TO>::store(y + ((b * T + t) * H + h) * D + lane * VEC, out);
    }
  }
}

template <int VEC, typename TI, typename TO>
__global__ void __launch_bounds__(kWarps * 32)
head_rmsnorm_bwd_kernel(const TI* __restrict__ o, const float* __restrict__ w,
                        const TO* __restrict__ dy, TI* __restrict__ d_o, float* __restrict__ dw,
                        int H, int T, float eps, long long rows) {
  constexpr int D = VEC * 32;
  __shared__ float red[kWarps][D];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long nw = static_cast<long long>(gridDim.x) * kWarps;
  float wr[VEC], acc[VEC];
#pragma unroll
  for (int v = 0; v < VEC; ++v) {
    wr[v] = w[lane * VEC + v];
    acc[v] = 0.f;
  }
  for (long long r0 = static_cast<long long>(blockIdx.x) * kWarps + warp; r0 < rows;
       r0 += nw * kRows) {
    float xs[kRows][VEC], gs[kRows][VEC];
#pragma unroll
    for (int k = 0; k < kRows; ++k) {
      const long long r = r0 + k * nw;
      if (r < rows) {
        const uint32_t ru = static_cast<uint32_t>(r);
        const uint32_t bh = ru / static_cast<uint32_t>(T);
        const long long t = ru - bh * static_cast<uint32_t>(T);
        const long long b = bh / static_cast<uint32_t>(H);
        const long long h = bh - static_cast<uint32_t>(b) * static_cast<uint32_t>(H);
        Vec<VEC, TI>::load(o + r * D + lane * VEC, xs[k]);
        Vec<VEC, TO>::load(dy + ((b * T + t) * H + h) * D + lane * VEC, gs[k]);
      }
    }
#pragma unroll
    for (int k = 0; k < kRows; ++k) {
      const long long r = r0 + k * nw;
      if (r >= rows) break;
      float* x = xs[k];
      float* g = gs[k];
      float ss = 0.f;
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        g[v] = to_f(from_f<TI>(g[v]));   // the cotangent in the input dtype
        ss = fmaf(x[v], x[v], ss);
      }
      const float rs = rsqrtf(warp_sum32(ss) * (1.f / D) + eps);
      float dot = 0.f;
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        x[v] *= rs;                        // x_hat
        acc[v] = fmaf(g[v], x[v], acc[v]);
        g[v] *= wr[v];                     // dL/dx_hat
        dot = fmaf(x[v], g[v], dot);
      }
      dot = warp_sum32(dot) * (1.f / D);
      float dx[VEC];
#pragma unroll
      for (int v = 0; v < VEC; ++v) dx[v] = (g[v] - x[v] * dot) * rs;
      Vec<VEC, TI>::store(d_o + r * D + lane * VEC, dx);
    }
  }
#pragma unroll
  for (int v = 0; v < VEC; ++v) red[warp][lane * VEC + v] = acc[v];
  __syncthreads();
  for (int c = threadIdx.x; c < D; c += kWarps * 32) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < kWarps; ++k) s += red[k][c];
    atomicAdd(dw + c, s);
  }
}

template <int VEC, typename TI, typename TO>
__global__ void __launch_bounds__(kWarps * 32)
head_rmsnorm_fwd_ring_kernel(const TI* __restrict__ o, const float* __restrict__ w,
                             TO* __restrict__ y, int H, int T, float eps, long long rows) {
  constexpr int D = VEC * 32;
  constexpr int VB = VEC * static_cast<int>(sizeof(TI));
  __shared__ __align__(16) uint8_t ring[kWarps][kRingF][32 * VB];
  const int lane = threadIdx.x & 31, wl = threadIdx.x >> 5;
  const long long nw = static_cast<long long>(gridDim.x) * kWarps;
  const long long gw = static_cast<long long>(blockIdx.x) * kWarps + wl;
  const long long nr = rows > gw ? (rows - gw + nw - 1) / nw : 0;   // rows of this warp
  float wr[VEC];
#pragma unroll
  for (int v = 0; v < VEC; ++v) wr[v] = w[lane * VEC + v];
  auto slot = [&](long long m) { return &ring[wl][m % kRingF][lane * VB]; };
  auto issue = [&](long long m) {
    if (m < nr) cp_async<VB>(slot(m), o + (gw + m * nw) * D + lane * VEC);
    cp_async_commit();
  };
#pragma unroll
  for (int m = 0; m < kRingF - 1; ++m) issue(m);
  for (long long m = 0; m < nr; ++m) {
    issue(m + kRingF - 1);   // refills the slot read for row m - 1
    cp_async_wait<kRingF - 1>();
    float x[VEC];
    Vec<VEC, TI>::load(reinterpret_cast<const TI*>(slot(m)), x);
    const long long r = gw + m * nw;
    const uint32_t ru = static_cast<uint32_t>(r);
    const uint32_t bh = ru / static_cast<uint32_t>(T);
    const long long t = ru - bh * static_cast<uint32_t>(T);
    const long long b = bh / static_cast<uint32_t>(H);
    const long long h = bh - static_cast<uint32_t>(b) * static_cast<uint32_t>(H);
    float ss = 0.f;
#pragma unroll
    for (int v = 0; v < VEC; ++v) ss = fmaf(x[v], x[v], ss);
    const float rs = rsqrtf(warp_sum32(ss) * (1.f / D) + eps);
    float out[VEC];
#pragma unroll
    for (int v = 0; v < VEC; ++v) out[v] = to_f(from_f<TI>(x[v] * rs * wr[v]));   // input dtype
    Vec<VEC, TO>::store(y + ((b * T + t) * H + h) * D + lane * VEC, out);
  }
  cp_async_wait<0>();
}

template <int VEC, typename TI, typename TO>
__global__ void __launch_bounds__(kWarps * 32)
head_rmsnorm_bwd_ring_kernel(const TI* __restrict__ o, const float* __restrict__ w,
                             const TO* __restrict__ dy, TI* __restrict__ d_o,
                             float* __restrict__ dw, int H, int T, float eps, long long rows) {
  constexpr int D = VEC * 32;
  constexpr int VBI = VEC * static_cast<int>(sizeof(TI));
  constexpr int VBO = VEC * static_cast<int>(sizeof(TO));
  __shared__ __align__(16) uint8_t ring_o[kWarps][kRingB][32 * VBI];
  __shared__ __align__(16) uint8_t ring_g[kWarps][kRingB][32 * VBO];
  __shared__ float red[kWarps][D];
  const int lane = threadIdx.x & 31, wl = threadIdx.x >> 5;
  const long long nw = static_cast<long long>(gridDim.x) * kWarps;
  const long long gw = static_cast<long long>(blockIdx.x) * kWarps + wl;
  const long long nr = rows > gw ? (rows - gw + nw - 1) / nw : 0;
  float wr[VEC], acc[VEC];
#pragma unroll
  for (int v = 0; v < VEC; ++v) {
    wr[v] = w[lane * VEC + v];
    acc[v] = 0.f;
  }
  auto issue = [&](long long m) {
    if (m < nr) {
      const long long r = gw + m * nw;
      const uint32_t ru = static_cast<uint32_t>(r);
      const uint32_t bh = ru / static_cast<uint32_t>(T);
      const long long t = ru - bh * static_cast<uint32_t>(T);
      const long long b = bh / static_cast<uint32_t>(H);
      const long long h = bh - static_cast<uint32_t>(b) * static_cast<uint32_t>(H);
      cp_async<VBI>(&ring_o[wl][m % kRingB][lane * VBI], o + r * D + lane * VEC);
      cp_async<VBO>(&ring_g[wl][m % kRingB][lane * VBO], dy + ((b * T + t) * H + h) * D + lane * VEC);
    }
    cp_async_commit();
  };
#pragma unroll
  for (int m = 0; m < kRingB - 1; ++m) issue(m);
  for (long long m = 0; m < nr; ++m) {
    issue(m + kRingB - 1);
    cp_async_wait<kRingB - 1>();
    float x[VEC], g[VEC];
    Vec<VEC, TI>::load(reinterpret_cast<const TI*>(&ring_o[wl][m % kRingB][lane * VBI]), x);
    Vec<VEC, TO>::load(reinterpret_cast<const TO*>(&ring_g[wl][m % kRingB][lane * VBO]), g);
    const long long r = gw + m * nw;
    float ss = 0.f;
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
      g[v] = to_f(from_f<TI>(g[v]));   // the cotangent in the input dtype
      ss = fmaf(x[v], x[v], ss);
    }
    const float rs = rsqrtf(warp_sum32(ss) * (1.f / D) + eps);
    float dot = 0.f;
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
      x[v] *= rs;                        // x_hat
      acc[v] = fmaf(g[v], x[v], acc[v]);
      g[v] *= wr[v];                     // dL/dx_hat
      dot = fmaf(x[v], g[v], dot);
    }
    dot = warp_sum32(dot) * (1.f / D);
    float dx[VEC];
#pragma unroll
    for (int v = 0; v < VEC; ++v) dx[v] = (g[v] - x[v] * dot) * rs;
    Vec<VEC, TI>::store(d_o + r * D + lane * VEC, dx);
  }
  cp_async_wait<0>();
#pragma unroll
  for (int v = 0; v < VEC; ++v) red[wl][lane * VEC + v] = acc[v];
  __syncthreads();
  for (int c = threadIdx.x; c < D; c += kWarps * 32) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < kWarps; ++k) s += red[k][c];
    atomicAdd(dw + c, s);
  }
}

int grid_for(long long rows) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long want = (rows + kWarps * kRows - 1) / (kWarps * kRows);
  const long long cap = static_cast<long long>(sms) * 8;   // 64 warps per SM
  return static_cast<int>(want < cap ? (want > 0 ? want : 1) : cap);
}

template <int VEC, typename TI, typename TO>
cudaError_t fwd_typed(const void* o, const float* w, void* y, int B, int H, int T, float eps,
                      cudaStream_t st) {
  const long long rows = static_cast<long long>(B) * H * T;
  if constexpr (VEC * sizeof(TI) >= 4)
    head_rmsnorm_fwd_ring_kernel<VEC, TI, TO><<<grid_for(rows), kWarps * 32, 0, st>>>(
        static_cast<const TI*>(o), w, static_cast<TO*>(y), H, T, eps, rows);
  else
    head_rmsnorm_fwd_kernel<VEC, TI, TO><<<grid_for(rows), kWarps * 32, 0, st>>>(
        static_cast<const TI*>(o), w, static_cast<TO*>(y), H, T, eps, rows);
  return cudaGetLastError();
}

template <int VEC, typename TI, typename TO>
cudaError_t bwd_typed(const void* o, const float* w, const void* dy, void* d_o, float* dw, int B,
                      int H, int T, float eps, cudaStream_t st) {
  const long long rows = static_cast<long long>(B) * H * T;
  if constexpr (VEC * sizeof(TI) >= 4 && VEC * sizeof(TO) >= 4)
    head_rmsnorm_bwd_ring_kernel<VEC, TI, TO><<<grid_for(rows), kWarps * 32, 0, st>>>(
        static_cast<const TI*>(o), w, static_cast<const TO*>(dy), static_cast<TI*>(d_o), dw, H,
        T, eps, rows);
  else
    head_rmsnorm_bwd_kernel<VEC, TI, TO><<<grid_for(rows), kWarps * 32, 0, st>>>(
        static_cast<const TI*>(o), w, static_cast<const TO*>(dy), static_cast<TI*>(d_o), dw, H,
        T, eps, rows);
  return cudaGetLastError();
}

template <int VEC>
cudaError_t fwd_vec(const void* o, const float* w, void* y, int B, int H, int T, float eps,
                    bool in_f32, bool out_f32, cudaStream_t st) {
  using bf = __nv_bfloat16;
  if (in_f32)
    return out_f32 ? fwd_typed<VEC, float, float>(o, w, y, B, H, T, eps, st)
                   : fwd_typed<VEC, float, bf>(o, w, y, B, H, T, eps, st);
  return out_f32 ? fwd_typed<VEC, bf, float>(o, w, y, B, H, T, eps, st)
                 : fwd_typed<VEC, bf, bf>(o, w, y, B, H, T, eps, st);
}

template <int VEC>
cudaError_t bwd_vec(const void* o, const float* w, const void* dy, void* d_o, float* dw, int B,
                    int H, int T, float eps, bool in_f32, bool out_f32, cudaStream_t st) {
  using bf = __nv_bfloat16;
  if (in_f32)
    return out_f32 ? bwd_typed<VEC, float, float>(o, w, dy, d_o, dw, B, H, T, eps, st)
                   : bwd_typed<VEC, float, bf>(o, w, dy, d_o, dw, B, H, T, eps, st);
  return out_f32 ? bwd_typed<VEC, bf, float>(o, w, dy, d_o, dw, B, H, T, eps, st)
                 : bwd_typed<VEC, bf, bf>(o, w, dy, d_o, dw, B, H, T, eps, st);
}

}  // namespace

cudaError_t head_rmsnorm_fwd(const void* o, const float* w, void* y, int B, int H, int T, int dh,
                             float eps, bool in_f32, bool out_f32, cudaStream_t st) {
  switch (dh) {
    case 32: return fwd_vec<1>(o, w, y, B, H, T, eps, in_f32, out_f32, st);
    case 64: return fwd_vec<2>(o, w, y, B, H, T, eps, in_f32, out_f32, st);
    case 128: return fwd_vec<4>(o, w, y, B, H, T, eps, in_f32, out_f32, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t head_rmsnorm_bwd(const void* o, const float* w, const void* dy, void* d_o, float* dw,
                             int B, int H, int T, int dh, float eps, bool in_f32, bool out_f32,
                             cudaStream_t st) {
  cudaError_t e = cudaMemsetAsync(dw, 0, sizeof(float) * dh, st);
  if (e != cudaSuccess) return e;
  switch (dh) {
    case 32: return bwd_vec<1>(o, w, dy, d_o, dw, B, H, T, eps, in_f32, out_f32, st);
    case 64: return bwd_vec<2>(o, w, dy, d_o, dw, B, H, T, eps, in_f32, out_f32, st);
    case 128: return bwd_vec<4>(o, w, dy, d_o, dw, B, H, T, eps, in_f32, out_f32, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace gmdn
