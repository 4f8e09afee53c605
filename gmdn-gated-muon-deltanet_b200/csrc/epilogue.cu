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
// Both kernels stream HBM once.  The wide kernels (below) give a lane 16
// bytes of a row and a warp several consecutive rows a step; the kernels
// described next (one warp per (b, h, t) row, dh / 32 elements per lane) take
// a bf16-in, fp32-out backward.  The input row is read contiguously from
// o (B, H, T, dh) and the
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

// Wide rows: a lane holds 16 bytes of a row of o (VEC = 8 bf16 or 4 fp32
// elements), so a warp step covers RPW = 32 * VEC / dh consecutive rows (2 at
// bf16 dh 128, 4 at dh 64) and the per-row work that does not grow with dh
// (the ring's copy issue and wait, the loop, the shuffle reduction over the
// LPR lanes of a row) is shared by RPW rows.  Each warp walks one contiguous
// run of rows (b, h, t), t advancing by RPW a step, so the output row's
// (b, t, h) place comes from a cursor instead of two divisions a row.  The
// channel arithmetic runs on element pairs (packed fp32x2 instructions).
template <int D, typename TI>
struct WideE {
  static constexpr int VEC = 16 / static_cast<int>(sizeof(TI));
  static constexpr int NP = VEC / 2;
  static constexpr int LPR = D / VEC;   // lanes a row
  static constexpr int RPW = 32 / LPR;  // rows a warp step
  static_assert(LPR >= 1 && LPR <= 32 && 32 % LPR == 0, "row width");
};

template <int LPR>
__device__ __forceinline__ float row_sum(float v) {
#pragma unroll
  for (int o = LPR / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }
__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

// VEC elements of T at p, in one or two 16-byte accesses
template <int VEC, typename T>
__device__ __forceinline__ void store_n(T* p, const float* x) {
  if constexpr (VEC * sizeof(T) <= 16) {
    Vec<VEC, T>::store(p, x);
  } else {
    Vec<VEC / 2, T>::store(p, x);
    Vec<VEC / 2, T>::store(p + VEC / 2, x + VEC / 2);
  }
}
// the lane's row of step m: (bh, t) cursor, advanced by RPW rows a step
struct RowCursor {
  int bh, t, b, h;
  __device__ __forceinline__ void init(int r, int T, int H) {
    bh = r / T;
    t = r - bh * T;
    b = bh / H;
    h = bh - b * H;
  }
  __device__ __forceinline__ void advance(int by, int T, int H) {
    t += by;
    while (t >= T) {   // rare: the run crosses into the next (b, h)
      t -= T;
      if (++h == H) {
        h = 0;
        ++b;
      }
    }
  }
};

template <int D, typename TI, typename TO>
__global__ void __launch_bounds__(kWarps * 32)
head_rmsnorm_fwd_wide_kernel(const TI* __restrict__ o, const float* __restrict__ w,
                             TO* __restrict__ y, int H, int T, float eps, int rows, int per) {
  using W = WideE<D, TI>;
  constexpr int VEC = W::VEC, NP = W::NP, LPR = W::LPR, RPW = W::RPW;
  __shared__ __align__(16) uint8_t ring[kWarps][kRingF][32 * 16];
  const int lane = threadIdx.x & 31, wl = threadIdx.x >> 5;
  const int gw = blockIdx.x * kWarps + wl;
  const int r0 = gw * per;   // this warp's rows: r0 .. r1 - 1 (per is a multiple of RPW)
  if (r0 >= rows) return;
  const int r1 = min(r0 + per, rows);
  const int sub = lane / LPR, col = (lane % LPR) * VEC;
  float2 wr[NP];
#pragma unroll
  for (int c = 0; c < NP; ++c) wr[c] = f2(w[col + 2 * c], w[col + 2 * c + 1]);
  const int n = (r1 - r0 + RPW - 1) / RPW;
  auto slot = [&](int m) { return &ring[wl][m % kRingF][lane * 16]; };
  auto issue = [&](int m) {
    const int r = r0 + m * RPW + sub;
    if (m < n && r < r1) cp_async_cg16(slot(m), o + static_cast<size_t>(r) * D + col);
    cp_async_commit();
  };
#pragma unroll
  for (int m = 0; m < kRingF - 1; ++m) issue(m);
  RowCursor cur;
  cur.init(r0 + sub, T, H);
  for (int m = 0; m < n; ++m) {
    issue(m + kRingF - 1);
    cp_async_wait<kRingF - 1>();
    float x[VEC];
    Vec<VEC, TI>::load(reinterpret_cast<const TI*>(slot(m)), x);
    float2 ss2 = f2(0.f);
#pragma unroll
    for (int c = 0; c < NP; ++c) {
      const float2 xc = f2(x[2 * c], x[2 * c + 1]);
      ss2 = fma2(xc, xc, ss2);
    }
    const float2 rs = f2(rsqrtf(row_sum<LPR>(ss2.x + ss2.y) * (1.f / D) + eps));
    float out[VEC];
#pragma unroll
    for (int c = 0; c < NP; ++c) {
      const float2 v = mul2(mul2(f2(x[2 * c], x[2 * c + 1]), rs), wr[c]);
      out[2 * c] = to_f(from_f<TI>(v.x));   // input dtype
      out[2 * c + 1] = to_f(from_f<TI>(v.y));
    }
    if (r0 + m * RPW + sub < r1)
      store_n<VEC, TO>(y + ((static_cast<size_t>(cur.b) * T + cur.t) * H + cur.h) * D + col, out);
    cur.advance(RPW, T, H);
  }
  cp_async_wait<0>();
}

template <int D, typename TI, typename TO>
__global__ void __launch_bounds__(kWarps * 32)
head_rmsnorm_bwd_wide_kernel(const TI* __restrict__ o, const float* __restrict__ w,
                             const TO* __restrict__ dy, TI* __restrict__ d_o,
                             float* __restrict__ dw, int H, int T, float eps, int rows, int per) {
  using W = WideE<D, TI>;
  constexpr int VEC = W::VEC, NP = W::NP, LPR = W::LPR, RPW = W::RPW;
  constexpr int VBO = VEC * static_cast<int>(sizeof(TO));
  static_assert(VBO == 4 || VBO == 8 || VBO == 16, "cotangent slice");
  __shared__ __align__(16) uint8_t ring_o[kWarps][kRingB][32 * 16];
  __shared__ __align__(16) uint8_t ring_g[kWarps][kRingB][32 * VBO];
  __shared__ float red[kWarps][D];
  const int lane = threadIdx.x & 31, wl = threadIdx.x >> 5;
  const int gw = blockIdx.x * kWarps + wl;
  const int r0 = gw * per;
  const int r1 = min(r0 + per, rows);
  const int sub = lane / LPR, col = (lane % LPR) * VEC;
  float2 wr[NP], acc[NP];
#pragma unroll
  for (int c = 0; c < NP; ++c) {
    wr[c] = f2(w[col + 2 * c], w[col + 2 * c + 1]);
    acc[c] = f2(0.f);
  }
  if (r0 < rows) {
    const int n = (r1 - r0 + RPW - 1) / RPW;
    RowCursor ic;   // the cursor of the row being issued (kRingB - 1 steps ahead)
    ic.init(r0 + sub, T, H);
    auto issue = [&](int m) {
      const int r = r0 + m * RPW + sub;
      if (m < n && r < r1) {
        cp_async_cg16(&ring_o[wl][m % kRingB][lane * 16], o + static_cast<size_t>(r) * D + col);
        cp_async<VBO>(&ring_g[wl][m % kRingB][lane * VBO],
                      dy + ((static_cast<size_t>(ic.b) * T + ic.t) * H + ic.h) * D + col);
      }
      cp_async_commit();
      ic.advance(RPW, T, H);
    };
#pragma unroll
    for (int m = 0; m < kRingB - 1; ++m) issue(m);
    for (int m = 0; m < n; ++m) {
      issue(m + kRingB - 1);
      cp_async_wait<kRingB - 1>();
      float x[VEC], g[VEC];
      Vec<VEC, TI>::load(reinterpret_cast<const TI*>(&ring_o[wl][m % kRingB][lane * 16]), x);
      Vec<VEC, TO>::load(reinterpret_cast<const TO*>(&ring_g[wl][m % kRingB][lane * VBO]), g);
      const bool valid = r0 + m * RPW + sub < r1;
      if (!valid) {   // a row past the run: its slots were never filled
#pragma unroll
        for (int v = 0; v < VEC; ++v) x[v] = g[v] = 0.f;
      }
      float2 ss2 = f2(0.f);
#pragma unroll
      for (int c = 0; c < NP; ++c) {
        const float2 xc = f2(x[2 * c], x[2 * c + 1]);
        ss2 = fma2(xc, xc, ss2);
      }
      const float rs1 = rsqrtf(row_sum<LPR>(ss2.x + ss2.y) * (1.f / D) + eps);
      const float2 rs = f2(rs1);
      float2 xh[NP], gw2[NP], dot2 = f2(0.f);
#pragma unroll
      for (int c = 0; c < NP; ++c) {
        // the cotangent in the input dtype
        const float2 gc = f2(to_f(from_f<TI>(g[2 * c])), to_f(from_f<TI>(g[2 * c + 1])));
        xh[c] = mul2(f2(x[2 * c], x[2 * c + 1]), rs);   // x_hat
        acc[c] = fma2(gc, xh[c], acc[c]);
        gw2[c] = mul2(gc, wr[c]);                      // dL/dx_hat
        dot2 = fma2(xh[c], gw2[c], dot2);
      }
      const float2 dt = f2(row_sum<LPR>(dot2.x + dot2.y) * (1.f / D));
      float dx[VEC];
#pragma unroll
      for (int c = 0; c < NP; ++c) {
        const float2 d = mul2(fma2(xh[c], f2(-dt.x), gw2[c]), rs);
        dx[2 * c] = d.x;
        dx[2 * c + 1] = d.y;
      }
      if (valid) Vec<VEC, TI>::store(d_o + static_cast<size_t>(r0 + m * RPW + sub) * D + col, dx);
    }
    cp_async_wait<0>();
  }
  // dw: the RPW lanes of a column first, then the block's warps
#pragma unroll
  for (int c = 0; c < NP; ++c) {
#pragma unroll
    for (int off = LPR; off < 32; off <<= 1) {
      acc[c].x += __shfl_xor_sync(0xffffffffu, acc[c].x, off);
      acc[c].y += __shfl_xor_sync(0xffffffffu, acc[c].y, off);
    }
  }
  if (sub == 0) {
#pragma unroll
    for (int c = 0; c < NP; ++c) {
      red[wl][col + 2 * c] = acc[c].x;
      red[wl][col + 2 * c + 1] = acc[c].y;
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < D; c += kWarps * 32) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < kWarps; ++k) s += red[k][c];
    atomicAdd(dw + c, s);
  }
}

int wide_grid(int sms) { return sms * 8; }   // 64 warps an SM

int grid_for(long long rows) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long want = (rows + kWarps * kRows - 1) / (kWarps * kRows);
  const long long cap = static_cast<long long>(sms) * 8;   // 64 warps per SM
  return static_cast<int>(want < cap ? (want > 0 ? want : 1) : cap);
}

int sm_count() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

// rows a warp of the wide kernels walks: all rows over the grid's warps, a
// multiple of RPW
int wide_per(long long rows, int grid, int rpw) {
  const long long warps = static_cast<long long>(grid) * kWarps;
  long long per = (rows + warps - 1) / warps;
  per = (per + rpw - 1) / rpw * rpw;
  return static_cast<int>(per > 0 ? per : rpw);
}

template <int VEC, typename TI, typename TO>
cudaError_t fwd_typed(const void* o, const float* w, void* y, int B, int H, int T, float eps,
                      cudaStream_t st) {
  const long long rows = static_cast<long long>(B) * H * T;
  constexpr int D = VEC * 32;
  if constexpr (D / (16 / sizeof(TI)) <= 32) {
    const int grid = wide_grid(sm_count());
    head_rmsnorm_fwd_wide_kernel<D, TI, TO><<<grid, kWarps * 32, 0, st>>>(
        static_cast<const TI*>(o), w, static_cast<TO*>(y), H, T, eps, static_cast<int>(rows),
        wide_per(rows, grid, WideE<D, TI>::RPW));
    return cudaGetLastError();
  }
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
  constexpr int D = VEC * 32;
  if constexpr (D / (16 / sizeof(TI)) <= 32 && sizeof(TO) <= sizeof(TI)) {
    const int grid = wide_grid(sm_count());
    head_rmsnorm_bwd_wide_kernel<D, TI, TO><<<grid, kWarps * 32, 0, st>>>(
        static_cast<const TI*>(o), w, static_cast<const TO*>(dy), static_cast<TI*>(d_o), dw, H,
        T, eps, static_cast<int>(rows), wide_per(rows, grid, WideE<D, TI>::RPW));
    return cudaGetLastError();
  }
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
