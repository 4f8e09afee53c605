// Shared device helpers for the gmdn B200 kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace gmdn {

// Quintic Newton-Schulz coefficients and epsilons of the reference
// (fast_scan.py:32-34).
constexpr float kNsC0 = 3.4445f;
constexpr float kNsC1 = -4.7750f;
constexpr float kNsC2 = 2.0315f;
constexpr float kEpsNorm = 1e-7f;
constexpr float kEpsAdam = 1e-6f;
constexpr float kGateFloor = 1e-6f;  // clamp_min in train_ablation.py:155,170-175

constexpr int kThreads = 256;  // every CTA of the exact-fp32 path

__device__ __forceinline__ float bf16_to_f32(uint16_t x) {
  return __uint_as_float(static_cast<uint32_t>(x) << 16);
}

// Round-to-nearest-even fp32 -> bf16 (NaN kept quiet).
__device__ __forceinline__ uint16_t f32_to_bf16(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

// Element load / store of an activation tensor that is either bf16 or fp32.
__device__ __forceinline__ float load_act(const void* p, size_t i, bool f32) {
  return f32 ? static_cast<const float*>(p)[i]
             : bf16_to_f32(static_cast<const uint16_t*>(p)[i]);
}
__device__ __forceinline__ void store_act(void* p, size_t i, float v, bool f32) {
  if (f32) static_cast<float*>(p)[i] = v;
  else static_cast<uint16_t*>(p)[i] = f32_to_bf16(v);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Sum over the CTA (kThreads threads); every thread gets the result.
// `red` is 32 floats of shared memory; the call contains two barriers.
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = (lane < kThreads / 32) ? red[lane] : 0.f;
  t = warp_sum(t);
  __syncthreads();
  return t;
}

// ---------------------------------------------------------------------------
// CTA tile GEMM on CUDA cores, exact fp32 FMAs.
//
// acc[TM][TN] += sum_k opA(r, k) * opB(k, c), for an M x N output owned by a
// 16 x 16 grid of threads: thread (ty, tx) holds rows ty*TM + i and columns
// tx*TN + j.  opA / opB are callables returning floats; they are staged
// through shared memory BK rows of k at a time (`stage` must hold
// 2 * BK * (max(M, N) + 4) floats).  A_KFAST / B_KFAST say whether consecutive
// k are contiguous in memory for that operand, which picks the staging order
// that keeps the global loads coalesced.  Ends with a barrier.
// ---------------------------------------------------------------------------
constexpr int kBK = 16;

template <int M, int N, bool A_KFAST, bool B_KFAST, class LA, class LB>
__device__ __forceinline__ void tile_mm(float (&acc)[M / 16][N / 16], int kdim, LA opA,
                                        LB opB, float* stage) {
  constexpr int TM = M / 16, TN = N / 16;
  constexpr int PA = M + 4, PB = N + 4;
  float* As = stage;            // [kBK][PA]
  float* Bs = stage + kBK * PA; // [kBK][PB]
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  for (int k0 = 0; k0 < kdim; k0 += kBK) {
    for (int e = tid; e < kBK * M; e += kThreads) {
      int r, k;
      if (A_KFAST) { k = e % kBK; r = e / kBK; } else { r = e % M; k = e / M; }
      As[k * PA + r] = (k0 + k < kdim) ? opA(r, k0 + k) : 0.f;
    }
    for (int e = tid; e < kBK * N; e += kThreads) {
      int c, k;
      if (B_KFAST) { k = e % kBK; c = e / kBK; } else { c = e % N; k = e / N; }
      Bs[k * PB + c] = (k0 + k < kdim) ? opB(k0 + k, c) : 0.f;
    }
    __syncthreads();
#pragma unroll 4
    for (int k = 0; k < kBK; ++k) {
      float av[TM], bv[TN];
#pragma unroll
      for (int i = 0; i < TM; ++i) av[i] = As[k * PA + ty * TM + i];
#pragma unroll
      for (int j = 0; j < TN; ++j) bv[j] = Bs[k * PB + tx * TN + j];
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
}

template <int M, int N>
__device__ __forceinline__ void tile_zero(float (&acc)[M / 16][N / 16]) {
#pragma unroll
  for (int i = 0; i < M / 16; ++i)
#pragma unroll
    for (int j = 0; j < N / 16; ++j) acc[i][j] = 0.f;
}

__device__ __forceinline__ int tile_row(int i, int TM) { return (threadIdx.x >> 4) * TM + i; }
__device__ __forceinline__ int tile_col(int j, int TN) { return (threadIdx.x & 15) * TN + j; }

}  // namespace gmdn
