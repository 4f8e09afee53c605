// Exact-fp32 mixer-core kernels (phases 1 and 3 around the state scan).
//
// One CTA of 256 threads per (batch, head, chunk).  All products are fp32
// FMAs on CUDA cores (tile_mm of common.cuh) from bf16 or fp32 activations.
//
//   chunk_prep        Kw = k^T diag(w) k, Uv = v^T diag(w) k, chunk gate products
//                     (train_ablation.py:150-158, 164-165, 169-175)
//   chunk_out         A = tril(q k^T) * beta_col, Qt = q - A k, o = Qt S^T + A v
//                     (train_ablation.py:161-163, 166-167, 184-187)
//   chunk_state_grad  gS_i = dO_i^T Qt_i, the cotangent phase 3 sends into the scan
//   chunk_token_grad  cotangents of q, k, v and of every gate, from dO, S_i and
//                     the scan's dUv_i, dKw_i and chunk-gate cotangents
//
// The backward formulas are the chain rule of the forward above (derivation in
// the module docstring of the Python op); parity against autograd of the
// reference's forward is what the tests check.

#include "common.cuh"
#include "scan_kernels.h"

namespace gmdn {

namespace {

struct ChunkIdx {
  int bh, ci;
  size_t tok;   // first token row of this chunk in (B*H*T)
  size_t gi;    // (b, h, chunk) index
};

__device__ __forceinline__ ChunkIdx chunk_index(int N, int T, int C) {
  ChunkIdx x;
  x.bh = blockIdx.x / N;
  x.ci = blockIdx.x % N;
  x.tok = static_cast<size_t>(x.bh) * T + static_cast<size_t>(x.ci) * C;
  x.gi = static_cast<size_t>(x.bh) * N + x.ci;
  return x;
}

// Token weights w_s of the chunk gradient (train_ablation.py:151-158).
template <int C>
__device__ __forceinline__ void token_weights(const ChunkArgs& p, size_t tok, float* w) {
  const int s = threadIdx.x;
  if (s < C) {
    float val = 1.f;
    if (p.rule == 0) {
      val = p.beta[tok + s];
    } else if (p.rule == 1) {
      float acc = 0.f;
      for (int u = s + 1; u < C; ++u) acc += logf(fmaxf(p.mu[tok + u], kGateFloor));
      val = expf(acc);
    }
    w[s] = val;
  }
}

template <int C, int DH>
__global__ void __launch_bounds__(kThreads) chunk_prep_kernel(ChunkArgs p) {
  __shared__ float w[C];
  __shared__ float stage[2 * kBK * (DH + 4)];
  const ChunkIdx x = chunk_index(p.N, p.T, C);
  token_weights<C>(p, x.tok, w);
  if (threadIdx.x < 32) {
    float la = 0.f, lb = 0.f, lm = 0.f, ln = 0.f;
    for (int t = threadIdx.x; t < C; t += 32) {
      la += logf(fmaxf(p.alpha[x.tok + t], kGateFloor));
      lb += p.beta[x.tok + t];
      lm += logf(fmaxf(p.mu[x.tok + t], kGateFloor));
      if (p.nu) ln += logf(fmaxf(p.nu[x.tok + t], kGateFloor));
    }
    la = warp_sum(la);
    lb = warp_sum(lb);
    lm = warp_sum(lm);
    ln = warp_sum(ln);
    if (threadIdx.x == 0) {
      p.a_c[x.gi] = expf(la);
      p.b_c[x.gi] = lb / C;
      p.m_c[x.gi] = expf(lm);
      p.n_c[x.gi] = (p.nu && p.rule == 2) ? expf(ln) : 1.f;
    }
  }
  __syncthreads();
  const void* k = p.k;
  const void* v = p.v;
  const bool f32 = p.io_f32;
  const size_t row0 = x.tok * DH;
  constexpr int T = DH / 16;
  float acc[T][T];
  float* Kw = p.Kw + x.gi * DH * DH;
  float* Uv = p.Uv + x.gi * DH * DH;
  // Kw[a][b] = sum_s w_s k[s][a] k[s][b]
  tile_zero<DH, DH>(acc);
  tile_mm<DH, DH, false, false>(
      acc, C, [&](int a, int s) { return w[s] * load_act(k, row0 + s * DH + a, f32); },
      [&](int s, int b) { return load_act(k, row0 + s * DH + b, f32); }, stage);
#pragma unroll
  for (int i = 0; i < T; ++i)
#pragma unroll
    for (int j = 0; j < T; ++j) Kw[tile_row(i, T) * DH + tile_col(j, T)] = acc[i][j];
  // Uv[a][b] = sum_s w_s v[s][a] k[s][b]
  tile_zero<DH, DH>(acc);
  tile_mm<DH, DH, false, false>(
      acc, C, [&](int a, int s) { return w[s] * load_act(v, row0 + s * DH + a, f32); },
      [&](int s, int b) { return load_act(k, row0 + s * DH + b, f32); }, stage);
#pragma unroll
  for (int i = 0; i < T; ++i)
#pragma unroll
    for (int j = 0; j < T; ++j) Uv[tile_row(i, T) * DH + tile_col(j, T)] = acc[i][j];
}

// A (masked, beta-scaled) and Qt of one chunk into shared memory.
template <int C, int DH>
__device__ __forceinline__ void build_A_Qt(const ChunkArgs& p, const ChunkIdx& x, float* A,
                                           float* Qt, float* betaS, float* stage) {
  constexpr int PA = C + 1, PQ = DH + 1;
  const bool f32 = p.io_f32;
  const size_t row0 = x.tok * DH;
  if (threadIdx.x < C) betaS[threadIdx.x] = p.beta[x.tok + threadIdx.x];
  __syncthreads();
  {
    constexpr int TM = C / 16, TN = C / 16;
    float acc[TM][TN];
    tile_zero<C, C>(acc);
    tile_mm<C, C, true, true>(
        acc, DH, [&](int t, int d) { return load_act(p.q, row0 + t * DH + d, f32); },
        [&](int d, int s) { return load_act(p.k, row0 + s * DH + d, f32); }, stage);
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) {
        const int t = tile_row(i, TM), s = tile_col(j, TN);
        A[t * PA + s] = (s <= t) ? acc[i][j] * betaS[s] : 0.f;
      }
  }
  __syncthreads();
  {
    constexpr int TM = C / 16, TN = DH / 16;
    float acc[TM][TN];
    tile_zero<C, DH>(acc);
    tile_mm<C, DH, true, false>(
        acc, C, [&](int t, int s) { return A[t * PA + s]; },
        [&](int s, int d) { return load_act(p.k, row0 + s * DH + d, f32); }, stage);
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) {
        const int t = tile_row(i, TM), d = tile_col(j, TN);
        Qt[t * PQ + d] = load_act(p.q, row0 + t * DH + d, f32) - acc[i][j];
      }
  }
  __syncthreads();
}

template <int C, int DH>
constexpr int out_smem_floats() {
  return C * (C + 1) + C * (DH + 1) + C + 2 * kBK * ((C > DH ? C : DH) + 4);
}

template <int C, int DH>
__global__ void __launch_bounds__(kThreads) chunk_out_kernel(ChunkArgs p) {
  extern __shared__ float smem[];
  constexpr int PA = C + 1, PQ = DH + 1;
  float* A = smem;
  float* Qt = A + C * PA;
  float* betaS = Qt + C * PQ;
  float* stage = betaS + C;
  const ChunkIdx x = chunk_index(p.N, p.T, C);
  build_A_Qt<C, DH>(p, x, A, Qt, betaS, stage);
  const bool f32 = p.io_f32;
  const size_t row0 = x.tok * DH;
  const float* S = p.S + x.gi * DH * DH;
  constexpr int TM = C / 16, TN = DH / 16;
  float acc[TM][TN];
  tile_zero<C, DH>(acc);
  // o = Qt S^T + A v
  tile_mm<C, DH, true, true>(
      acc, DH, [&](int t, int d) { return Qt[t * PQ + d]; },
      [&](int d, int c) { return S[c * DH + d]; }, stage);
  tile_mm<C, DH, true, false>(
      acc, C, [&](int t, int s) { return A[t * PA + s]; },
      [&](int s, int c) { return load_act(p.v, row0 + s * DH + c, f32); }, stage);
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j)
      store_act(p.o, row0 + tile_row(i, TM) * DH + tile_col(j, TN), acc[i][j], f32);
}

template <int C, int DH>
__global__ void __launch_bounds__(kThreads) chunk_state_grad_kernel(ChunkArgs p) {
  extern __shared__ float smem[];
  constexpr int PA = C + 1, PQ = DH + 1;
  float* A = smem;
  float* Qt = A + C * PA;
  float* betaS = Qt + C * PQ;
  float* stage = betaS + C;
  const ChunkIdx x = chunk_index(p.N, p.T, C);
  build_A_Qt<C, DH>(p, x, A, Qt, betaS, stage);
  const bool f32 = p.io_f32;
  const size_t row0 = x.tok * DH;
  constexpr int T = DH / 16;
  float acc[T][T];
  tile_zero<DH, DH>(acc);
  // gS[a][b] = sum_t dO[t][a] Qt[t][b]
  tile_mm<DH, DH, false, false>(
      acc, C, [&](int a, int t) { return load_act(p.dO, row0 + t * DH + a, f32); },
      [&](int t, int b) { return Qt[t * PQ + b]; }, stage);
  float* gS = p.gS + x.gi * DH * DH;
#pragma unroll
  for (int i = 0; i < T; ++i)
#pragma unroll
    for (int j = 0; j < T; ++j) gS[tile_row(i, T) * DH + tile_col(j, T)] = acc[i][j];
}

template <int C, int DH>
constexpr int grad_smem_floats() {
  return 2 * C * (C + 1) + C * (DH + 1) + 4 * C + C * 17 + 2 * kBK * ((C > DH ? C : DH) + 4);
}

template <int C, int DH>
__global__ void __launch_bounds__(kThreads) chunk_token_grad_kernel(ChunkArgs p) {
  extern __shared__ float smem[];
  constexpr int PA = C + 1, PQ = DH + 1;
  float* P = smem;            // tril(q k^T), unscaled
  float* dA = P + C * PA;     // cotangent of A, masked
  float* dQt = dA + C * PA;
  float* betaS = dQt + C * PQ;
  float* w = betaS + C;
  float* dbp = w + C;         // sum_t dA[t][s] P[t][s]
  float* dw = dbp + C;
  float* dwp = dw + C;        // [C][17] partial sums of dw
  float* stage = dwp + C * 17;
  const ChunkIdx x = chunk_index(p.N, p.T, C);
  const bool f32 = p.io_f32;
  const size_t row0 = x.tok * DH;
  const size_t mat0 = x.gi * DH * DH;
  const float* S = p.S + mat0;
  const float* dUv = p.dUv + mat0;
  const float* dKw = p.dKw + mat0;
  if (threadIdx.x < C) betaS[threadIdx.x] = p.beta[x.tok + threadIdx.x];
  token_weights<C>(p, x.tok, w);
  __syncthreads();
  auto q_at = [&](int t, int d) { return load_act(p.q, row0 + t * DH + d, f32); };
  auto k_at = [&](int t, int d) { return load_act(p.k, row0 + t * DH + d, f32); };
  auto v_at = [&](int t, int d) { return load_act(p.v, row0 + t * DH + d, f32); };
  auto g_at = [&](int t, int d) { return load_act(p.dO, row0 + t * DH + d, f32); };
  {
    constexpr int TM = C / 16, TN = C / 16;
    float acc[TM][TN];
    tile_zero<C, C>(acc);
    tile_mm<C, C, true, true>(acc, DH, q_at, [&](int d, int s) { return k_at(s, d); }, stage);
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) {
        const int t = tile_row(i, TM), s = tile_col(j, TN);
        P[t * PA + s] = (s <= t) ? acc[i][j] : 0.f;
      }
  }
  {
    constexpr int TM = C / 16, TN = DH / 16;
    float acc[TM][TN];
    tile_zero<C, DH>(acc);
    // dQt = dO S
    tile_mm<C, DH, true, false>(acc, DH, g_at, [&](int c, int d) { return S[c * DH + d]; },
                                stage);
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) dQt[tile_row(i, TM) * PQ + tile_col(j, TN)] = acc[i][j];
  }
  __syncthreads();
  {
    constexpr int TM = C / 16, TN = C / 16;
    float acc[TM][TN];
    tile_zero<C, C>(acc);
    // dA = dO v^T - dQt k^T (on the causal triangle)
    tile_mm<C, C, true, true>(acc, DH, g_at, [&](int c, int s) { return v_at(s, c); }, stage);
    tile_mm<C, C, true, true>(
        acc, DH, [&](int t, int d) { return -dQt[t * PQ + d]; },
        [&](int d, int s) { return k_at(s, d); }, stage);
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) {
        const int t = tile_row(i, TM), s = tile_col(j, TN);
        dA[t * PA + s] = (s <= t) ? acc[i][j] : 0.f;
      }
  }
  __syncthreads();
  if (threadIdx.x < C) {
    const int s = threadIdx.x;
    float acc = 0.f;
    for (int t = s; t < C; ++t) acc = fmaf(dA[t * PA + s], P[t * PA + s], acc);
    dbp[s] = acc;
  }
  constexpr int TM = C / 16, TN = DH / 16;
  {
    // dq = dQt + (dA * beta_col) k
    float acc[TM][TN];
    tile_zero<C, DH>(acc);
    tile_mm<C, DH, true, false>(
        acc, C, [&](int t, int s) { return dA[t * PA + s] * betaS[s]; }, k_at, stage);
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) {
        const int t = tile_row(i, TM), d = tile_col(j, TN);
        store_act(p.dq, row0 + t * DH + d, dQt[t * PQ + d] + acc[i][j], f32);
      }
  }
  float dwrow[TM];
#pragma unroll
  for (int i = 0; i < TM; ++i) dwrow[i] = 0.f;
  {
    // dv = A^T dO + w_s (k dUv^T)
    float acc1[TM][TN], acc2[TM][TN];
    tile_zero<C, DH>(acc1);
    tile_zero<C, DH>(acc2);
    tile_mm<C, DH, false, false>(
        acc1, C, [&](int s, int t) { return P[t * PA + s] * betaS[s]; }, g_at, stage);
    tile_mm<C, DH, true, true>(acc2, DH, k_at, [&](int b, int c) { return dUv[c * DH + b]; },
                               stage);
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) {
        const int s = tile_row(i, TM), c = tile_col(j, TN);
        store_act(p.dv, row0 + s * DH + c, acc1[i][j] + w[s] * acc2[i][j], f32);
        dwrow[i] = fmaf(v_at(s, c), acc2[i][j], dwrow[i]);
      }
  }
  {
    // dk = -A^T dQt + (dA*beta)^T q + w_s (k dKw + k dKw^T + v dUv)
    float acc1[TM][TN], acc2[TM][TN], acc3[TM][TN];
    tile_zero<C, DH>(acc1);
    tile_zero<C, DH>(acc2);
    tile_zero<C, DH>(acc3);
    tile_mm<C, DH, false, false>(
        acc1, C, [&](int s, int t) { return -P[t * PA + s] * betaS[s]; },
        [&](int t, int d) { return dQt[t * PQ + d]; }, stage);
    tile_mm<C, DH, false, false>(
        acc1, C, [&](int s, int t) { return dA[t * PA + s] * betaS[s]; }, q_at, stage);
    tile_mm<C, DH, true, false>(acc2, DH, k_at, [&](int b, int d) { return dKw[b * DH + d]; },
                                stage);
    tile_mm<C, DH, true, false>(acc2, DH, v_at, [&](int a, int d) { return dUv[a * DH + d]; },
                                stage);
    tile_mm<C, DH, true, true>(acc3, DH, k_at, [&](int b, int d) { return dKw[d * DH + b]; },
                               stage);
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) {
        const int s = tile_row(i, TM), d = tile_col(j, TN);
        store_act(p.dk, row0 + s * DH + d,
                  acc1[i][j] + w[s] * (acc2[i][j] + acc3[i][j]), f32);
        dwrow[i] = fmaf(k_at(s, d), acc3[i][j], dwrow[i]);
      }
  }
  {
    const int tx = threadIdx.x & 15;
#pragma unroll
    for (int i = 0; i < TM; ++i) dwp[tile_row(i, TM) * 17 + tx] = dwrow[i];
  }
  __syncthreads();
  if (threadIdx.x < C) {
    const int s = threadIdx.x;
    float acc = 0.f;
    for (int u = 0; u < 16; ++u) acc += dwp[s * 17 + u];
    dw[s] = acc;
  }
  __syncthreads();
  if (threadIdx.x < C) {
    const int s = threadIdx.x;
    const size_t g = x.tok + s;
    const float da_c = p.da_c[x.gi], db_c = p.db_c[x.gi], dm_c = p.dm_c[x.gi];
    const float al = p.alpha[g];
    p.dalpha[g] = (al >= kGateFloor) ? da_c * p.a_c[x.gi] / fmaxf(al, kGateFloor) : 0.f;
    p.dbeta[g] = dbp[s] + db_c / C + (p.rule == 0 ? dw[s] : 0.f);
    const float mu = p.mu[g];
    float dmu = 0.f;
    if (mu >= kGateFloor) {
      const float muc = fmaxf(mu, kGateFloor);
      dmu = dm_c * p.m_c[x.gi] / muc;
      if (p.rule == 1) {
        float pre = 0.f;
        for (int u = 0; u < s; ++u) pre = fmaf(dw[u], w[u], pre);
        dmu += pre / muc;
      }
    }
    p.dmu[g] = dmu;
    if (p.dnu) {
      float dnu = 0.f;
      if (p.rule == 2 && p.nu) {
        const float nu = p.nu[g];
        if (nu >= kGateFloor) dnu = p.dn_c[x.gi] * p.n_c[x.gi] / fmaxf(nu, kGateFloor);
      }
      p.dnu[g] = dnu;
    }
  }
}

template <class F>
cudaError_t launch_dyn(F kernel, int grid, int smem_bytes, const ChunkArgs& p,
                       cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       smem_bytes);
  if (e != cudaSuccess) return e;
  kernel<<<grid, kThreads, smem_bytes, st>>>(p);
  return cudaGetLastError();
}

template <int C, int DH>
cudaError_t run_prep(const ChunkArgs& p, cudaStream_t st) {
  chunk_prep_kernel<C, DH><<<p.BH * p.N, kThreads, 0, st>>>(p);
  return cudaGetLastError();
}
template <int C, int DH>
cudaError_t run_out(const ChunkArgs& p, cudaStream_t st) {
  return launch_dyn(chunk_out_kernel<C, DH>, p.BH * p.N,
                    out_smem_floats<C, DH>() * (int)sizeof(float), p, st);
}
template <int C, int DH>
cudaError_t run_state_grad(const ChunkArgs& p, cudaStream_t st) {
  return launch_dyn(chunk_state_grad_kernel<C, DH>, p.BH * p.N,
                    out_smem_floats<C, DH>() * (int)sizeof(float), p, st);
}
template <int C, int DH>
cudaError_t run_token_grad(const ChunkArgs& p, cudaStream_t st) {
  return launch_dyn(chunk_token_grad_kernel<C, DH>, p.BH * p.N,
                    grad_smem_floats<C, DH>() * (int)sizeof(float), p, st);
}

#define GMDN_CHUNK_DISPATCH(fn)                                   \
  switch (p.C * 1000 + p.dh) {                                    \
    case 32016: return fn<32, 16>(p, st);                         \
    case 32032: return fn<32, 32>(p, st);                         \
    case 32064: return fn<32, 64>(p, st);                         \
    case 32128: return fn<32, 128>(p, st);                        \
    case 64016: return fn<64, 16>(p, st);                         \
    case 64032: return fn<64, 32>(p, st);                         \
    case 64064: return fn<64, 64>(p, st);                         \
    case 64128: return fn<64, 128>(p, st);                        \
    default: return cudaErrorInvalidValue;                        \
  }

}  // namespace

cudaError_t chunk_prep_ieee(const ChunkArgs& p, cudaStream_t st) { GMDN_CHUNK_DISPATCH(run_prep) }
cudaError_t chunk_out_ieee(const ChunkArgs& p, cudaStream_t st) { GMDN_CHUNK_DISPATCH(run_out) }
cudaError_t chunk_state_grad_ieee(const ChunkArgs& p, cudaStream_t st) {
  GMDN_CHUNK_DISPATCH(run_state_grad)
}
cudaError_t chunk_token_grad_ieee(const ChunkArgs& p, cudaStream_t st) {
  GMDN_CHUNK_DISPATCH(run_token_grad)
}

}  // namespace gmdn
