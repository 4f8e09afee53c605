// Exact-fp32 (IEEE FMA) state scan, forward and backward, all three rules.
//
// One CTA of 256 threads per (batch, head) walks the N chunks in order
// (forward) or in reverse (backward).  The dh x dh state lives in a per-CTA
// scratch slab of global memory that stays in L2; products go through the
// CUDA-core tile GEMM of common.cuh.  This is the set_precision('ieee') path
// of the reference (fast_scan.py:47-50, 196-199): every product is a true
// fp32 FMA chain, so it meets the 1e-4 bar against the fp32 recurrence.
//
// Math: fast_scan.py:5-15 (recurrence), :72-95 (forward), :134-186 (reverse
// scan), :107-131 (msign VJP).  The backward keeps the NS iterates of the
// current chunk in scratch, so the msign VJP costs O(ns) products instead of
// the reference's O(ns^2) recompute (fast_scan.py:256-259).

#include "common.cuh"
#include "scan_kernels.h"

namespace gmdn {

namespace {

template <int DH>
struct Own {
  static constexpr int T = DH / 16;
  static constexpr size_t MAT = static_cast<size_t>(DH) * DH;
};

#define GMDN_OWN(T_)                                 \
  _Pragma("unroll") for (int i = 0; i < T_; ++i)     \
  _Pragma("unroll") for (int j = 0; j < T_; ++j)

template <int DH>
__global__ void __launch_bounds__(kThreads)
scan_fwd_ieee_kernel(const float* __restrict__ U, const float* __restrict__ K,
                     const float* __restrict__ ga, const float* __restrict__ gb,
                     const float* __restrict__ gm, const float* __restrict__ gn,
                     float* __restrict__ S_out, float* __restrict__ M_hist,
                     float* __restrict__ V_hist, float* __restrict__ scratch, int N,
                     int rule, int ns) {
  constexpr int T = Own<DH>::T;
  constexpr size_t MAT = Own<DH>::MAT;
  __shared__ float stage[2 * kBK * (DH + 4)];
  __shared__ float red[32];
  const int bh = blockIdx.x;
  const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
  float* Ssc = scratch + static_cast<size_t>(bh) * kScanFwdScratchMats * MAT;
  float* Msc = Ssc + MAT;
  float* Vsc = Msc + MAT;
  float* Xsc = Vsc + MAT;
  float* Gsc = Xsc + MAT;
  float* Psc = Gsc + MAT;

  float s[T][T], acc[T][T];
  GMDN_OWN(T) {
    const int idx = (ty * T + i) * DH + tx * T + j;
    s[i][j] = 0.f;
    Ssc[idx] = 0.f;
    Msc[idx] = 0.f;
    Vsc[idx] = 0.f;
  }
  __syncthreads();

  for (int ci = 0; ci < N; ++ci) {
    const size_t base = (static_cast<size_t>(bh) * N + ci) * MAT;
    const float* Ui = U + base;
    const float* Ki = K + base;
    // pre-update state (and moments) for this chunk
    GMDN_OWN(T) {
      const int idx = (ty * T + i) * DH + tx * T + j;
      S_out[base + idx] = s[i][j];
      if (rule != 0) M_hist[base + idx] = Msc[idx];
      if (rule == 2) V_hist[base + idx] = Vsc[idx];
    }
    // G = U - S K
    tile_zero<DH, DH>(acc);
    tile_mm<DH, DH, true, false>(
        acc, DH, [&](int r, int k) { return Ssc[r * DH + k]; },
        [&](int k, int c) { return Ki[k * DH + c]; }, stage);
    const size_t gi = static_cast<size_t>(bh) * N + ci;
    const float a = ga[gi];
    GMDN_OWN(T) {
      const int idx = (ty * T + i) * DH + tx * T + j;
      acc[i][j] = Ui[idx] - acc[i][j];
    }
    if (rule == 0) {
      GMDN_OWN(T) s[i][j] = a * s[i][j] + acc[i][j];
    } else if (rule == 2) {
      const float b = gb[gi], mu = gm[gi], nu = gn[gi];
      GMDN_OWN(T) {
        const int idx = (ty * T + i) * DH + tx * T + j;
        const float g = acc[i][j];
        const float m1 = mu * Msc[idx] + (1.f - mu) * g;
        const float v1 = nu * Vsc[idx] + (1.f - nu) * g * g;
        Msc[idx] = m1;
        Vsc[idx] = v1;
        s[i][j] = a * s[i][j] + b * m1 / (sqrtf(v1) + kEpsAdam);
      }
    } else {
      const float b = gb[gi], mu = gm[gi];
      float sq = 0.f;
      GMDN_OWN(T) {
        const int idx = (ty * T + i) * DH + tx * T + j;
        const float m1 = mu * Msc[idx] + acc[i][j];
        Msc[idx] = m1;
        sq = fmaf(m1, m1, sq);
      }
      const float den = sqrtf(block_sum(sq, red)) + kEpsNorm;
      GMDN_OWN(T) {
        const int idx = (ty * T + i) * DH + tx * T + j;
        Xsc[idx] = Msc[idx] / den;
      }
      __syncthreads();
      for (int st = 0; st < ns; ++st) {
        // Gram = X X^T
        tile_zero<DH, DH>(acc);
        tile_mm<DH, DH, true, true>(
            acc, DH, [&](int r, int k) { return Xsc[r * DH + k]; },
            [&](int k, int c) { return Xsc[c * DH + k]; }, stage);
        GMDN_OWN(T) Gsc[(ty * T + i) * DH + tx * T + j] = acc[i][j];
        __syncthreads();
        // Poly = c1 Gram + c2 Gram^2
        tile_zero<DH, DH>(acc);
        tile_mm<DH, DH, true, false>(
            acc, DH, [&](int r, int k) { return Gsc[r * DH + k]; },
            [&](int k, int c) { return Gsc[k * DH + c]; }, stage);
        GMDN_OWN(T) {
          const int idx = (ty * T + i) * DH + tx * T + j;
          Psc[idx] = kNsC1 * Gsc[idx] + kNsC2 * acc[i][j];
        }
        __syncthreads();
        // X <- c0 X + Poly X
        tile_zero<DH, DH>(acc);
        tile_mm<DH, DH, true, false>(
            acc, DH, [&](int r, int k) { return Psc[r * DH + k]; },
            [&](int k, int c) { return Xsc[k * DH + c]; }, stage);
        GMDN_OWN(T) {
          const int idx = (ty * T + i) * DH + tx * T + j;
          Xsc[idx] = kNsC0 * Xsc[idx] + acc[i][j];
        }
        __syncthreads();
      }
      GMDN_OWN(T) {
        const int idx = (ty * T + i) * DH + tx * T + j;
        s[i][j] = a * s[i][j] + b * Xsc[idx];
      }
    }
    GMDN_OWN(T) Ssc[(ty * T + i) * DH + tx * T + j] = s[i][j];
    __syncthreads();
  }
}

template <int DH>
__global__ void __launch_bounds__(kThreads)
scan_bwd_ieee_kernel(const float* __restrict__ U, const float* __restrict__ K,
                     const float* __restrict__ ga, const float* __restrict__ gb,
                     const float* __restrict__ gm, const float* __restrict__ gn,
                     const float* __restrict__ S_all, const float* __restrict__ M_hist,
                     const float* __restrict__ V_hist, const float* __restrict__ gS,
                     float* __restrict__ dU, float* __restrict__ dK, float* __restrict__ da,
                     float* __restrict__ db, float* __restrict__ dm, float* __restrict__ dn,
                     float* __restrict__ scratch, int N, int rule, int ns) {
  constexpr int T = Own<DH>::T;
  constexpr size_t MAT = Own<DH>::MAT;
  __shared__ float stage[2 * kBK * (DH + 4)];
  __shared__ float red[32];
  const int bh = blockIdx.x;
  const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
  float* Gsc = scratch + static_cast<size_t>(bh) * scan_bwd_scratch_mats(ns) * MAT;
  float* Mb = Gsc + MAT;
  float* Vb = Mb + MAT;
  float* Gb = Vb + MAT;
  float* Mi = Gb + MAT;
  float* Xbar = Mi + MAT;
  float* Bbar = Xbar + MAT;
  float* Gbar = Bbar + MAT;
  float* Gsym = Gbar + MAT;
  float* Xs = Gsym + MAT;              // ns + 1 iterates
  float* Grams = Xs + (ns + 1) * MAT;  // ns
  float* Polys = Grams + ns * MAT;     // ns

  float sb[T][T], acc[T][T];
  GMDN_OWN(T) {
    const int idx = (ty * T + i) * DH + tx * T + j;
    sb[i][j] = 0.f;
    Mb[idx] = 0.f;
    Vb[idx] = 0.f;
  }

  for (int ci = N - 1; ci >= 0; --ci) {
    const size_t base = (static_cast<size_t>(bh) * N + ci) * MAT;
    const size_t gi = static_cast<size_t>(bh) * N + ci;
    const float* Si = S_all + base;
    const float* Ui = U + base;
    const float* Ki = K + base;
    const float a = ga[gi];
    // G = U - S K
    tile_zero<DH, DH>(acc);
    tile_mm<DH, DH, true, false>(
        acc, DH, [&](int r, int k) { return Si[r * DH + k]; },
        [&](int k, int c) { return Ki[k * DH + c]; }, stage);
    float part = 0.f;
    GMDN_OWN(T) {
      const int idx = (ty * T + i) * DH + tx * T + j;
      Gsc[idx] = Ui[idx] - acc[i][j];
      part = fmaf(sb[i][j], Si[idx], part);
    }
    const float da_i = block_sum(part, red);
    float db_i = 0.f, dm_i = 0.f, dn_i = 0.f;
    if (rule == 0) {
      GMDN_OWN(T) Gb[(ty * T + i) * DH + tx * T + j] = sb[i][j];
    } else if (rule == 2) {
      const float b = gb[gi], mu = gm[gi], nu = gn[gi];
      float pb = 0.f, pm = 0.f, pn = 0.f;
      GMDN_OWN(T) {
        const int idx = (ty * T + i) * DH + tx * T + j;
        const float g = Gsc[idx], g2 = g * g;
        const float mp = M_hist[base + idx], vp = V_hist[base + idx];
        const float m1 = mu * mp + (1.f - mu) * g;
        const float v1 = nu * vp + (1.f - nu) * g2;
        const float root = sqrtf(v1);
        const float den = root + kEpsAdam;
        pb = fmaf(sb[i][j], m1 / den, pb);
        const float ub = b * sb[i][j];
        const float mt = Mb[idx] + ub / den;
        const float vt = Vb[idx] - ub * m1 / (den * den) / (2.f * fmaxf(root, 1e-12f));
        pm = fmaf(mt, mp - g, pm);
        pn = fmaf(vt, vp - g2, pn);
        Mb[idx] = mu * mt;
        Vb[idx] = nu * vt;
        Gb[idx] = (1.f - mu) * mt + 2.f * (1.f - nu) * g * vt;
      }
      db_i = block_sum(pb, red);
      dm_i = block_sum(pm, red);
      dn_i = block_sum(pn, red);
    } else {
      const float b = gb[gi], mu = gm[gi];
      float sq = 0.f;
      GMDN_OWN(T) {
        const int idx = (ty * T + i) * DH + tx * T + j;
        const float m1 = mu * M_hist[base + idx] + Gsc[idx];
        Mi[idx] = m1;
        sq = fmaf(m1, m1, sq);
      }
      const float nf = sqrtf(block_sum(sq, red));
      const float den = nf + kEpsNorm;
      GMDN_OWN(T) {
        const int idx = (ty * T + i) * DH + tx * T + j;
        Xs[idx] = Mi[idx] / den;
      }
      __syncthreads();
      for (int st = 0; st < ns; ++st) {
        const float* X = Xs + st * MAT;
        float* Gr = Grams + st * MAT;
        float* Po = Polys + st * MAT;
        float* Xn = Xs + (st + 1) * MAT;
        tile_zero<DH, DH>(acc);
        tile_mm<DH, DH, true, true>(
            acc, DH, [&](int r, int k) { return X[r * DH + k]; },
            [&](int k, int c) { return X[c * DH + k]; }, stage);
        GMDN_OWN(T) Gr[(ty * T + i) * DH + tx * T + j] = acc[i][j];
        __syncthreads();
        tile_zero<DH, DH>(acc);
        tile_mm<DH, DH, true, false>(
            acc, DH, [&](int r, int k) { return Gr[r * DH + k]; },
            [&](int k, int c) { return Gr[k * DH + c]; }, stage);
        GMDN_OWN(T) {
          const int idx = (ty * T + i) * DH + tx * T + j;
          Po[idx] = kNsC1 * Gr[idx] + kNsC2 * acc[i][j];
        }
        __syncthreads();
        tile_zero<DH, DH>(acc);
        tile_mm<DH, DH, true, false>(
            acc, DH, [&](int r, int k) { return Po[r * DH + k]; },
            [&](int k, int c) { return X[k * DH + c]; }, stage);
        GMDN_OWN(T) {
          const int idx = (ty * T + i) * DH + tx * T + j;
          Xn[idx] = kNsC0 * X[idx] + acc[i][j];
        }
        __syncthreads();
      }
      const float* Y = Xs + ns * MAT;
      float pb = 0.f;
      GMDN_OWN(T) {
        const int idx = (ty * T + i) * DH + tx * T + j;
        pb = fmaf(sb[i][j], Y[idx], pb);
        Xbar[idx] = b * sb[i][j];
      }
      db_i = block_sum(pb, red);  // barrier inside also publishes Xbar
      for (int st = ns - 1; st >= 0; --st) {
        const float* X = Xs + st * MAT;
        const float* Gr = Grams + st * MAT;
        const float* Po = Polys + st * MAT;
        // Bbar = Xbar X^T
        tile_zero<DH, DH>(acc);
        tile_mm<DH, DH, true, true>(
            acc, DH, [&](int r, int k) { return Xbar[r * DH + k]; },
            [&](int k, int c) { return X[c * DH + k]; }, stage);
        GMDN_OWN(T) Bbar[(ty * T + i) * DH + tx * T + j] = acc[i][j];
        __syncthreads();
        // Gbar = c1 Bbar + c2 (Bbar Gram + Gram Bbar)
        tile_zero<DH, DH>(acc);
        tile_mm<DH, DH, true, false>(
            acc, DH, [&](int r, int k) { return Bbar[r * DH + k]; },
            [&](int k, int c) { return Gr[k * DH + c]; }, stage);
        tile_mm<DH, DH, true, false>(
            acc, DH, [&](int r, int k) { return Gr[r * DH + k]; },
            [&](int k, int c) { return Bbar[k * DH + c]; }, stage);
        GMDN_OWN(T) {
          const int idx = (ty * T + i) * DH + tx * T + j;
          Gbar[idx] = kNsC1 * Bbar[idx] + kNsC2 * acc[i][j];
        }
        __syncthreads();
        GMDN_OWN(T) {
          const int r = ty * T + i, c = tx * T + j;
          Gsym[r * DH + c] = Gbar[r * DH + c] + Gbar[c * DH + r];
        }
        __syncthreads();
        // Xbar <- c0 Xbar + Poly Xbar + Gsym X
        tile_zero<DH, DH>(acc);
        tile_mm<DH, DH, true, false>(
            acc, DH, [&](int r, int k) { return Po[r * DH + k]; },
            [&](int k, int c) { return Xbar[k * DH + c]; }, stage);
        tile_mm<DH, DH, true, false>(
            acc, DH, [&](int r, int k) { return Gsym[r * DH + k]; },
            [&](int k, int c) { return X[k * DH + c]; }, stage);
        GMDN_OWN(T) {
          const int idx = (ty * T + i) * DH + tx * T + j;
          Xbar[idx] = kNsC0 * Xbar[idx] + acc[i][j];
        }
        __syncthreads();
      }
      float pin = 0.f;
      GMDN_OWN(T) {
        const int idx = (ty * T + i) * DH + tx * T + j;
        pin = fmaf(Xbar[idx], Mi[idx], pin);
      }
      const float inner = block_sum(pin, red);
      const float inv_nf = 1.f / fmaxf(nf, 1e-12f);
      float pm = 0.f;
      GMDN_OWN(T) {
        const int idx = (ty * T + i) * DH + tx * T + j;
        const float vjp = Xbar[idx] / den - inner / (den * den) * (Mi[idx] * inv_nf);
        const float mt = Mb[idx] + vjp;
        pm = fmaf(mt, M_hist[base + idx], pm);
        Mb[idx] = mu * mt;
        Gb[idx] = mt;
      }
      dm_i = block_sum(pm, red);
    }
    if (threadIdx.x == 0) {
      da[gi] = da_i;
      db[gi] = db_i;
      dm[gi] = dm_i;
      dn[gi] = dn_i;
    }
    GMDN_OWN(T) {
      const int idx = (ty * T + i) * DH + tx * T + j;
      dU[base + idx] = Gb[idx];
    }
    __syncthreads();
    // dK = -S^T Gbar
    tile_zero<DH, DH>(acc);
    tile_mm<DH, DH, false, false>(
        acc, DH, [&](int r, int k) { return Si[k * DH + r]; },
        [&](int k, int c) { return Gb[k * DH + c]; }, stage);
    GMDN_OWN(T) dK[base + (ty * T + i) * DH + tx * T + j] = -acc[i][j];
    // Sbar <- a Sbar - Gbar K^T + gS
    tile_zero<DH, DH>(acc);
    tile_mm<DH, DH, true, true>(
        acc, DH, [&](int r, int k) { return Gb[r * DH + k]; },
        [&](int k, int c) { return Ki[c * DH + k]; }, stage);
    GMDN_OWN(T) {
      const int idx = (ty * T + i) * DH + tx * T + j;
      sb[i][j] = a * sb[i][j] - acc[i][j] + gS[base + idx];
    }
  }
}

template <int DH>
cudaError_t launch_fwd(const ScanArgs& p, cudaStream_t st) {
  scan_fwd_ieee_kernel<DH><<<p.BH, kThreads, 0, st>>>(p.U, p.K, p.a, p.b, p.m, p.n, p.S,
                                                      p.M_hist, p.V_hist, p.scratch, p.N,
                                                      p.rule, p.ns);
  return cudaGetLastError();
}

template <int DH>
cudaError_t launch_bwd(const ScanArgs& p, cudaStream_t st) {
  scan_bwd_ieee_kernel<DH><<<p.BH, kThreads, 0, st>>>(
      p.U, p.K, p.a, p.b, p.m, p.n, p.S, p.M_hist, p.V_hist, p.gS, p.dU, p.dK, p.da, p.db,
      p.dm, p.dn, p.scratch, p.N, p.rule, p.ns);
  return cudaGetLastError();
}

}  // namespace

cudaError_t scan_fwd_ieee(const ScanArgs& p, cudaStream_t st) {
  switch (p.dh) {
    case 16: return launch_fwd<16>(p, st);
    case 32: return launch_fwd<32>(p, st);
    case 64: return launch_fwd<64>(p, st);
    case 128: return launch_fwd<128>(p, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t scan_bwd_ieee(const ScanArgs& p, cudaStream_t st) {
  switch (p.dh) {
    case 16: return launch_bwd<16>(p, st);
    case 32: return launch_bwd<32>(p, st);
    case 64: return launch_bwd<64>(p, st);
    case 128: return launch_bwd<128>(p, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace gmdn
