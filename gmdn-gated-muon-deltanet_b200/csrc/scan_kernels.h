// Internal launch interface between the C ABI (abi.cu) and the kernels.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace gmdn {

// Per-(b,h) scratch matrices (dh x dh fp32) of the exact-fp32 scan.
constexpr int kScanFwdScratchMats = 6;  // S, M, V, X, Gram, Poly
__host__ __device__ constexpr int scan_bwd_scratch_mats(int ns) {
  // G, Mbar, Vbar, Gbar, Mi, Xbar, Bbar, GramBar, GramBarSym + NS iterates,
  // Grams and Polys of one chunk
  return 9 + (ns + 1) + 2 * ns;
}

struct ScanArgs {
  const float *U, *K, *a, *b, *m, *n;
  float* S;          // forward: output states; backward: input states
  float *M_hist, *V_hist;
  const float* gS;
  float *dU, *dK, *da, *db, *dm, *dn;
  float* scratch;
  int BH, N, dh, rule, ns;
};

cudaError_t scan_fwd_ieee(const ScanArgs& p, cudaStream_t st);
cudaError_t scan_bwd_ieee(const ScanArgs& p, cudaStream_t st);

// Mixer-core (chunk) kernels of the exact-fp32 path.
struct ChunkArgs {
  const void *q, *k, *v, *dO;     // (B, H, T, dh) bf16 or fp32 (io_f32)
  const float *alpha, *beta, *mu, *nu;  // (B, H, T); nu may be null
  void* o;                        // forward output
  void *dq, *dk, *dv;             // backward outputs
  float *dalpha, *dbeta, *dmu, *dnu;
  // per-chunk products and scalars (workspace / saved)
  float *Kw, *Uv, *S, *gS, *dUv, *dKw;
  float *a_c, *b_c, *m_c, *n_c;        // chunk gate products (B, H, N)
  float *da_c, *db_c, *dm_c, *dn_c;    // their cotangents
  int BH, T, N, C, dh, rule;
  bool io_f32;
};

cudaError_t chunk_prep_ieee(const ChunkArgs& p, cudaStream_t st);
cudaError_t chunk_out_ieee(const ChunkArgs& p, cudaStream_t st);
cudaError_t chunk_state_grad_ieee(const ChunkArgs& p, cudaStream_t st);
cudaError_t chunk_token_grad_ieee(const ChunkArgs& p, cudaStream_t st);

}  // namespace gmdn
