// Tensor-core (tcgen05) paths, selected by GMDN_PREC_FAST.
#pragma once

#include <cuda.h>

#include "scan_kernels.h"

namespace gmdn {

// Buffers of the tensor-core path, carved by the C ABI from the caller's
// `saved` (forward -> backward) and `workspace` buffers.
//
// Per-thread slab layouts: the state warps own row c (a TMEM lane) and one
// half (64 columns) of every dh x dh matrix.  Matrices only they touch are
// stored so that one warp-wide 16-byte access covers 512 contiguous bytes:
//   fp32 slab: float4 index ((bh * 2 + half) * 16 + f) * 128 + c, f = column / 4 in the half
//   bf16 slab: uint4 index ((m * 2 + half) * 8 + g) * 128 + c, g = column / 8 in the half,
//              m = bh * N + j (one matrix per chunk)
struct TcBufs {
  uint32_t* status;       // device status word (workspace)
  uint16_t* S_hist;       // saved: S_j, bf16 row-major (every rule)
  uint16_t* S_lo_hist;    // saved, muon: S_j - bf16(S_j), bf16 row-major
  uint16_t* G_hist;       // saved, adam: G_j, bf16 slab
  uint16_t* Mp_hist;      // saved, adam: pre-update M_j, bf16 slab
  uint16_t* Vp_hist;      // saved, adam: pre-update V_j, bf16 slab
  float* M_hist;          // saved, muon: M_{j+1} (post-update), fp32 slab per chunk
  uint8_t* X_hist;        // saved, muon: Newton-Schulz inputs X_0..X_{ns-1}, split bf16
                          //   SW128 tiles, 64 KB per step (hi 32 KB, lo 32 KB), ns per chunk
  uint16_t* Gbar_hist;    // workspace: cotangent of G_j, bf16 row-major (delta: Sb_{j+1})
  uint16_t* Gbar_lo_hist; // workspace, muon: its bf16 remainder (Gb - bf16(Gb)); the muon
                          //   cotangent is large while its contractions with k are small
  float* M_ws;            // workspace, adam: fp32 slab of M (forward) / Mbar (backward)
  float* V_ws;            // workspace, adam: fp32 slab of V (forward) / Vbar (backward)
  float *dac, *dbc, *dmc, *dnc;  // workspace, adam: cotangents of a_c, b_c, mu_c, nu_c
  uint32_t* progress;     // workspace, delta: per (b, h), chunks whose Gb_j the fused
                          //   backward's chain has stored (counted from the last)
};

// True when the driver's cuTensorMapEncodeTiled could be resolved (every
// tensor-core path needs it).
bool tma_encode_available();

// Fused mixer core forward (phases 1-3), delta and adam rules, dh 128 or 64,
// chunk 64, bf16.
bool chunk_fwd_tc_supported(const ChunkArgs& p);
cudaError_t chunk_fwd_tc(const ChunkArgs& p, const TcBufs& b, cudaStream_t st);

// Fused mixer core forward, muon rule (Newton-Schulz on the tensor cores with
// split bf16 operands), dh 128, chunk 64, bf16.
bool chunk_fwd_muon_tc_supported(const ChunkArgs& p);
cudaError_t chunk_fwd_muon_tc(const ChunkArgs& p, const TcBufs& b, int ns, cudaStream_t st);
// Reverse chain of the muon forward (msign VJP with split bf16 products); the
// token gradients then come from chunk_bwd2_tc.
cudaError_t chunk_bwd1_muon_tc(const ChunkArgs& p, const TcBufs& b, int ns, cudaStream_t st);

// Backward of the fused forward (same shapes): bw1 runs the reverse state
// chain per (b, h) and writes the cotangent of G_j (bf16) per chunk, plus the
// chunk-scalar cotangents for adam; bw2 computes every token and gate
// gradient per (b, h, chunk).
bool chunk_bwd_tc_supported(const ChunkArgs& p);
cudaError_t chunk_bwd1_tc(const ChunkArgs& p, const TcBufs& b, cudaStream_t st);
// first > 0: only the tiles the fused backward left (its n_fused on)
cudaError_t chunk_bwd2_tc(const ChunkArgs& p, const TcBufs& b, cudaStream_t st, int first = 0);
// Delta with fewer sequences than SMs: one cooperative launch runs the chains
// and, on the SMs they leave, the token gradients of the first n_fused tiles
// in the order the chains finish them; chunk_bwd2_tc(..., n_fused) does the
// rest.  chunk_bwd_fused_tiles is n_fused (0: use bw1 + bw2).
int chunk_bwd_fused_tiles(const ChunkArgs& p);
cudaError_t chunk_bwd_fused_tc(const ChunkArgs& p, const TcBufs& b, int n_fused,
                               cudaStream_t st);

// Phase-2 state scan on the tensor cores (scan_tc.cu): gmdn_scan_fwd with
// GMDN_PREC_FAST, delta and adam, dh 128; split-bf16 products.  `status` is
// the device status word (bounded waits).
bool scan_fwd_tc_supported(const ScanArgs& p);
cudaError_t scan_fwd_tc(const ScanArgs& p, uint32_t* status, cudaStream_t st);
// Its backward, delta at dh 128: the reverse chain (dU) on the tensor cores,
// then dK = -S^T dU and da = <dU, S> for every matrix in a second kernel.
bool scan_bwd_tc_supported(const ScanArgs& p);
cudaError_t scan_bwd_chain_tc(const ScanArgs& p, uint32_t* status, cudaStream_t st);
cudaError_t scan_bwd_dk_tc(const ScanArgs& p, uint32_t* status, cudaStream_t st);

// Mixer epilogue (epilogue.cu): per-head RMSNorm of o (B, H, T, dh) into
// y (B, T, H*dh), and its backward (dw is zeroed, then accumulated); dh 32, 64
// or 128, bf16 or fp32 input and output.
cudaError_t head_rmsnorm_fwd(const void* o, const float* w, void* y, int B, int H, int T, int dh,
                             float eps, bool in_f32, bool out_f32, cudaStream_t st);
cudaError_t head_rmsnorm_bwd(const void* o, const float* w, const void* dy, void* d_o, float* dw,
                             int B, int H, int T, int dh, float eps, bool in_f32, bool out_f32,
                             cudaStream_t st);

// Mixer prologue (prologue.cu): causal depthwise conv (k=4) + SiLU + q/k L2
// norm of u (B, T, 3D) into q, k, v (B, H, T, dh), sigmoid of the gate logits
// (B, T, nG*H) into g (nG, B, H, T); backward (dcw, dcb zeroed, then
// accumulated).  dh 32, 64 or 128; bf16 or fp32 I/O; conv weight / bias fp32.
cudaError_t mixer_prologue_fwd(const void* u, const float* cw, const float* cb, const void* gl,
                               void* q, void* k, void* v, void* g, int B, int T, int H, int dh,
                               int n_gates, bool io_f32, cudaStream_t st);
cudaError_t mixer_prologue_bwd(const void* u, const float* cw, const float* cb, const void* gl,
                               const void* dq, const void* dk, const void* dv, const void* dg,
                               void* du, float* dcw, float* dcb, void* dgl, int B, int T, int H,
                               int dh, int n_gates, bool io_f32, cudaStream_t st);

// Failure-detection self-test (selftest.cu): one CTA's bounded wait on an
// mbarrier nothing arrives on gives up after limit_ns and sets bit 0 of *status.
cudaError_t wait_timeout_selftest(uint32_t* status, uint64_t limit_ns, cudaStream_t st);

// rows x width bf16 row-major matrix (width 64 or 128) as a TMA map with
// 64 x box_rows boxes and 128-byte swizzle.  With width 64 the box at column
// 64 lies wholly outside the matrix and a load of it fills the shared-memory
// panel with zeros: the dh-128 kernels read a dh-64 head as one whose upper
// 64 features are zero.
cudaError_t make_tmap_rows128(CUtensorMap* map, const void* base, uint64_t rows,
                              uint32_t box_rows, uint32_t width = 128);

}  // namespace gmdn
