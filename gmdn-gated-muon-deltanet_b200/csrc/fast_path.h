// Tensor-core (tcgen05) paths, selected by GMDN_PREC_FAST.
#pragma once

#include <cuda.h>

#include "scan_kernels.h"

namespace gmdn {

// Fused mixer core forward (phases 1-3), delta rule, dh 128, chunk 64, bf16.
bool chunk_fwd_tc_supported(const ChunkArgs& p);
size_t chunk_fwd_tc_saved_bytes(int BH, int N);
cudaError_t chunk_fwd_tc(const ChunkArgs& p, uint16_t* S_hist, uint32_t* status,
                         cudaStream_t st);

// Backward of the fused forward (same shapes): bw1 runs the reverse state
// chain per (b, h) and writes Sb_{j+1} (bf16) per chunk; bw2 computes every
// token and gate gradient per (b, h, chunk).
bool chunk_bwd_tc_supported(const ChunkArgs& p);
size_t chunk_bwd_tc_workspace_bytes(int BH, int N);
cudaError_t chunk_bwd1_tc(const ChunkArgs& p, uint16_t* Sbar_hist, uint32_t* status,
                          cudaStream_t st);
cudaError_t chunk_bwd2_tc(const ChunkArgs& p, const uint16_t* S_hist, const uint16_t* Sbar_hist,
                          uint32_t* status, cudaStream_t st);

// rows x 128 bf16 row-major matrix as a TMA map with 64 x box_rows boxes and
// 128-byte swizzle.
cudaError_t make_tmap_rows128(CUtensorMap* map, const void* base, uint64_t rows,
                              uint32_t box_rows);

}  // namespace gmdn
