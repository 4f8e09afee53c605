// Tensor-core (tcgen05) scan path, selected by GMDN_PREC_FAST.
#pragma once

#include "scan_kernels.h"

namespace gmdn {

// True when the tensor-core kernels are built for this shape / rule.
bool fast_scan_supported(const ScanArgs& p);
cudaError_t scan_fwd_fast(const ScanArgs& p, cudaStream_t st);
cudaError_t scan_bwd_fast(const ScanArgs& p, cudaStream_t st);

}  // namespace gmdn
