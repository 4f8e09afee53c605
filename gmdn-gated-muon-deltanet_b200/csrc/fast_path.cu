// Tensor-core scan path: not built yet for any shape, so GMDN_PREC_FAST runs
// the exact-fp32 kernels.
#include "fast_path.h"

namespace gmdn {

bool fast_scan_supported(const ScanArgs&) { return false; }
cudaError_t scan_fwd_fast(const ScanArgs&, cudaStream_t) { return cudaErrorNotSupported; }
cudaError_t scan_bwd_fast(const ScanArgs&, cudaStream_t) { return cudaErrorNotSupported; }

}  // namespace gmdn
