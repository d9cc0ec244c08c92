// Forward dispatch for 16-bit inputs whose X is not per-head or whose D is at most 64:
// the row-pair kernel (fmlp_fwd_pair.cu) covers D <= 128, including the shared-input form;
// per-head X with 64 < D <= 256 runs on CTA pairs (fmlp_fwd2sm.cu), chosen by the C ABI.
// All of them replace flashmlp_fwd_kernel (flashmlp.py:63-158).
#include "fmlp_kernels.h"

namespace fmlp {

cudaError_t launch_fwd(const FwdLaunch& a) {
  switch (a.dp) {
    case 64:
    case 128: return launch_fwd_pair(a);
  }
  return cudaErrorNotSupported;
}

}  // namespace fmlp
