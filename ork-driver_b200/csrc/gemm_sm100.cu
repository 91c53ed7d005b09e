// gemm_sm100.cu -- tensor-core (tcgen05) path for batched M. Placeholder until the kernel lands: the
// decode GEMV serves every M meanwhile.
#include "ork_internal.h"

namespace orkb {

bool gemm_tc_supports(int, int, int, int) { return false; }

cudaError_t launch_gemm_tc(const RunArgs &, cudaStream_t, bool, int *) { return cudaErrorNotSupported; }

}  // namespace orkb
