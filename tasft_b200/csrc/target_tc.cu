// Tensor-core tile max for the gate target (filled in with the tcgen05 kernel).
#include "tc.cuh"

namespace tasft {
int gate_target_blockmax_tc(const tasft_target_args&, float*, cudaStream_t) { return TASFT_ERR_UNSUPPORTED; }
}  // namespace tasft
