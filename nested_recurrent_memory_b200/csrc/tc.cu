// Tensor-core (tcgen05) kernel family.
#include "tc_api.cuh"

namespace ngdn2 {

bool tc_supports(const ngdn2_fwd_args*) { return false; }
size_t tc_workspace_bytes(const FwdParams&) { return 0; }
cudaError_t launch_fwd_tc(FwdParams, void*, int, cudaStream_t) { return cudaErrorNotSupported; }
int num_launches_tc(const FwdParams&) { return 0; }

}  // namespace ngdn2
