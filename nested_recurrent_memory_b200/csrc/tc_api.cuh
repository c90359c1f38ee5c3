// Interface of the tensor-core (tcgen05) kernel family to the ABI layer.
#pragma once

#include "fwd_params.cuh"

namespace ngdn2 {

// Whether the tensor-core path runs this call.
bool tc_supports(const ngdn2_fwd_args* a);
// Workspace bytes the tensor-core path needs for this call.
size_t tc_workspace_bytes(const FwdParams& p);
// Launch the tensor-core forward (stage 0 = all, 1 = prep, 2 = scan).
cudaError_t launch_fwd_tc(FwdParams p, void* workspace, int stage, cudaStream_t stream);
// Kernel launches per forward.
int num_launches_tc(const FwdParams& p);

}  // namespace ngdn2
