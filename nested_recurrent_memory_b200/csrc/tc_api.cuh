// Interface of the tensor-core (tcgen05) kernel family to the ABI layer.
#pragma once

#include <cuda.h>

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

// Whether the level-segmented tensor-core family runs this call, its
// workspace, launches and launch count (csrc/seg.cu).
bool seg_supports(const ngdn2_fwd_args* a);
size_t seg_workspace_bytes(const FwdParams& p);
cudaError_t launch_fwd_seg(FwdParams p, void* workspace, int stage, cudaStream_t stream);
int num_launches_seg(const FwdParams& p);

namespace tcx { struct TcLayout; }
// Pieces of the fused family that the segmented family reuses (csrc/tc.cu):
// the promotion-operand layouts, the chunk prep, and q's tensor map for the
// upper levels' query tiles (hl_mode 2: no map, read q with plain loads).
cudaError_t launch_tc_params(const FwdParams& p, const tcx::TcLayout& lay, char* ws,
                             cudaStream_t stream);
cudaError_t launch_tc_prep(const FwdParams& p, const tcx::TcLayout& lay, char* ws,
                           cudaStream_t stream);
bool tc_make_q_map(const FwdParams& p, CUtensorMap* m, int* hl_mode);

}  // namespace ngdn2
