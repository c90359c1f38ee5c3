"""B200-native nested Gated DeltaNet (nested GDN-2) hot path.

A drop-in for the reference's ``nested_gdn2.ops`` ops (``chunk_nested_gdn2``
with its backward, ``chunk_nested_gdn2_fwd``, ``chunk_nested_gdn2_bwd``,
``update_state``, ``update_state_bwd``, and the one-token decode step
``naive_step_nested_gdn2`` as ``step_nested_gdn2``), computed by hand-written
sm_100a CUDA kernels behind the C ABI in ``include/ngdn2.h``. ``HostPipeline``
runs the op over host-resident batches with their copies overlapped.
"""

from .ops import (  # noqa: F401
    FwdCall,
    KernelStatusError,
    check_status,
    chunk_nested_gdn2,
    chunk_nested_gdn2_bwd,
    chunk_nested_gdn2_fwd,
    fwd_workspace_bytes,
    last_path,
    n_firings,
    n_groups,
    step_nested_gdn2,
    update_state,
    update_state_bwd,
)
from .host import HostPipeline  # noqa: F401

__version__ = "0.1.0"
