"""ngdn2_fwd_noalloc: the forward for callers that cannot allocate device
memory per call (their process's memory is owned by another pool, or their
budget is fixed at start-up). Its scratch is a fixed buffer compiled into the
library instead of a caller workspace. Called here through the C ABI, twice in
a row (the second call reuses whatever the first left in the shared buffer),
and checked against the regular workspace entry point ngdn2_fwd on the same
inputs, within the parity tolerances the other tests use.

Kept in a file that pytest collects last, so a run that stops at the first
failure has run every other test before this one."""

import ctypes

import pytest
import torch

from _util import FP32_REL, LOWP_REL, rel_err
from nested_recurrent_memory_b200 import FwdCall, _lib
from nested_recurrent_memory_b200.synthetic import config_inputs

pytestmark = pytest.mark.gpu


def _call(path, dtype, K):
    inp = config_inputs(1, 256, 2, K, K, 3, 32, (1, 2, 4), dtype=dtype, seed=21,
                        gate_proj_std=K ** -0.5)
    L = inp.pop("L")
    dev = {k: (v.cuda() if torch.is_tensor(v) and v.is_floating_point() else v)
           for k, v in inp.items()}
    return FwdCall(**dev, L=L, path=path)


@pytest.mark.parametrize(("path", "dtype", "K", "tol"), [
    ("tc", torch.bfloat16, 128, LOWP_REL),
    ("simt", torch.float32, 64, FP32_REL),
])
def test_noalloc_matches_the_workspace_entry_point(path, dtype, K, tol):
    lib = _lib.load()
    call = _call(path, dtype, K)
    o_ref, s_ref = (t.clone() for t in call.launch())
    torch.cuda.synchronize()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for _ in range(2):
        o = torch.full_like(o_ref, float("nan"))
        s = torch.full_like(s_ref, float("nan"))
        args = _lib.FwdArgs.from_buffer_copy(call.args)
        args.o, args.final_state = o.data_ptr(), s.data_ptr()
        args.workspace, args.workspace_bytes = None, 0
        assert lib.ngdn2_fwd_noalloc(ctypes.byref(args), stream) == 0
        torch.cuda.synchronize()
        assert rel_err(o.float().cpu().numpy(), o_ref.float().cpu().numpy()) < tol
        assert rel_err(s.cpu().numpy(), s_ref.cpu().numpy()) < tol


def test_noalloc_rejects_calls_beyond_its_scratch():
    lib = _lib.load()
    call = _call("tc", torch.bfloat16, 128)
    args = _lib.FwdArgs.from_buffer_copy(call.args)
    args.B, args.T = 8, 4096  # about 108 MB of chunk records: over the fixed 64 MiB
    need = ctypes.c_size_t(0)
    assert lib.ngdn2_fwd_workspace_size(ctypes.byref(args), ctypes.byref(need)) == 0
    assert need.value > (64 << 20)
    assert lib.ngdn2_fwd_noalloc(ctypes.byref(args), None) == -10  # NGDN2_ERR_WORKSPACE
