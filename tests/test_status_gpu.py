"""Device-side failures reach the caller through the public API.

Every forward reports into a sticky per-device status word. These tests make
a wait run out without faulting anything: the forward is given a start gate
(a device word that nothing sets) and a short poll limit, so its first
kernel gives up before any other work, sets NGDN2_STATUS_GATE_TIMEOUT, and
every later kernel of that forward returns at once. The error must then
surface through ``FwdCall.check``, ``check_status`` and the next launch on
the device, and the outputs must be untouched.
"""

import pytest
import torch

from nested_recurrent_memory_b200 import FwdCall, KernelStatusError, check_status
from nested_recurrent_memory_b200.synthetic import config_inputs

pytestmark = pytest.mark.gpu


def _inputs(d, dtype):
    inp = config_inputs(1, 256, 2, d, d, 3, 16, (1, 2, 4), dtype=dtype, seed=5,
                        gate_proj_std=d ** -0.5)
    L = inp.pop("L")
    return {k: (v.cuda() if torch.is_tensor(v) and v.is_floating_point() else v)
            for k, v in inp.items()}, L


@pytest.mark.parametrize(("path", "dtype", "d"), [("tc", torch.bfloat16, 128),
                                                   ("simt", torch.float32, 64)])
def test_closed_gate_reports_and_computes_nothing(path, dtype, d):
    inp, L = _inputs(d, dtype)
    check_status()  # start clean
    ref_o, ref_s = (t.clone() for t in FwdCall(**inp, L=L, path=path).launch())
    gate = torch.zeros(1, dtype=torch.int32, device="cuda")
    call = FwdCall(**inp, L=L, path=path, gate=gate, gate_polls=2000)
    call.o.fill_(float("nan"))
    call.final.fill_(float("nan"))
    call.launch()
    with pytest.raises(KernelStatusError, match="start gate"):
        call.check()
    assert torch.isnan(call.o).all() and torch.isnan(call.final).all()
    # cleared after raising: the same call with the gate open runs normally
    gate.fill_(1)
    o, s = call.launch()
    call.check()
    assert torch.equal(o, ref_o) and torch.equal(s, ref_s)


def test_timeout_surfaces_at_the_next_launch():
    inp, L = _inputs(128, torch.bfloat16)
    check_status()
    gate = torch.zeros(1, dtype=torch.int32, device="cuda")
    gated = FwdCall(**inp, L=L, path="tc", gate=gate, gate_polls=2000)
    plain = FwdCall(**inp, L=L, path="tc")
    gated.launch()
    torch.cuda.synchronize()  # the status copy has landed
    with pytest.raises(KernelStatusError):
        plain.launch()
    plain.launch()  # the word was cleared
    check_status()


def test_open_gate_matches_ungated_bit_for_bit():
    inp, L = _inputs(128, torch.bfloat16)
    ref = [t.clone() for t in FwdCall(**inp, L=L, path="tc").launch()]
    gate = torch.ones(1, dtype=torch.int32, device="cuda")
    got = FwdCall(**inp, L=L, path="tc", gate=gate, gate_polls=10).launch()
    check_status()
    assert all(torch.equal(a, b) for a, b in zip(got, ref))
