"""The differentiable torch oracle (oracle/naive_torch.py) pinned against the
reference: its forward against the numpy oracle, and its autograd gradients
against golden gradients taken by autograd through the reference's own
naive_chunk_nested_gdn2 (tests/golden/bwd_*.npz, written by
tests/golden/make_golden_bwd.py). CPU only."""

import numpy as np
import pytest
import torch

import oracle
from _util import GOLDEN, OP_ARGS, rel_err
from oracle import naive_torch

LEAVES = OP_ARGS[:12]
# float64 oracle against the fp32 reference autograd: only rounding differs.
PIN = 1e-4


def bwd_case_names():
    return sorted(p.stem for p in GOLDEN.glob("bwd_*.npz"))


def oracle_grads(d, L, promotion, dtype=torch.float64):
    """Autograd through the torch oracle of sum(o * d_o) + sum(final * d_final)."""
    leaves = {n: torch.tensor(d[n], dtype=dtype, requires_grad=True) for n in LEAVES}
    init = d.get("initial_state")
    init_t = torch.tensor(init, dtype=dtype, requires_grad=True) if init is not None else None
    o, s = naive_torch.chunk_forward(
        **leaves, n_queries_per_level=list(d["n_queries_per_level"]),
        firing_intervals=list(d["firing_intervals"]), L=L, initial_state=init_t,
        promotion=promotion, dtype=dtype)
    loss = (o * torch.tensor(d["d_o"], dtype=dtype)).sum() + \
        (s * torch.tensor(d["d_final"], dtype=dtype)).sum()
    loss.backward()
    grads = {n: (t.grad if t.grad is not None else torch.zeros_like(t)).numpy()
             for n, t in leaves.items()}
    if init_t is not None:
        grads["initial_state"] = init_t.grad.numpy()
    return o.detach().numpy(), s.detach().numpy(), grads


@pytest.mark.parametrize("name", bwd_case_names())
def test_torch_oracle_gradients_match_reference(name):
    d = dict(np.load(GOLDEN / f"{name}.npz"))
    L, promotion = int(d["L"]), str(d["promotion"])
    o, s, grads = oracle_grads(d, L, promotion)
    assert rel_err(o, d["out_o"]) < PIN
    assert rel_err(s, d["out_final"]) < PIN
    for n, gr in grads.items():
        ref = d[f"grad_{n}"]
        if ref.size == 0:
            assert gr.size == 0, n
        elif np.abs(ref).max() == 0:
            assert np.abs(gr).max() < 1e-12, n
        else:
            assert rel_err(gr, ref) < PIN, n


@pytest.mark.parametrize("promotion", ["learned", "merge"])
def test_torch_oracle_forward_matches_numpy_oracle(promotion):
    from nested_recurrent_memory_b200.synthetic import op_inputs
    inp = op_inputs(2, 200, 2, 32, 32, 3, 16, firing_intervals=(1, 2, 4), seed=3)
    L = inp.pop("L")
    init = np.random.RandomState(0).randn(2, 2, 3, 32, 32) * 0.1
    a = {k: (v.double().numpy() if torch.is_tensor(v) and v.is_floating_point() else v)
         for k, v in inp.items()}
    ro, rs = oracle.chunk_forward(**a, L=L, initial_state=init, output_final_state=True,
                                  promotion=promotion)
    o, s = naive_torch.chunk_forward(**inp, L=L, initial_state=torch.tensor(init),
                                     promotion=promotion)
    assert rel_err(o.numpy(), ro) < 1e-12
    assert rel_err(s.numpy(), rs) < 1e-12


def update_oracle_grads(d, dtype=torch.float64):
    """Autograd through the torch oracle's write scan of
    sum(states * d_states) + sum(final * d_final)."""
    names = ("keys", "values", "g", "b", "w")
    leaves = {n: torch.tensor(d[n], dtype=dtype, requires_grad=True) for n in names}
    init = d.get("initial_state")
    init_t = torch.tensor(init, dtype=dtype, requires_grad=True) if init is not None else None
    states, final = naive_torch.update_scan(**leaves, n_groups=int(d["n_groups"]),
                                            initial_state=init_t)
    loss = (states * torch.tensor(d["d_states"], dtype=dtype)).sum() + \
        (final * torch.tensor(d["d_final"], dtype=dtype)).sum()
    loss.backward()
    out = {n: t.grad.numpy() for n, t in leaves.items()}
    if init_t is not None:
        out["initial_state"] = init_t.grad.numpy()
    return states.detach().numpy(), final.detach().numpy(), out


def test_torch_oracle_update_scan_gradients_match_reference():
    d = dict(np.load(GOLDEN / "bwdupd_scan.npz"))
    states, final, grads = update_oracle_grads(d)
    assert rel_err(states, d["out_states"]) < 1e-12
    assert rel_err(final, d["out_final"]) < 1e-12
    for n, gr in grads.items():
        assert rel_err(gr, d[f"grad_{n}"]) < 1e-10, n
