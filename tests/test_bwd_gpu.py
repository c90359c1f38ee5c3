"""The backward (ngdn2_bwd behind ChunkNestedGDN2Function.backward) on the GPU
against autograd through the torch oracle (oracle/naive_torch.py, float64 on
the CPU; its gradients are pinned to autograd through the reference's own
oracle by tests/test_oracle_bwd.py), and against those golden gradients
directly. Cases follow the reference's own backward test
(tests/ops/test_chunk.py:19-83: fp32 inputs, random upstream gradient, both
promotion arms) at sizes the oracle finishes in seconds.

Bar: fp32 inputs, every gradient within 1e-3 of the oracle's scale
(max |got - ref| / max |ref|): the backward runs in fp32 through a 64 x 64
triangular solve and the promotion chain. bf16 inputs: 2e-2, the reference's
own tolerance (test_chunk.py:17)."""

import numpy as np
import pytest
import torch

from _util import GOLDEN, LOWP_REL, OP_ARGS, rel_err
from nested_recurrent_memory_b200 import chunk_nested_gdn2
from nested_recurrent_memory_b200.synthetic import op_inputs
from test_oracle_bwd import bwd_case_names, oracle_grads

pytestmark = pytest.mark.gpu

LEAVES = OP_ARGS[:12]
BWD_REL = 1e-3


def _cuda_grads(d, L, promotion, dtype=torch.float32):
    """Autograd through this package's op of sum(o * d_o) + sum(final * d_final)."""
    leaves = {n: torch.tensor(d[n]).to("cuda", dtype).requires_grad_(True) for n in LEAVES}
    init = d.get("initial_state")
    init_t = (torch.tensor(init, dtype=torch.float32, device="cuda").requires_grad_(True)
              if init is not None else None)
    o, s = chunk_nested_gdn2(**leaves, n_queries_per_level=list(d["n_queries_per_level"]),
                             firing_intervals=list(d["firing_intervals"]), L=L,
                             initial_state=init_t, output_final_state=True, promotion=promotion)
    loss = (o.float() * torch.tensor(d["d_o"], device="cuda")).sum() + \
        (s * torch.tensor(d["d_final"], device="cuda")).sum()
    loss.backward()
    torch.cuda.synchronize()
    grads = {n: (t.grad.float().cpu().numpy() if t.grad is not None
                 else np.zeros(t.shape, np.float32)) for n, t in leaves.items()}
    if init_t is not None:
        grads["initial_state"] = init_t.grad.cpu().numpy()
    return grads


def _compare(got, ref, tol):
    for n, r in ref.items():
        g = got[n]
        assert g.shape == r.shape, n
        if r.size == 0:
            continue
        if np.abs(r).max() == 0:
            assert np.abs(g).max() < 1e-6, n
        else:
            assert rel_err(g, r) < tol, (n, rel_err(g, r))


def _case(B, T, H, K, V, L, N, firing, nq=None, seed=0, with_init=False):
    inp = op_inputs(B, T, H, K, V, L, N, firing_intervals=firing, n_queries_per_level=nq,
                    seed=seed)
    L = inp.pop("L")
    d = {n: (t.numpy() if torch.is_tensor(t) else np.asarray(t)) for n, t in inp.items()}
    gen = torch.Generator().manual_seed(seed + 1)
    d["d_o"] = torch.randn(B, T, H, V, generator=gen).numpy()
    d["d_final"] = (torch.randn(B, H, L, K, V, generator=gen) * 0.1).numpy()
    if with_init:
        d["initial_state"] = (torch.randn(B, H, L, K, V, generator=gen) * 0.1).numpy()
    return d, L


@pytest.mark.parametrize("name", bwd_case_names())
def test_gradients_match_reference_golden(name):
    d = dict(np.load(GOLDEN / f"{name}.npz"))
    L, promotion = int(d["L"]), str(d["promotion"])
    got = _cuda_grads(d, L, promotion)
    ref = {n: d[f"grad_{n}"] for n in LEAVES}
    if "grad_initial_state" in d:
        ref["initial_state"] = d["grad_initial_state"]
    _compare(got, ref, BWD_REL)


# (B, T, H, K, V, L, N, firing, n_queries): the reference's test_chunk.py
# CASES at oracle-friendly sizes, plus a ragged T and K = V = 128.
CASES = [
    (1, 128, 2, 64, 64, 2, 16, (1, 2), None),
    (2, 256, 2, 32, 32, 3, 16, (1, 2, 4), None),
    (1, 256, 1, 64, 64, 3, 32, (1, 2, 4), (32, 16)),
    (1, 256, 2, 32, 32, 2, 16, (1, 1), None),
    (1, 200, 1, 32, 32, 3, 16, (1, 2, 4), None),
    (1, 192, 1, 128, 128, 2, 64, (1, 2), None),
]


@pytest.mark.parametrize("promotion", ["learned", "merge"])
@pytest.mark.parametrize(("B", "T", "H", "K", "V", "L", "N", "firing", "nq"), CASES)
def test_gradients_match_oracle(B, T, H, K, V, L, N, firing, nq, promotion):
    d, L = _case(B, T, H, K, V, L, N, firing, nq, seed=B * 7 + T + K)
    _, _, ref = oracle_grads(d, L, promotion)
    got = _cuda_grads(d, L, promotion)
    _compare(got, ref, BWD_REL)


@pytest.mark.parametrize("promotion", ["learned", "merge"])
def test_initial_state_gradient(promotion):
    """test_chunk.py:94-111 with d_final as well."""
    d, L = _case(2, 256, 2, 32, 32, 2, 16, (1, 2), seed=4, with_init=True)
    _, _, ref = oracle_grads(d, L, promotion)
    got = _cuda_grads(d, L, promotion)
    _compare(got, ref, BWD_REL)


@pytest.mark.parametrize("lift", [0.02, 0.1])
def test_positive_log_decays(lift):
    """Log-decays above zero on 8 channels of the second chunk: the local
    pass takes the clamped per-term sums on those channels and the running
    products everywhere else (and the checkpointing prep its per-element
    decay loop for that chunk). All against the float64 oracle."""
    d, L = _case(1, 256, 2, 64, 64, 2, 16, (1, 2), seed=12)
    d["g"] = d["g"].copy()
    d["g"][:, 64:128, :, :8] = lift
    _, _, ref = oracle_grads(d, L, "learned")
    _compare(_cuda_grads(d, L, "learned"), ref, BWD_REL)


def test_l1_reduces_to_level_zero():
    d, L = _case(1, 192, 2, 64, 32, 1, 16, (1,), seed=6, with_init=True)
    _, _, ref = oracle_grads(d, L, "learned")
    _compare(_cuda_grads(d, L, "learned"), ref, BWD_REL)


def test_bf16_inputs_within_reference_tolerance():
    """test_chunk.py:135-144 runs the backward under autocast: here bf16
    inputs (the forward on the tensor-core path) against the fp64 oracle of
    the bf16-rounded inputs, at the reference's 2e-2."""
    d, L = _case(1, 256, 2, 128, 128, 3, 64, (1, 2, 4), seed=8)
    for n in LEAVES:
        d[n] = torch.tensor(d[n]).to(torch.bfloat16).float().numpy()
    _, _, ref = oracle_grads(d, L, "learned")
    got = _cuda_grads(d, L, "learned", dtype=torch.bfloat16)
    for n in ("q", "k", "v", "g", "b", "w", "mix_weights"):
        assert np.isfinite(got[n]).all(), n
    _compare(got, ref, LOWP_REL)


def test_unused_final_state_and_repeatability():
    """Only o carries gradient; two runs give the same bits (the parameter
    gradients are summed over batch rows in a fixed order)."""
    d, L = _case(2, 128, 2, 32, 32, 2, 16, (1, 2), seed=9)
    leaves = {n: torch.tensor(d[n]).cuda().requires_grad_(True) for n in LEAVES}
    kw = dict(n_queries_per_level=[16], firing_intervals=[1, 2], L=L)
    grads = []
    for _ in range(2):
        for t in leaves.values():
            t.grad = None
        o, _ = chunk_nested_gdn2(**leaves, **kw)
        o.sum().backward()
        grads.append({n: t.grad.clone() for n, t in leaves.items()})
    for n in LEAVES:
        assert torch.equal(grads[0][n], grads[1][n]), n
