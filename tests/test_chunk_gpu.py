"""The CUDA forward against the reference's golden outputs and the CPU
oracle, through the reference-facing Python API (which calls the C ABI).

Tolerances (max |got - ref| / max |ref| per tensor):
  fp32 inputs on the CUDA-core path: 1e-4;
  bf16/fp16 inputs: 2e-2 on outputs and states, against the oracle run on
  the same (cast-back) inputs.
"""

import numpy as np
import pytest
import torch

import oracle
from _util import FP32_REL, LOWP_REL, OP_ARGS, chunk_case_names, load_case, rel_err
from nested_recurrent_memory_b200 import chunk_nested_gdn2, chunk_nested_gdn2_fwd, last_path
from nested_recurrent_memory_b200.synthetic import config_inputs, op_inputs

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _to_dev(args, dtype=None):
    out = {}
    for k, v in args.items():
        t = torch.as_tensor(np.asarray(v)) if not torch.is_tensor(v) else v
        if k not in ("n_queries_per_level", "firing_intervals") and dtype is not None:
            t = t.to(dtype)
        out[k] = t.to(DEV)
    return out


def _np(t):
    return t.detach().float().cpu().numpy()


def _oracle(inp, L, promotion="learned", initial_state=None):
    a = {k: (_np(v) if torch.is_tensor(v) else v) for k, v in inp.items() if k in OP_ARGS}
    init = _np(initial_state) if initial_state is not None else None
    return oracle.chunk_forward(**a, L=L, initial_state=init, output_final_state=True,
                                promotion=promotion)


@pytest.mark.parametrize("path", ["simt"])
@pytest.mark.parametrize("name", chunk_case_names())
def test_golden_fp32(name, path):
    args, extra, d = load_case(name)
    dev = _to_dev(args)
    init = (torch.as_tensor(extra["initial_state"]).to(DEV)
            if extra["initial_state"] is not None else None)
    o, s = chunk_nested_gdn2_fwd(**dev, L=extra["L"], initial_state=init,
                                 output_final_state=True, promotion=extra["promotion"],
                                 path=path)
    assert last_path() == path
    assert rel_err(_np(o), d["out_o"]) < FP32_REL
    assert rel_err(_np(s), d["out_final"]) < FP32_REL


#  B,   T, H,   K,   V, L,  N, firing,    n_queries  (tests/ops/test_chunk.py:20-28)
CASES = [
    (1, 128, 2, 64, 64, 2, 16, (1, 2), None),
    (2, 256, 2, 64, 64, 2, 16, (1, 2), None),
    (1, 256, 4, 64, 64, 2, 32, (1, 4), None),
    (2, 512, 2, 64, 64, 3, 16, (1, 2, 4), None),
    (1, 512, 2, 64, 64, 3, 32, (1, 2, 4), (32, 16)),
    (1, 256, 2, 128, 128, 2, 16, (1, 2), None),
    (1, 256, 2, 64, 64, 2, 16, (1, 1), None),
]


@pytest.mark.parametrize("promotion", ["learned", "merge"])
@pytest.mark.parametrize(("B", "T", "H", "K", "V", "L", "N", "firing", "nq"), CASES)
def test_reference_cases_fp32(B, T, H, K, V, L, N, firing, nq, promotion):
    inp = op_inputs(B, T, H, K, V, L, N, firing_intervals=firing, n_queries_per_level=nq)
    L = inp.pop("L")
    dev = _to_dev(inp)
    o, s = chunk_nested_gdn2(**dev, L=L, output_final_state=True, promotion=promotion)
    ro, rs = _oracle(inp, L, promotion)
    assert rel_err(_np(o), ro) < FP32_REL
    assert rel_err(_np(s), rs) < FP32_REL


@pytest.mark.parametrize("T", [64, 100, 192, 320])
def test_short_and_ragged_sequences(T):
    """test_chunk.py:124-132, plus a T that is not a whole number of chunks:
    the partial last chunk still fires."""
    inp = op_inputs(1, T, 2, 64, 64, 3, 16, firing_intervals=(1, 2, 4))
    L = inp.pop("L")
    o, s = chunk_nested_gdn2(**_to_dev(inp), L=L, output_final_state=True)
    ro, rs = _oracle(inp, L)
    assert rel_err(_np(o), ro) < FP32_REL
    assert rel_err(_np(s), rs) < FP32_REL


@pytest.mark.parametrize("promotion", ["learned", "merge"])
def test_initial_state(promotion):
    inp = op_inputs(2, 256, 2, 64, 64, 2, 16, firing_intervals=(1, 2))
    L = inp.pop("L")
    init = torch.randn(2, 2, 2, 64, 64, generator=torch.Generator().manual_seed(1)) * 0.1
    o, s = chunk_nested_gdn2(**_to_dev(inp), L=L, initial_state=init.to(DEV),
                             output_final_state=True, promotion=promotion)
    ro, rs = _oracle(inp, L, promotion, init)
    assert rel_err(_np(o), ro) < FP32_REL
    assert rel_err(_np(s), rs) < FP32_REL


@pytest.mark.parametrize("lift", [0.02, 0.1])
def test_positive_log_decays_fp32(lift):
    """Log-decays above zero on some channels: the chunk's cumulative decay is
    no longer monotone there, so the CUDA-core path takes its exact
    (per-element) intra-chunk branch for that chunk and the factorised one
    elsewhere; both must match the oracle."""
    inp = op_inputs(1, 256, 2, 64, 64, 2, 16, firing_intervals=(1, 2))
    L = inp.pop("L")
    g = inp["g"].clone()
    g[:, 64:128, :, :8] = lift          # second chunk: positive on 8 channels
    inp["g"] = g
    o, s = chunk_nested_gdn2_fwd(**_to_dev(inp), L=L, output_final_state=True,
                                 path="simt")
    assert last_path() == "simt"
    ro, rs = _oracle(inp, L)
    assert rel_err(_np(o), ro) < FP32_REL
    assert rel_err(_np(s), rs) < FP32_REL


def test_l1_reduces_to_level_zero():
    inp = op_inputs(2, 256, 2, 64, 64, 1, 16, firing_intervals=(1,))
    L = inp.pop("L")
    o, s = chunk_nested_gdn2(**_to_dev(inp), L=L, output_final_state=True)
    ro, rs = _oracle(inp, L)
    assert rel_err(_np(o), ro) < FP32_REL
    assert rel_err(_np(s), rs) < FP32_REL


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_low_precision_inputs(dtype):
    inp = op_inputs(1, 256, 2, 64, 64, 3, 16, firing_intervals=(1, 2, 4), dtype=dtype)
    L = inp.pop("L")
    o, s = chunk_nested_gdn2(**_to_dev(inp), L=L, output_final_state=True)
    assert o.dtype == dtype and s.dtype == torch.float32
    ro, rs = _oracle(inp, L)
    assert rel_err(_np(o), ro) < LOWP_REL
    assert rel_err(_np(s), rs) < LOWP_REL


def test_broadcast_gates_match_dense():
    """Scalar-per-head gates passed as stride-0 views give the same result as
    the materialised tensors."""
    kw = dict(dtype=torch.float32, seed=3)
    dense = config_inputs(1, 256, 2, 64, 64, 2, 16, (1, 2), **kw)
    bcast = config_inputs(1, 256, 2, 64, 64, 2, 16, (1, 2), dense_gates=False, **kw)
    assert bcast["b"].stride(-1) == 0
    L = dense.pop("L")
    bcast.pop("L")
    o1, s1 = chunk_nested_gdn2(**_to_dev(dense), L=L, output_final_state=True)
    o2, s2 = chunk_nested_gdn2(**_to_dev(bcast), L=L, output_final_state=True)
    assert torch.equal(o1, o2) and torch.equal(s1, s2)


def test_config0_full_size_fp32():
    """BASELINE config 0 at its full size, fp32 parity at 1e-4."""
    inp = config_inputs(1, 1024, 4, 64, 64, 2, 64, (1, 4), dtype=torch.float32)
    L = inp.pop("L")
    o, s = chunk_nested_gdn2(**_to_dev(inp), L=L, output_final_state=True)
    ro, rs = _oracle(inp, L)
    assert rel_err(_np(o), ro) < FP32_REL
    assert rel_err(_np(s), rs) < FP32_REL


@pytest.mark.parametrize("promotion", ["learned", "merge"])
def test_prefill_then_step_matches_one_pass(promotion):
    """test_chunk.py:161-197: the op's final state hands off to the token step."""
    B, T, H, K, V, L, N, prefill = 1, 256, 2, 64, 64, 3, 16, 128
    inp = op_inputs(B, T, H, K, V, L, N, firing_intervals=(1, 2, 4))
    inp.pop("L")
    dev = _to_dev(inp)
    kw = dict(L=L, promotion=promotion)
    o_full, s_full = chunk_nested_gdn2(**dev, output_final_state=True, **kw)
    per_token = ("q", "k", "v", "g", "b", "w", "mix_weights")
    pre = {n: (t[:, :prefill] if n in per_token else t) for n, t in dev.items()}
    o_pre, state = chunk_nested_gdn2(**pre, output_final_state=True, **kw)
    state = _np(state).astype(np.float64)
    outs = [_np(o_pre)]
    a = {n: _np(t) if torch.is_tensor(t) else t for n, t in inp.items()}
    for t in range(prefill, T):
        o_t, state = oracle.step(*(a[n][:, t] for n in per_token), state, t,
                                 a["query_banks"], a["key_projections"], a["b_projections"],
                                 a["w_projections"], a["g_projections"],
                                 a["n_queries_per_level"], a["firing_intervals"], L,
                                 promotion=promotion)
        outs.append(o_t[:, None])
    assert rel_err(np.concatenate(outs, 1), _np(o_full)) < FP32_REL
    assert rel_err(state, _np(s_full)) < FP32_REL


def test_repeatable_bit_exact():
    inp = op_inputs(1, 256, 2, 64, 64, 3, 16, firing_intervals=(1, 2, 4))
    L = inp.pop("L")
    dev = _to_dev(inp)
    o1, s1 = chunk_nested_gdn2(**dev, L=L, output_final_state=True)
    o2, s2 = chunk_nested_gdn2(**dev, L=L, output_final_state=True)
    assert torch.equal(o1, o2) and torch.equal(s1, s2)


def test_backward_reaches_only_differentiable_inputs():
    """Autograd through the op: q gets a gradient, the int schedule tensors
    none (the backward's parity is tests/test_bwd_gpu.py)."""
    inp = op_inputs(1, 128, 1, 64, 64, 2, 16, firing_intervals=(1, 2))
    L = inp.pop("L")
    dev = _to_dev(inp)
    dev["q"].requires_grad_(True)
    o, _ = chunk_nested_gdn2(**dev, L=L)
    o.sum().backward()
    assert dev["q"].grad is not None and torch.isfinite(dev["q"].grad).all()
    assert dev["q"].grad.shape == dev["q"].shape
