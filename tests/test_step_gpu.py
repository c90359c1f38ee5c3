"""The one-token decode step (naive.py:42-134, naive_step_nested_gdn2) on the
GPU against the CPU oracle's token step: fp32 inputs at 1e-4, 16-bit inputs
at 2e-2 (max |got - ref| / max |ref|), with rows at different positions so
that some fire and some do not, both promotion arms, in-place states, and
the layer's prefill-then-step hand-off (nested_gdn2.py:204-224)."""

import numpy as np
import pytest
import torch

import oracle
from _util import FP32_REL, LOWP_REL, rel_err
from nested_recurrent_memory_b200 import chunk_nested_gdn2, step_nested_gdn2
from nested_recurrent_memory_b200.synthetic import config_inputs, op_inputs

pytestmark = pytest.mark.gpu

PER_TOKEN = ("q", "k", "v", "g", "b", "w", "mix_weights")
WEIGHTS = ("query_banks", "key_projections", "b_projections", "w_projections", "g_projections",
           "n_queries_per_level", "firing_intervals")


def _np(t):
    return t.detach().float().cpu().numpy()


def _token(inp, t):
    return {n: inp[n][:, t] for n in PER_TOKEN}


def _run_both(inp, t, state, position, L, promotion, **kw):
    tok = _token(inp, t)
    dev = {n: x.cuda() for n, x in tok.items()}
    wts = {n: inp[n].cuda() if inp[n].is_floating_point() else inp[n] for n in WEIGHTS}
    pos_dev = torch.as_tensor(position).cuda() if not isinstance(position, int) else position
    o, s = step_nested_gdn2(**dev, state=state.cuda(), position=pos_dev, **wts, L=L,
                            promotion=promotion, **kw)
    torch.cuda.synchronize()
    a = {n: _np(x) for n, x in tok.items()}
    ro, rs = oracle.step(*(a[n] for n in PER_TOKEN), _np(state).astype(np.float64),
                         np.asarray(position), *(_np(inp[n]) if inp[n].is_floating_point()
                                                 else inp[n].numpy() for n in WEIGHTS[:5]),
                         inp["n_queries_per_level"], inp["firing_intervals"], L,
                         promotion=promotion)
    return o, s, ro, rs


@pytest.mark.parametrize("promotion", ["learned", "merge"])
def test_rows_at_different_positions_fp32(promotion):
    """Rows 0..3 at positions 62, 63, 127, 255 with firing (1, 2, 4): row 0
    does not fire, row 1 fires level 1, rows 2 and 3 fire levels 1 and 2."""
    inp = op_inputs(4, 8, 2, 64, 64, 3, 16, firing_intervals=(1, 2, 4))
    L = inp.pop("L")
    state = torch.randn(4, 2, L, 64, 64, generator=torch.Generator().manual_seed(2)) * 0.2
    o, s, ro, rs = _run_both(inp, 3, state, [62, 63, 127, 255], L, promotion)
    assert o.dtype == torch.float32
    assert rel_err(_np(o), ro) < FP32_REL
    assert rel_err(_np(s), rs) < FP32_REL


def test_bf16_inputs_k128_scalar_position():
    inp = config_inputs(2, 4, 2, 128, 128, 3, 64, (1, 1, 2), dtype=torch.bfloat16, seed=4,
                        gate_proj_std=128 ** -0.5)
    L = inp.pop("L")
    state = torch.randn(2, 2, L, 128, 128, generator=torch.Generator().manual_seed(3)) * 0.05
    o, s, ro, rs = _run_both(inp, 1, state, 127, L, "learned")  # fires levels 1 and 2
    assert o.dtype == torch.bfloat16
    assert rel_err(_np(o), ro) < LOWP_REL
    assert rel_err(_np(s), rs) < LOWP_REL


def test_no_firing_and_in_place():
    inp = op_inputs(2, 4, 2, 64, 64, 2, 16, firing_intervals=(1, 1))
    L = inp.pop("L")
    state = (torch.randn(2, 2, L, 64, 64, generator=torch.Generator().manual_seed(5)) * 0.2).cuda()
    dev = {n: x.cuda() for n, x in _token(inp, 0).items()}
    wts = {n: inp[n].cuda() if inp[n].is_floating_point() else inp[n] for n in WEIGHTS}
    o1, s1 = step_nested_gdn2(**dev, state=state, position=10, **wts, L=L)
    s_in = state.clone()
    o2, s2 = step_nested_gdn2(**dev, state=s_in, position=10, **wts, L=L, out_state=s_in)
    torch.cuda.synchronize()
    assert s2.data_ptr() == s_in.data_ptr()
    assert torch.equal(o1, o2) and torch.equal(s1, s2)
    assert torch.equal(s1[:, :, 1], state[:, :, 1])  # no firing: level 1 unchanged


@pytest.mark.parametrize("promotion", ["learned", "merge"])
def test_prefill_then_cuda_steps_match_one_pass(promotion):
    """The layer's hand-off (nested_gdn2.py:204-224): the chunked op over a
    whole-chunk prefix, then one step per token, equals the chunked op over
    the whole sequence when it ends on a chunk boundary."""
    B, T, H, K, V, L, N, prefill = 1, 192, 2, 64, 64, 3, 16, 128
    inp = op_inputs(B, T, H, K, V, L, N, firing_intervals=(1, 1, 3))
    inp.pop("L")
    dev = {n: (x.cuda() if torch.is_tensor(x) and x.is_floating_point() else x)
           for n, x in inp.items()}
    o_full, s_full = chunk_nested_gdn2(**dev, L=L, output_final_state=True, promotion=promotion)
    pre = {n: (x[:, :prefill] if n in PER_TOKEN else x) for n, x in dev.items()}
    o_pre, state = chunk_nested_gdn2(**pre, L=L, output_final_state=True, promotion=promotion)
    wts = {n: dev[n] for n in WEIGHTS}
    outs = [o_pre]
    for t in range(prefill, T):
        o_t, state = step_nested_gdn2(**{n: dev[n][:, t] for n in PER_TOKEN}, state=state,
                                      position=t, **wts, L=L, promotion=promotion)
        outs.append(o_t[:, None])
    torch.cuda.synchronize()
    assert rel_err(_np(torch.cat(outs, 1)), _np(o_full)) < FP32_REL
    assert rel_err(_np(state), _np(s_full)) < FP32_REL
