"""Properties of the CUDA forward that hold at any size, on both kernel
families (CUDA-core fp32 and tensor-core bf16):

* (b, h) independence: every (batch row, head) pair is its own recurrence
  (update_fwd.py:44, 77-80), so a run on a subset of batch rows, or of heads
  with their parameters, reproduces those rows / heads of the full run bit
  for bit. This is what lets the multi-GPU runs shard (b, h) with no
  collective.
* query-pair order: a promotion's update sums over the query-bank pairs
  (naive.py:7-39), so permuting the bank's rows changes only the rounding
  (tests/ops/test_update_fwd.py checks the same of update_state).
"""

import pytest
import torch

from _util import FP32_REL, LOWP_REL, rel_err
from nested_recurrent_memory_b200 import chunk_nested_gdn2
from nested_recurrent_memory_b200.synthetic import config_inputs

pytestmark = pytest.mark.gpu

PARAMS = ("query_banks", "key_projections", "b_projections", "w_projections", "g_projections")
PER_TOKEN = ("q", "k", "v", "g", "b", "w", "mix_weights")


def _case(dtype, K, seed):
    inp = config_inputs(3, 320, 4, K, K, 3, 32, (1, 2, 4), dtype=dtype, seed=seed,
                        gate_proj_std=K ** -0.5)
    L = inp.pop("L")
    dev = {k: (v.cuda() if torch.is_tensor(v) and v.is_floating_point() else v)
           for k, v in inp.items()}
    init = torch.randn(3, 4, L, K, K, generator=torch.Generator().manual_seed(seed)).cuda() * 0.1
    return dev, L, init


def _run(a, L, init, promotion):
    return chunk_nested_gdn2(**a, L=L, initial_state=init, output_final_state=True,
                             promotion=promotion)


FAMILIES = [(torch.float32, 64), (torch.bfloat16, 128)]


@pytest.mark.parametrize("promotion", ["learned", "merge"])
@pytest.mark.parametrize(("dtype", "K"), FAMILIES)
def test_batch_rows_and_heads_are_independent(dtype, K, promotion):
    a, L, init = _case(dtype, K, seed=31)
    o, s = _run(a, L, init, promotion)
    # batch rows 1..2
    sub = {k: (v[1:3] if k in PER_TOKEN else v) for k, v in a.items()}
    o_b, s_b = _run(sub, L, init[1:3].contiguous(), promotion)
    assert torch.equal(o_b, o[1:3])
    assert torch.equal(s_b, s[1:3])
    # heads 1 and 3, with their parameters
    hs = torch.tensor([1, 3], device="cuda")
    sub = {}
    for k, v in a.items():
        if k == "q":
            sub[k] = v.index_select(2, hs).contiguous()
        elif k in PER_TOKEN:
            sub[k] = v.index_select(2, hs).contiguous()
        elif k in PARAMS:
            sub[k] = v.index_select(1, hs).contiguous()
        else:
            sub[k] = v
    o_h, s_h = _run(sub, L, init.index_select(1, hs).contiguous(), promotion)
    assert torch.equal(o_h, o.index_select(2, hs))
    assert torch.equal(s_h, s.index_select(1, hs))


@pytest.mark.parametrize(("dtype", "K"), FAMILIES)
def test_query_pair_order_changes_only_rounding(dtype, K):
    a, L, init = _case(dtype, K, seed=37)
    nq = int(a["n_queries_per_level"][0])
    o, s = _run(a, L, init, "learned")
    perm = torch.randperm(nq, generator=torch.Generator().manual_seed(5)).cuda()
    qb = a["query_banks"].clone()
    qb[:, :, :nq] = a["query_banks"][:, :, :nq].index_select(2, perm)
    o_p, s_p = _run(dict(a, query_banks=qb), L, init, "learned")
    tol = FP32_REL if dtype == torch.float32 else LOWP_REL
    assert rel_err(o_p.float().cpu().numpy(), o.float().cpu().numpy()) < tol
    assert rel_err(s_p.cpu().numpy(), s.cpu().numpy()) < tol
