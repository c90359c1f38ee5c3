"""update_state (the promotion write scan) against the float64 oracle scan,
mirroring tests/ops/test_update_fwd.py of the reference."""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle
from _util import GOLDEN, rel_err
from nested_recurrent_memory_b200 import update_state

pytestmark = pytest.mark.gpu

# fp32 CUDA-core arithmetic against a float64 scan.
TOL = dict(rtol=1e-4, atol=1e-5)
CONSISTENCY = dict(rtol=1e-5, atol=1e-6)


def _inputs(B, NF, H, K, V, N, *, seed=0, identity_keys=False):
    gen = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=gen)  # noqa: E731
    keys = (torch.eye(K, device="cuda").expand(B, NF, H, K, K) if identity_keys
            else F.normalize(r(B, NF, H, N, K), dim=-1).cuda())
    out = dict(values=r(B, NF, H, N, V) * V ** -0.5,
               g=-F.softplus(r(B, NF, H, K)), b=torch.sigmoid(r(B, NF, H, N, K)),
               w=torch.sigmoid(r(B, NF, H, N, V)))
    return {"keys": keys, **{k: v.cuda() for k, v in out.items()}}


def _scan(inp, NG, init=None):
    a = {k: v.double().cpu().numpy() for k, v in inp.items()}
    return oracle.update_scan(a["keys"], a["values"], a["g"], a["b"], a["w"], NG,
                              None if init is None else init.double().cpu().numpy())


CASES = [(1, 4, 4, 2, 16, 32, 16), (2, 5, 4, 1, 16, 16, 16), (1, 3, 3, 2, 32, 32, 32),
         (1, 4, 4, 2, 128, 128, 64)]


@pytest.mark.parametrize("with_init", [False, True])
@pytest.mark.parametrize(("B", "NG", "NF", "H", "K", "V", "N"), CASES)
def test_matches_oracle_scan(B, NG, NF, H, K, V, N, with_init):
    inp = _inputs(B, NF, H, K, V, N)
    init = torch.randn(B, H, K, V, device="cuda") * K ** -0.5 if with_init else None
    states, final = update_state(**inp, n_groups=NG, initial_state=init)
    rs, rf = _scan(inp, NG, init)
    torch.testing.assert_close(states.double().cpu(), torch.from_numpy(rs), **TOL)
    torch.testing.assert_close(final.double().cpu(), torch.from_numpy(rf), **TOL)


def test_golden_update():
    d = dict(np.load(GOLDEN / "update_scan.npz"))
    inp = {k: torch.from_numpy(d[k]).float().cuda() for k in ("keys", "values", "g", "b", "w")}
    st, fi = update_state(**inp, n_groups=int(d["n_groups"]),
                          initial_state=torch.from_numpy(d["initial_state"]).float().cuda())
    assert rel_err(st.cpu().numpy(), d["out_states"]) < 1e-5
    assert rel_err(fi.cpu().numpy(), d["out_final"]) < 1e-5


def test_pairs_may_be_written_in_any_order():
    inp = _inputs(1, 4, 2, 16, 32, 16)
    perm = torch.randperm(16, generator=torch.Generator().manual_seed(0)).cuda()
    shuffled = {k: (t[:, :, :, perm] if t.dim() == 5 else t) for k, t in inp.items()}
    for a, c in zip(update_state(**inp, n_groups=4), update_state(**shuffled, n_groups=4)):
        torch.testing.assert_close(a, c, **TOL)


def test_broadcast_identity_keys_match_a_materialized_one():
    inp = _inputs(2, 4, 2, 16, 32, 16, identity_keys=True)
    assert inp["keys"].stride()[:3] == (0, 0, 0)
    dense = {**inp, "keys": inp["keys"].contiguous()}
    for a, c in zip(update_state(**inp, n_groups=4), update_state(**dense, n_groups=4)):
        assert torch.equal(a, c)


@pytest.mark.parametrize("block_v", [16, 32, 64])
def test_block_v_does_not_change_the_result(block_v):
    inp = _inputs(2, 4, 2, 16, 64, 16)
    ref = update_state(**inp, n_groups=4, block_v=16)
    got = update_state(**inp, n_groups=4, block_v=block_v)
    for a, c in zip(ref, got):
        torch.testing.assert_close(a, c, **CONSISTENCY)


def test_a_trailing_group_without_a_firing_holds_the_final_state():
    states, final = update_state(**_inputs(2, 4, 2, 16, 32, 16), n_groups=5)
    assert torch.equal(states[:, -1], final)


def test_states_start_at_the_initial_state():
    init = torch.randn(2, 2, 16, 32, device="cuda") * 16 ** -0.5
    states, _ = update_state(**_inputs(2, 4, 2, 16, 32, 16), n_groups=4, initial_state=init)
    torch.testing.assert_close(states[:, 0], init, rtol=0, atol=0)


def test_bf16_pairs():
    inp = {k: v.bfloat16() if k != "g" else v for k, v in _inputs(1, 4, 2, 32, 32, 16).items()}
    states, final = update_state(**inp, n_groups=4)
    rs, rf = _scan({k: v.float() for k, v in inp.items()}, 4)
    assert rel_err(final.cpu().numpy(), rf) < 1e-4
