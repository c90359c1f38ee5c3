"""update_state_bwd (ngdn2_update_state_bwd) on the GPU against autograd
through the torch oracle's write scan in float64 (oracle/naive_torch.py,
pinned to autograd through the reference's own scan by
tests/test_oracle_bwd.py), following tests/ops/test_update_bwd.py: the
reference's cases with and without an initial state, block_v invariance,
broadcast identity keys, and the merge arm's identity keys. Bar: 1e-3 of
each gradient's scale (fp32 on CUDA cores; the reference's TF32 kernel is
held to rtol 2e-2, test_update_bwd.py:25)."""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from _util import GOLDEN, rel_err
from nested_recurrent_memory_b200 import update_state, update_state_bwd
from test_oracle_bwd import update_oracle_grads

pytestmark = pytest.mark.gpu

NAMES = ("keys", "values", "g", "b", "w")
BWD_REL = 1e-3


def _inputs(B, NF, H, K, V, N, seed=0, identity_keys=False):
    """test_update_bwd.py's recipe (_update_ref.py:16-31), seeded on the CPU."""
    gen = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=gen)  # noqa: E731
    keys = (torch.eye(K).expand(B, NF, H, K, K) if identity_keys
            else F.normalize(r(B, NF, H, N, K), dim=-1))
    return {"keys": keys, "values": r(B, NF, H, N, V) * V ** -0.5,
            "g": -F.softplus(r(B, NF, H, K)), "b": torch.sigmoid(r(B, NF, H, N, K)),
            "w": torch.sigmoid(r(B, NF, H, N, V))}


def _run(inp, NG, init, d_states, d_final, block_v=16):
    dev = {n: (t.cuda() if n != "keys" or t.stride(0) != 0 else
               torch.eye(t.shape[-1], device="cuda").expand(t.shape)) for n, t in inp.items()}
    states, _ = update_state(**dev, n_groups=NG,
                             initial_state=init.cuda() if init is not None else None)
    out = update_state_bwd(states=states, **dev, d_states=d_states.cuda(),
                           d_final=d_final.cuda(), has_init=init is not None, block_v=block_v)
    torch.cuda.synchronize()
    return {k: v.cpu() for k, v in out.items()}


def _case(B, NG, NF, H, K, V, N, with_init, seed=0, identity_keys=False):
    inp = _inputs(B, NF, H, K, V, N, seed=seed, identity_keys=identity_keys)
    gen = torch.Generator().manual_seed(seed + 1)
    init = torch.randn(B, H, K, V, generator=gen) * K ** -0.5 if with_init else None
    d_states = torch.randn(B, NG, H, K, V, generator=gen)
    d_final = torch.randn(B, H, K, V, generator=gen)
    return inp, init, d_states, d_final


def _oracle(inp, NG, init, d_states, d_final):
    d = {n: t.contiguous().numpy() for n, t in inp.items()}
    d.update(n_groups=NG, d_states=d_states.numpy(), d_final=d_final.numpy())
    if init is not None:
        d["initial_state"] = init.numpy()
    return update_oracle_grads(d)[2]


CASES = [(1, 4, 4, 2, 16, 32, 16), (2, 5, 4, 1, 16, 16, 16), (1, 3, 3, 2, 32, 32, 32),
         (1, 3, 2, 1, 128, 128, 64)]


@pytest.mark.parametrize("with_init", [False, True])
@pytest.mark.parametrize(("B", "NG", "NF", "H", "K", "V", "N"), CASES)
def test_matches_autograd(B, NG, NF, H, K, V, N, with_init):
    inp, init, ds, dfin = _case(B, NG, NF, H, K, V, N, with_init, seed=B + NG + K)
    got = _run(inp, NG, init, ds, dfin)
    ref = _oracle(inp, NG, init, ds, dfin)
    for n in NAMES:
        assert rel_err(got["d" + n].numpy(), ref[n]) < BWD_REL, n
    if with_init:
        assert rel_err(got["dinit"].numpy(), ref["initial_state"]) < BWD_REL


def test_matches_reference_golden():
    d = dict(np.load(GOLDEN / "bwdupd_scan.npz"))
    inp = {n: torch.tensor(d[n], dtype=torch.float32) for n in NAMES}
    got = _run(inp, int(d["n_groups"]), torch.tensor(d["initial_state"], dtype=torch.float32),
               torch.tensor(d["d_states"], dtype=torch.float32),
               torch.tensor(d["d_final"], dtype=torch.float32))
    for n in NAMES:
        assert rel_err(got["d" + n].numpy(), d[f"grad_{n}"]) < BWD_REL, n
    assert rel_err(got["dinit"].numpy(), d["grad_initial_state"]) < BWD_REL


@pytest.mark.parametrize("block_v", [16, 32, 64])
def test_block_v_does_not_change_the_gradients(block_v):
    inp, init, ds, dfin = _case(2, 4, 4, 2, 16, 64, 16, False, seed=3)
    ref = _run(inp, 4, init, ds, dfin, block_v=16)
    got = _run(inp, 4, init, ds, dfin, block_v=block_v)
    for n in NAMES:
        assert torch.equal(got["d" + n], ref["d" + n]), n


def test_broadcast_identity_keys_match_a_materialized_one():
    inp, init, ds, dfin = _case(2, 4, 4, 2, 16, 32, 16, False, seed=5, identity_keys=True)
    dense = dict(inp, keys=inp["keys"].contiguous())
    a = _run(inp, 4, init, ds, dfin)
    c = _run(dense, 4, init, ds, dfin)
    for n in NAMES:
        assert torch.equal(a["d" + n], c["d" + n]), n


def test_identity_keys_gradients_match_autograd():
    """Merge's keys carry no gradient path; the other four must be right."""
    inp, init, ds, dfin = _case(2, 4, 4, 2, 16, 32, 16, False, seed=7, identity_keys=True)
    got = _run(inp, 4, init, ds, dfin)
    ref = _oracle(dict(inp, keys=inp["keys"].contiguous()), 4, init, ds, dfin)
    for n in ("values", "g", "b", "w"):
        assert rel_err(got["d" + n].numpy(), ref[n]) < BWD_REL, n


@pytest.mark.parametrize(("kw", "msg"), [
    (dict(N=24), "power of two"), (dict(block_v=24), "block_v"),
    (dict(V=48, block_v=32), "divisible"), (dict(NG=7), "inconsistent"),
])
def test_errors_match_reference(kw, msg):
    B, NG, NF, H, K, V, N = 1, 4, 4, 1, 16, kw.get("V", 32), kw.get("N", 16)
    NG = kw.get("NG", NG)
    inp = _inputs(B, NF, H, K, V, N)
    dev = {n: t.cuda() for n, t in inp.items()}
    states = torch.zeros(B, NG, H, K, V, device="cuda")
    with pytest.raises(ValueError, match=msg):
        update_state_bwd(states=states, **dev, d_states=torch.zeros_like(states),
                         d_final=torch.zeros(B, H, K, V, device="cuda"),
                         block_v=kw.get("block_v", 16))
