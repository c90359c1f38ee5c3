"""The CPU oracle (oracle/naive_np.py) pinned against the reference's own
outputs (tests/golden/*.npz, written by tests/golden/make_golden.py from the
reference's naive.py and probe.py), plus the properties the reference tests
hold its oracle to. CPU only."""

import numpy as np
import pytest

import oracle
from _util import GOLDEN, chunk_case_names, load_case, rel_err

# float64 oracle against the fp32 reference: only the reference's rounding differs.
PIN = 1e-5


@pytest.mark.parametrize("name", chunk_case_names())
def test_chunk_forward_matches_reference(name):
    args, extra, d = load_case(name)
    o, s = oracle.chunk_forward(**args, L=extra["L"], initial_state=extra["initial_state"],
                                output_final_state=True, promotion=extra["promotion"])
    assert rel_err(o, d["out_o"]) < PIN
    assert rel_err(s, d["out_final"]) < PIN


@pytest.mark.parametrize("name", [n for n in chunk_case_names() if n.startswith("chunk_")])
def test_recurrent_forward_matches_reference(name):
    args, extra, d = load_case(name)
    o, s = oracle.recurrent_forward(**args, L=extra["L"], initial_state=extra["initial_state"],
                                    output_final_state=True, chunk_size=64,
                                    promotion=extra["promotion"])
    assert rel_err(o, d["out_rec_o"]) < PIN
    assert rel_err(s, d["out_rec_final"]) < PIN


@pytest.mark.parametrize("name", [n for n in chunk_case_names()
                                  if n.startswith("chunk_") and "ragged" not in n])
def test_chunk_equals_recurrent(name):
    """test_naive.py:398-455: the chunkwise form equals the token recurrence
    when T is a whole number of chunks."""
    args, extra, _ = load_case(name)
    kw = dict(L=extra["L"], initial_state=extra["initial_state"], output_final_state=True,
              promotion=extra["promotion"])
    o1, s1 = oracle.chunk_forward(**args, **kw)
    o2, s2 = oracle.recurrent_forward(**args, chunk_size=64, **kw)
    assert rel_err(o1, o2) < 1e-10
    assert rel_err(s1, s2) < 1e-10


def test_ragged_last_chunk_fires_in_chunk_form_only():
    """A partial last chunk fires in the chunkwise form (chunk.py:26-36,
    nested_gdn2.py:197-200) but not token by token, so outputs agree and the
    upper levels' final states differ."""
    args, extra, d = load_case("chunk_ragged_t100")
    assert rel_err(d["out_o"], d["out_rec_o"]) < 1e-5
    assert rel_err(d["out_final"][:, :, 1:], d["out_rec_final"][:, :, 1:]) > 1e-3
    assert rel_err(d["out_final"][:, :, 0], d["out_rec_final"][:, :, 0]) < 1e-5


def test_update_scan_matches_reference():
    d = dict(np.load(GOLDEN / "update_scan.npz"))
    st, fi = oracle.update_scan(d["keys"], d["values"], d["g"], d["b"], d["w"],
                                int(d["n_groups"]), d["initial_state"])
    np.testing.assert_allclose(st, d["out_states"], rtol=0, atol=1e-12)
    np.testing.assert_allclose(fi, d["out_final"], rtol=0, atol=1e-12)


@pytest.mark.parametrize("arm", ["learned", "merge"])
def test_probes_match_reference(arm):
    d = dict(np.load(GOLDEN / "probes.npz"))
    res = oracle.naive_np.PROBES[arm](d["state_below"].astype(np.float64), d["query_bank"],
                                      d["key_proj"], d["b_proj"], d["w_proj"], d["g_proj"],
                                      int(d["n_queries"]))
    for got, nm in zip(res, ("keys", "values", "b", "w", "g")):
        np.testing.assert_allclose(got, d[f"out_{arm}_{nm}"], rtol=0, atol=1e-6)


def test_update_is_pair_order_invariant():
    """test_update_fwd.py:50-60: all pairs act on the pre-firing state."""
    rng = np.random.default_rng(0)
    B, NF, H, K, V, N = 2, 3, 2, 16, 16, 16
    keys = rng.standard_normal((B, NF, H, N, K))
    keys /= np.linalg.norm(keys, axis=-1, keepdims=True)
    vals = rng.standard_normal((B, NF, H, N, V)) / 4
    g = -np.logaddexp(0, rng.standard_normal((B, NF, H, K)))
    b = 1 / (1 + np.exp(-rng.standard_normal((B, NF, H, N, K))))
    w = 1 / (1 + np.exp(-rng.standard_normal((B, NF, H, N, V))))
    perm = rng.permutation(N)
    a = oracle.update_scan(keys, vals, g, b, w, NF)
    c = oracle.update_scan(keys[:, :, :, perm], vals[:, :, :, perm], g,
                           b[:, :, :, perm], w[:, :, :, perm], NF)
    for x, y in zip(a, c):
        np.testing.assert_allclose(x, y, rtol=0, atol=1e-12)


def test_gate_offsets_with_zero_projections():
    """test_probe.py:66-77: zero projections give exactly the offsets."""
    rng = np.random.default_rng(1)
    S = rng.standard_normal((1, 2, 16, 16))
    z = np.zeros((2, 16, 16))
    _, _, b, w, g = oracle.probe_learned(S, rng.standard_normal((2, 16, 16)),
                                         rng.standard_normal((2, 16, 16)), z, z, z, 16)
    np.testing.assert_allclose(b, 1 / (1 + np.exp(4.0)), rtol=1e-15)
    np.testing.assert_allclose(w, 0.5, rtol=1e-15)
    np.testing.assert_allclose(g, -np.log1p(np.exp(-4.0)), rtol=1e-15)


def test_schedule_arithmetic():
    """chunk.py:26-55."""
    assert oracle.n_groups(5, 2) == 3 and oracle.n_firings(5, 2) == 2
    assert oracle.n_groups(4, 4) == 1 and oracle.n_firings(4, 4) == 1
    assert oracle.source_index(1, 4, 8) == [4, 8]
    assert oracle.source_index(4, 16, 32) == [4, 8]
