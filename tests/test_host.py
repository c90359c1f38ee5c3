"""Host-side behaviour of the reference-facing API that needs no GPU: the
reference's ValueError messages (raised before any device work), loud
failure on CPU tensors, schedule helpers and the input recipes."""

import pytest
import torch
import torch.nn.functional as F

from nested_recurrent_memory_b200 import (chunk_nested_gdn2, chunk_nested_gdn2_fwd, n_firings,
                                          n_groups, update_state)
from nested_recurrent_memory_b200.synthetic import CONFIGS, config_inputs, op_inputs


def _small(L=2, n_queries=None, N=32):
    inp = op_inputs(1, 256, 2, 64, 64, L, N, firing_intervals=[1] + [2] * (L - 1),
                    n_queries_per_level=n_queries)
    L = inp.pop("L")
    return inp, L


@pytest.mark.parametrize("bad_bt", [16, 32, 128])
def test_rejects_non_64_chunk_size(bad_bt):
    inp, L = _small()
    with pytest.raises(ValueError, match="chunk_size must be 64"):
        chunk_nested_gdn2(**inp, L=L, chunk_size=bad_bt)


@pytest.mark.parametrize("bad", [4, 8, 24])
def test_rejects_bad_n_queries(bad):
    inp, L = _small(n_queries=(bad,))
    with pytest.raises(ValueError, match="power of two"):
        chunk_nested_gdn2(**inp, L=L, chunk_size=64)


def test_unknown_promotion_is_a_key_error():
    inp, L = _small()
    with pytest.raises(KeyError):
        chunk_nested_gdn2_fwd(**inp, L=L, promotion="nope")


def test_cpu_tensors_fail_loudly():
    inp, L = _small()
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        chunk_nested_gdn2(**inp, L=L)


def _upd(V=32, N=16):
    gen = torch.Generator().manual_seed(0)
    r = lambda *s: torch.randn(*s, generator=gen)  # noqa: E731
    return dict(keys=F.normalize(r(1, 4, 1, N, 16), dim=-1), values=r(1, 4, 1, N, V),
                g=-F.softplus(r(1, 4, 1, 16)), b=torch.sigmoid(r(1, 4, 1, N, 16)),
                w=torch.sigmoid(r(1, 4, 1, N, V)))


@pytest.mark.parametrize(("V", "N", "n_groups_", "block_v", "match"), [
    (32, 8, 4, 16, "power of two"),
    (32, 16, 4, 8, "block_v"),
    (24, 16, 4, 16, "divisible"),
    (32, 16, 9, 16, "inconsistent"),
])
def test_update_rejects_bad_shapes(V, N, n_groups_, block_v, match):
    """test_update_fwd.py:103-115, same messages."""
    with pytest.raises(ValueError, match=match):
        update_state(**_upd(V, N), n_groups=n_groups_, block_v=block_v)


def test_update_rejects_keys_that_are_not_unit_stride_along_k():
    inp = _upd()
    inp["keys"] = torch.randn(1, 4, 1, 16, 32)[..., ::2]
    with pytest.raises(ValueError, match="unit-stride"):
        update_state(**inp, n_groups=4)


def test_schedule_helpers():
    assert n_groups(128, 4) == 32 and n_firings(128, 4) == 32
    assert n_groups(129, 4) == 33 and n_firings(129, 4) == 32


def test_config_recipe():
    B, T, H, K, V, L, m, firing, dtype = CONFIGS["config0"]
    inp = config_inputs(B, 128, H, K, V, L, m, firing, dtype=dtype)
    torch.testing.assert_close(inp["q"].norm(dim=-1), torch.ones(B, 128, H, L))
    assert torch.equal(inp["b"][..., 0], inp["w"][..., 0])
    assert (inp["g"] < 0).all()
    assert torch.count_nonzero(inp["b_projections"]) == 0
    again = config_inputs(B, 128, H, K, V, L, m, firing, dtype=dtype)
    assert torch.equal(inp["v"], again["v"])


def test_host_pipeline_rejects_pageable_inputs_before_touching_cuda():
    """HostPipeline only takes pinned host batches (its copies are
    asynchronous); a pageable tensor is refused at construction."""
    from nested_recurrent_memory_b200 import HostPipeline
    with pytest.raises(ValueError, match="pinned"):
        HostPipeline({"q": torch.zeros(1, 64, 1, 2, 16)}, L=2)


def test_compact_view_of_broadcast_inputs():
    # The distinct elements of a stride-0 (broadcast) view, as HostPipeline
    # and bench --gates broadcast upload them; a dense tensor is its own.
    from nested_recurrent_memory_b200.host import compact_view
    beta = torch.randn(2, 5, 3)
    b = beta.unsqueeze(-1).expand(2, 5, 3, 64)
    c = compact_view(b)
    assert c.shape == (2, 5, 3, 1) and c.is_contiguous()
    assert torch.equal(c.expand(b.shape), b)
    dense = torch.randn(2, 5, 3, 64)
    assert compact_view(dense) is dense
    inp = config_inputs(1, 128, 2, 64, 64, 2, 16, (1, 2), dtype=torch.float32, dense_gates=False)
    for k in ("b", "w", "g"):
        assert compact_view(inp[k]).numel() == 128 * 2
