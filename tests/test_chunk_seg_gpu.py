"""The level-segmented tensor-core family (path "tc_seg", csrc/seg.cu)
against the CPU oracle: bf16 inputs at K = V = 128, parity bar 2e-2
(max |got - ref| / max |ref|) on outputs and final states.

Each level runs as a segmented scan (compose, combine, replay) with its
step records from the chunk prep (level 0) or from the probe of the level
below (levels >= 1), so the cases cover every way a level's schedule can
look: several segments and one, a level that never fires, firing intervals
that do not divide one another, a ragged last chunk, an initial state, both
promotion arms, 64 and 128 pairs per firing, and the long-context shape
(L = 4, firing 1/4/16/64, m = 128) up to T = 65536."""

import numpy as np
import pytest
import torch

import oracle
from _util import LOWP_REL, OP_ARGS, rel_err
from nested_recurrent_memory_b200 import FwdCall, check_status
from nested_recurrent_memory_b200.synthetic import config_inputs, op_inputs

pytestmark = pytest.mark.gpu


def _dev(inp):
    return {k: (v.cuda() if torch.is_tensor(v) and v.is_floating_point() else v)
            for k, v in inp.items()}


def _np(t):
    return t.detach().float().cpu().numpy()


def _oracle(inp, L, promotion="learned", initial_state=None):
    a = {k: (_np(v) if torch.is_tensor(v) else v) for k, v in inp.items() if k in OP_ARGS}
    init = _np(initial_state) if initial_state is not None else None
    return oracle.chunk_forward(**a, L=L, initial_state=init, output_final_state=True,
                                promotion=promotion)


def _run(inp, L, path="tc_seg", **kw):
    call = FwdCall(**_dev(inp), L=L, path=path, **kw)
    o, s = call.launch()
    call.check()
    assert call.path == path
    return o, s


def _check(inp, L, promotion="learned", initial_state=None, label=""):
    o, s = _run(inp, L, promotion=promotion, initial_state=initial_state)
    ro, rs = _oracle(inp, L, promotion, initial_state)
    eo, es = rel_err(_np(o), ro), rel_err(_np(s), rs)
    print(f"tc_seg {label}: o rel {eo:.2e}, final rel {es:.2e}")
    assert eo < LOWP_REL and es < LOWP_REL, (eo, es)


@pytest.mark.parametrize("promotion", ["learned", "merge"])
@pytest.mark.parametrize(("L", "firing", "T", "m"), [
    (1, (1,), 320, 64),
    (2, (1, 2), 256, 64),
    (3, (1, 2, 4), 640, 64),
    (3, (1, 4, 16), 1024, 64),
    (4, (1, 2, 4, 8), 1088, 128),
    (4, (1, 4, 16, 64), 4096, 128),
])
def test_config_recipe(L, firing, T, m, promotion):
    inp = config_inputs(1, T, 2, 128, 128, L, m, firing, dtype=torch.bfloat16, seed=31,
                        gate_proj_std=128 ** -0.5)
    inp.pop("L")
    _check(inp, L, promotion, label=f"L{L} f{firing} T{T} m{m} {promotion}")


@pytest.mark.parametrize(("T", "firing", "nq"), [
    (100, (1, 1, 2), (16, 32)),        # one partial chunk: every level fires on it
    (64 * 9 + 17, (1, 4, 16), (64, 64)),   # level 2 never fires
    (64 * 33, (1, 3, 4), (32, 16)),    # intervals that do not nest
])
def test_schedules_and_ragged_t(T, firing, nq):
    inp = op_inputs(1, T, 2, 128, 128, 3, 64, firing_intervals=firing, n_queries_per_level=nq,
                    dtype=torch.bfloat16, seed=32)
    inp.pop("L")
    _check(inp, 3, label=f"T{T} f{firing} nq{nq}")


@pytest.mark.parametrize("promotion", ["learned", "merge"])
def test_initial_state(promotion):
    inp = config_inputs(1, 1280, 2, 128, 128, 3, 64, (1, 2, 8), dtype=torch.bfloat16, seed=33,
                        gate_proj_std=128 ** -0.5)
    inp.pop("L")
    init = torch.randn(1, 2, 3, 128, 128, generator=torch.Generator().manual_seed(34)) * 0.1
    _check(inp, 3, promotion, initial_state=init.cuda(), label=f"init {promotion}")


def test_fused_and_segmented_agree():
    """Same inputs through both tensor-core families (L = 3)."""
    inp = config_inputs(2, 1024, 4, 128, 128, 3, 64, (1, 4, 16), dtype=torch.bfloat16, seed=35,
                        gate_proj_std=128 ** -0.5)
    inp.pop("L")
    o1, s1 = _run(inp, 3, path="tc")
    o2, s2 = _run(inp, 3, path="tc_seg")
    assert rel_err(_np(o2), _np(o1)) < LOWP_REL
    assert rel_err(_np(s2), _np(s1)) < LOWP_REL


def test_head_subset_reproduces_full_run():
    """Different (batch, head) counts give different segment splits; a run
    on two of eight heads must agree with those heads of the full run within
    the path's tolerance (the per-head results do not depend on how the
    sequence was cut)."""
    inp = config_inputs(1, 4096, 8, 128, 128, 4, 128, (1, 4, 16, 64), dtype=torch.bfloat16,
                        seed=36, gate_proj_std=128 ** -0.5)
    inp.pop("L")
    o, s = _run(inp, 4)
    per_token = ("q", "k", "v", "g", "b", "w", "mix_weights")
    sub = {k: (v[:, :, 2:4] if k in per_token else v[:, 2:4] if k.endswith(("banks", "projections")) else v)
           for k, v in inp.items()}
    so, ss = _run({k: (v.contiguous() if torch.is_tensor(v) else v) for k, v in sub.items()}, 4)
    assert rel_err(_np(so), _np(o[:, :, 2:4])) < LOWP_REL
    assert rel_err(_np(ss), _np(s[:, 2:4])) < LOWP_REL


@pytest.mark.parametrize("T", [8192, 65536])
def test_long_context_shape(T):
    """The long-context configuration's levels (L = 4, firing 1/4/16/64,
    m = 128) at T = 8192 on two heads and at its full T = 65536 on one head:
    1024 chunks, 256 / 64 / 16 firings, bf16 operand error compounding
    across the whole sequence. The bar stays 2e-2."""
    H = 2 if T <= 8192 else 1
    inp = config_inputs(1, T, H, 128, 128, 4, 128, (1, 4, 16, 64), dtype=torch.bfloat16, seed=37,
                        gate_proj_std=128 ** -0.5)
    inp.pop("L")
    _check(inp, 4, label=f"long T{T} H{H}")


def test_no_wait_timeouts_at_occupancy():
    """A full-width launch (many segments and CTAs at once) completes with a
    clear status word, three times over, with the same bits each time."""
    inp = config_inputs(1, 8192, 4, 128, 128, 4, 128, (1, 4, 16, 64), dtype=torch.bfloat16, seed=38)
    inp.pop("L")
    call = FwdCall(**_dev(inp), L=4, path="tc_seg")
    ref = None
    for _ in range(3):
        o, s = call.launch()
        check_status()
        if ref is None:
            ref = (o.clone(), s.clone())
        else:
            assert torch.equal(o, ref[0]) and torch.equal(s, ref[1])


def test_query_layouts_and_fp16_agree():
    """The upper-level read kernel takes q through a tensor map in either
    (head, level) order -- [B, T, H, L, K] or the layer's transposed
    [B, T, L, H, K] view -- or, for a q whose rows do not collapse (a view
    cut from a longer sequence), with plain loads. Same values, same bits
    out. fp16 inputs (converted to bf16 tiles in the read kernel) meet the
    oracle at the same bar."""
    inp = config_inputs(1, 1024, 2, 128, 128, 4, 128, (1, 2, 4, 8), dtype=torch.bfloat16, seed=40,
                        gate_proj_std=128 ** -0.5)
    inp.pop("L")
    d = _dev(inp)
    q = d["q"]
    longer = torch.zeros(1, 1100, *q.shape[2:], dtype=q.dtype, device="cuda")
    longer[:, :1024] = q
    outs = []
    for qq in (q, q.transpose(2, 3).contiguous().transpose(2, 3), longer[:, :1024]):
        call = FwdCall(**dict(d, q=qq), L=4, path="tc_seg")
        outs.append([t.clone() for t in call.launch()])
        call.check()
    for o, s in outs[1:]:
        assert torch.equal(o, outs[0][0]) and torch.equal(s, outs[0][1])
    half = config_inputs(1, 1024, 2, 128, 128, 4, 128, (1, 2, 4, 8), dtype=torch.float16, seed=40,
                         gate_proj_std=128 ** -0.5)
    half.pop("L")
    _check(half, 4, label="fp16 L4")


def test_broadcast_gates_match_dense():
    """Stride-0 broadcast gates (b, w, g views of per-token scalars) give the
    same bits as the materialised tensors."""
    kw = dict(dtype=torch.bfloat16, seed=41)
    dense = config_inputs(1, 2048, 2, 128, 128, 3, 64, (1, 4, 16), **kw)
    bcast = config_inputs(1, 2048, 2, 128, 128, 3, 64, (1, 4, 16), dense_gates=False, **kw)
    dense.pop("L")
    bcast.pop("L")
    o1, s1 = _run(dense, 3)
    o2, s2 = _run(bcast, 3)
    assert torch.equal(o1, o2) and torch.equal(s1, s2)
