"""HostPipeline (nested_recurrent_memory_b200/host.py): batches in pinned host
memory through the op with uploads, compute and downloads on three streams.
Its outputs must be bit-identical to calling chunk_nested_gdn2 on the same
batch directly (same kernels, same inputs), for every batch of a run in
which the two device buffer slots are each reused."""

import pytest
import torch

from nested_recurrent_memory_b200 import HostPipeline, chunk_nested_gdn2
from nested_recurrent_memory_b200.synthetic import config_inputs

pytestmark = pytest.mark.gpu


def _batch(seed):
    inp = config_inputs(2, 320, 2, 128, 128, 3, 64, (1, 2, 4), dtype=torch.bfloat16, seed=seed)
    L = inp.pop("L")
    tensors = {k: v.pin_memory() for k, v in inp.items() if torch.is_tensor(v) and v.is_floating_point()}
    rest = {k: v for k, v in inp.items() if k not in tensors}
    return tensors, rest, L


def test_pipeline_matches_direct_calls():
    batches = [_batch(seed) for seed in range(5)]
    _, rest, L = batches[0]
    pipe = HostPipeline(batches[0][0], L=L, **rest)
    got = []
    handles = []
    for tensors, _, _ in batches:
        handles.append(pipe.submit(tensors))
        if len(handles) == 2:
            # A slot's host outputs are valid until the slot is reused.
            o, s = pipe.result(handles.pop(0))
            got.append((o.clone(), s.clone()))
    for h in handles:
        o, s = pipe.result(h)
        got.append((o.clone(), s.clone()))
    for (tensors, rest_b, Lb), (o, s) in zip(batches, got):
        dev = {k: v.cuda() for k, v in tensors.items()}
        ro, rs = chunk_nested_gdn2(**dev, L=Lb, output_final_state=True, **rest_b)
        torch.cuda.synchronize()
        assert torch.equal(o, ro.cpu())
        assert torch.equal(s, rs.cpu())


def test_pipeline_rejects_pageable_inputs():
    tensors, rest, L = _batch(0)
    tensors["q"] = tensors["q"].clone()  # not pinned
    with pytest.raises(ValueError, match="pinned"):
        HostPipeline(tensors, L=L, **rest)


def test_pipeline_uploads_broadcast_gates_compactly():
    # b, w, g as stride-0 views of pinned per-token, per-head scalars: the
    # pipeline uploads the scalars only and expands them on the device; the
    # results equal the direct call with the dense gates, bit for bit.
    from nested_recurrent_memory_b200.host import compact_view
    inp = config_inputs(2, 320, 2, 128, 128, 3, 64, (1, 2, 4), dtype=torch.bfloat16, seed=7,
                        dense_gates=False)
    L = inp.pop("L")
    tensors = {k: (compact_view(v).contiguous().pin_memory().expand(v.shape)
                   if v.stride()[-1] == 0 else v.contiguous().pin_memory())
               for k, v in inp.items() if torch.is_tensor(v) and v.is_floating_point()}
    rest = {k: v for k, v in inp.items() if k not in tensors}
    for k in ("b", "w", "g"):
        assert tensors[k].stride()[-1] == 0 and tensors[k].is_pinned()
    pipe = HostPipeline(tensors, L=L, **rest)
    for k in ("b", "w", "g"):
        assert pipe.slots[0][k].numel() == tensors[k].numel() // tensors[k].shape[-1]
    o, s = pipe.result(pipe.submit(tensors))
    dense = {k: v.contiguous().cuda() for k, v in tensors.items()}
    ro, rs = chunk_nested_gdn2(**dense, L=L, output_final_state=True, **rest)
    torch.cuda.synchronize()
    assert torch.equal(o, ro.cpu())
    assert torch.equal(s, rs.cpu())
