"""Running the op over batches that live in host memory.

A caller whose inputs arrive in (pinned) host memory -- a data loader
feeding an inference server, say -- pays a host-to-device copy of every
input and a device-to-host copy of the outputs per batch. On B200 those
PCIe copies take far longer than the op itself (config 1: about 39 ms of
uploads and 5 ms of downloads against 2.1 ms of kernels), so the useful
schedule overlaps them: batch k + 1 uploads while batch k runs and
downloads (PCIe moves both directions at once).

``HostPipeline`` does that with two sets of device input buffers and three
CUDA streams (upload, compute, download). Each ``submit`` enqueues one
batch and returns at once; ``result`` waits for a batch's outputs in host
memory. Every batch still uploads all of its inputs and downloads its
outputs: only the ordering across batches changes. The op itself is
``chunk_nested_gdn2``, unchanged.

Inputs given as broadcast views (stride 0 along some dimensions, e.g. gates
that are one scalar per token and head expanded over the head dimension,
which the op reads as such) upload only their distinct elements and are
expanded again on the device.
"""

from __future__ import annotations

import torch

from .ops import chunk_nested_gdn2


def compact_view(t: torch.Tensor) -> torch.Tensor:
    """``t`` restricted to index 0 along its stride-0 dimensions: the
    distinct elements of a broadcast view (``t`` itself when it has none)."""
    if all(st != 0 or n <= 1 for st, n in zip(t.stride(), t.shape)):
        return t
    return t[tuple(slice(0, 1) if (st == 0 and n > 1) else slice(None)
                   for st, n in zip(t.stride(), t.shape))]


class HostPipeline:
    """Double-buffered ``chunk_nested_gdn2`` over host-resident batches.

    ``example`` is a dict of the op's tensor arguments as pinned CPU
    tensors (the shapes and dtypes every batch will have); other keyword
    arguments of the op (``n_queries_per_level``, ``firing_intervals``,
    ``L``, ``promotion`` ...) go in ``op_kwargs`` and are passed through.
    Output buffers are pinned host tensors owned by the pipeline, one pair
    per in-flight slot; ``result(handle)`` returns them after the batch's
    download has finished, and they stay valid until that slot is reused
    two submissions later. An input that is a broadcast view of a pinned
    tensor uploads only its distinct elements (``compact_view``).
    """

    def __init__(self, example: dict, device=None, **op_kwargs):
        self.device = torch.device(device if device is not None else "cuda")
        for k, t in example.items():
            if not t.is_pinned():
                raise ValueError(f"input {k!r} must be a pinned host tensor")
        self.names = list(example)
        self.op_kwargs = op_kwargs
        self.shapes = {k: t.shape for k, t in example.items()}
        self.slots = [{k: torch.empty(compact_view(t).shape, dtype=t.dtype, device=self.device)
                       for k, t in example.items()} for _ in range(2)]
        self.up, self.run, self.down = (torch.cuda.Stream(self.device) for _ in range(3))
        self.freed = [torch.cuda.Event() for _ in range(2)]      # slot inputs no longer read
        self.uploaded = [torch.cuda.Event() for _ in range(2)]
        self.computed = [torch.cuda.Event() for _ in range(2)]
        self.downloaded = [torch.cuda.Event() for _ in range(2)]
        self.out_host = [None, None]
        self.count = 0

    def submit(self, host_inputs: dict):
        """Enqueue one batch (pinned CPU tensors shaped like ``example``);
        returns a handle for ``result``.

        The uploads are asynchronous: they read ``host_inputs`` after this
        call returns. The caller must leave those host tensors unchanged
        until ``wait_uploaded(handle)`` returns (or ``result(handle)``,
        which implies it); refilling one pinned staging buffer right after
        ``submit`` would upload a mix of two batches."""
        s = self.count % 2
        bufs = self.slots[s]
        with torch.cuda.stream(self.up):
            if self.count >= 2:
                self.up.wait_event(self.freed[s])
            for k in self.names:
                bufs[k].copy_(compact_view(host_inputs[k]), non_blocking=True)
            self.uploaded[s].record(self.up)
        with torch.cuda.stream(self.run):
            self.run.wait_event(self.uploaded[s])
            args = {k: bufs[k].expand(self.shapes[k]) for k in self.names}
            o, fs = chunk_nested_gdn2(**args, output_final_state=True, **self.op_kwargs)
            self.freed[s].record(self.run)
            self.computed[s].record(self.run)
        with torch.cuda.stream(self.down):
            self.down.wait_event(self.computed[s])
            if self.out_host[s] is None:
                self.out_host[s] = (torch.empty(o.shape, dtype=o.dtype).pin_memory(),
                                    torch.empty(fs.shape, dtype=fs.dtype).pin_memory())
            oh, sh = self.out_host[s]
            oh.copy_(o, non_blocking=True)
            sh.copy_(fs, non_blocking=True)
            # The outputs were allocated on the compute stream; keep their
            # memory from being reused before this download has read it.
            o.record_stream(self.down)
            fs.record_stream(self.down)
            self.downloaded[s].record(self.down)
        self.count += 1
        return s, self.count - 1

    def wait_uploaded(self, handle):
        """Block until a batch's host inputs have been copied to the device,
        after which the caller may reuse those host tensors. Only valid for
        one of the two most recent submissions (a slot's event is re-recorded
        when the slot is reused)."""
        s, _ = handle
        self.uploaded[s].synchronize()

    def uploaded_event(self, handle):
        """The CUDA event recorded after a batch's uploads (valid for one of
        the two most recent submissions)."""
        return self.uploaded[handle[0]]

    def result(self, handle):
        """Wait for a batch and return its (o, final_state) host tensors."""
        s, _ = handle
        self.downloaded[s].synchronize()
        return self.out_host[s]

    def last_event(self):
        """The event recorded after the most recent download (for timing)."""
        return self.downloaded[(self.count - 1) % 2]

    def first_stream(self):
        """The upload stream (record a start event there for timing)."""
        return self.up
