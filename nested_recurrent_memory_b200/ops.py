"""Drop-in replacements for the reference's ``nested_gdn2.ops`` forward ops.

Same names, argument meanings, defaults, return values and ValueError
messages as the reference (awehrs/nested_recurrent_memory):

* ``chunk_nested_gdn2``      -- nested_gdn2/ops/chunk.py:722-766
* ``chunk_nested_gdn2_fwd``  -- nested_gdn2/ops/chunk.py:159-304
* ``update_state``           -- nested_gdn2/ops/update_fwd.py:131-204
* ``step_nested_gdn2``       -- nested_gdn2/ops/naive.py:42-134 (naive_step_nested_gdn2,
  the one-token decode step; same signature)
* ``n_groups``, ``n_firings`` -- nested_gdn2/ops/chunk.py:26-36

The work is done by hand-written sm_100a CUDA kernels behind the C ABI of
``libngdn2.so`` (include/ngdn2.h); this module only validates arguments,
allocates outputs and workspace with torch, and passes raw pointers and the
current CUDA stream. There is no CPU or framework fallback: CPU tensors or a
missing library raise.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

__all__ = [
    "chunk_nested_gdn2",
    "chunk_nested_gdn2_fwd",
    "chunk_nested_gdn2_bwd",
    "update_state",
    "update_state_bwd",
    "step_nested_gdn2",
    "n_groups",
    "n_firings",
    "fwd_workspace_bytes",
    "last_path",
    "check_status",
    "KernelStatusError",
    "FwdCall",
]

_DTYPES = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16, torch.float16: _lib.F16}
_LAST_PATH = [None]


class KernelStatusError(RuntimeError):
    """A forward's kernels reported a device status (include/ngdn2.h
    NGDN2_STATUS_*): a bounded wait gave up, so that forward's outputs are
    not valid."""


def _status_message(bits: int) -> str:
    parts = []
    if bits & _lib.STATUS_WAIT_TIMEOUT:
        parts.append("a bounded pipeline wait timed out (outputs invalid; treat the CUDA "
                     "context as suspect)")
    if bits & _lib.STATUS_GATE_TIMEOUT:
        parts.append("the start gate stayed closed (nothing was computed)")
    return "; ".join(parts) or f"status bits {bits:#x}"


class _DeviceStatus:
    """The sticky status word every forward on one device reports into.

    Kernels only OR bits into the device word. After each launch a 4-byte
    copy of it goes to pinned host memory on the launching stream, and an
    event marks that copy; the next launch on the device (or ``check``)
    reads the copy once its event has completed and raises
    ``KernelStatusError`` for a nonzero word, then clears it. So a timed-out
    wait surfaces at the latest one call later, with no synchronisation on
    the fast path; ``check(sync=True)`` waits for the device instead.
    With NGDN2_SYNC_CHECK=1 in the environment every launch checks
    synchronously. During CUDA-graph capture no copy is queued; the word is
    still set on replay and ``check_status`` reads it."""

    _by_device: dict = {}

    def __init__(self, device):
        self.device = device
        self.word = torch.zeros(1, dtype=torch.int32, device=device)
        self.host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self.copied = torch.cuda.Event()
        self.pending = False

    @classmethod
    def get(cls, device) -> "_DeviceStatus":
        key = (device.type, device.index if device.index is not None else torch.cuda.current_device())
        st = cls._by_device.get(key)
        if st is None:
            st = cls._by_device[key] = cls(torch.device("cuda", key[1]))
        return st

    def _raise_if_set(self, bits: int):
        if bits:
            self.word.zero_()
            self.host.zero_()
            raise KernelStatusError(f"nested GDN-2 forward: {_status_message(bits)}")

    def poll(self):
        """Raise for a status copied back by an earlier launch, if its copy is done."""
        if self.pending and self.copied.query():
            self.pending = False
            self._raise_if_set(int(self.host.item()))

    def after_launch(self):
        stream = torch.cuda.current_stream(self.device)
        if torch.cuda.is_current_stream_capturing():
            return
        if _SYNC_CHECK:
            self.check(sync=True)
            return
        self.host.copy_(self.word, non_blocking=True)
        self.copied.record(stream)
        self.pending = True

    def check(self, sync: bool = True):
        if sync:
            self.pending = False
            self._raise_if_set(int(self.word.item()))
        else:
            self.poll()


_SYNC_CHECK = __import__("os").environ.get("NGDN2_SYNC_CHECK", "0") not in ("", "0")


def check_status(device=None, sync: bool = True):
    """Raise ``KernelStatusError`` if a forward on ``device`` (default: the
    current CUDA device) reported a device status since the last check, then
    clear it. ``sync=True`` waits for the device's queued work first."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    _DeviceStatus.get(dev).check(sync=sync)


def last_path():
    """Kernel family ("simt" or "tc") that ran the most recent forward."""
    return _LAST_PATH[0]


def n_groups(n_chunks: int, firing_interval: int) -> int:
    """How many runs of ``firing_interval`` chunks cover ``n_chunks``
    (chunk.py:26-31). The last run may be short; it is read but never fired."""
    return (n_chunks + firing_interval - 1) // firing_interval


def n_firings(n_chunks: int, firing_interval: int) -> int:
    """How many firings occur in ``n_chunks``: one per complete run (chunk.py:34-36)."""
    return n_chunks // firing_interval


def _code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}; expected float32, bfloat16 or float16") from None


def _require_cuda(*ts):
    for t in ts:
        if t is not None and t.device.type != "cuda":
            raise RuntimeError(
                "nested_recurrent_memory_b200 runs on CUDA tensors only (no CPU fallback); "
                f"got a tensor on {t.device}")


def _fill_tok(args, name, t, rank):
    setattr(args, name, t.data_ptr())
    setattr(args, f"{name}_dtype", _code(t))
    st = getattr(args, f"{name}_stride")
    for i, s in enumerate(t.stride()[:rank]):
        st[i] = s


def _raise_for(rc: int, what: str, **ctx):
    if rc == 0:
        return
    msg = _lib.error_string(rc)
    if rc == _lib.ERR_CHUNK_SIZE:
        raise ValueError(f"chunk_size must be 64 for GDN-2, got {ctx.get('chunk_size')}")
    if rc == _lib.ERR_N_POW2:
        raise ValueError(f"pairs per firing must be a power of two >= 16, got {ctx.get('N')}")
    if rc == _lib.ERR_BLOCK_V:
        raise ValueError(f"block_v must be a power of two >= 16, got {ctx.get('block_v')}")
    if rc == _lib.ERR_DIVISIBLE:
        raise ValueError(f"V={ctx.get('V')} must be divisible by block_v={ctx.get('block_v')}")
    if rc == _lib.ERR_UNIT_STRIDE:
        raise ValueError("keys must be unit-stride along K")
    if rc == _lib.ERR_INCONSISTENT:
        raise ValueError(f"NF={ctx.get('NF')} inconsistent with n_groups={ctx.get('NG')}")
    raise RuntimeError(f"{what} failed: {msg} (code {rc})")


def _build_fwd_args(q, k, v, g, b, w, mix_weights, params, n_max, nq, firing, L, scale,
                    init, o, final, chunk_size, promotion, path):
    B, T, H, _, K = q.shape
    V = v.shape[-1]
    a = _lib.FwdArgs()
    a.abi_version = _lib.ABI_VERSION
    a.path = _lib.PATHS[path]
    a.B, a.T, a.H, a.K, a.V, a.L = B, T, H, K, V, L
    a.chunk_size = chunk_size
    a.promotion = _lib.PROMOTION[promotion]
    a.dtype = _code(o)
    a.param_dtype = _code(params[0]) if params else _lib.F32
    a.scale = float(scale)
    a.n_max = n_max
    for i, n in enumerate(nq):
        a.n_queries[i] = n
    for i, f in enumerate(firing):
        a.firing[i] = f
    _fill_tok(a, "q", q, 5)
    for name, t in (("k", k), ("v", v), ("g", g), ("b", b), ("w", w), ("mix", mix_weights)):
        _fill_tok(a, name, t, 4)
    if params:
        (a.query_banks, a.key_projections, a.b_projections, a.w_projections,
         a.g_projections) = (p.data_ptr() for p in params)
    a.initial_state = init.data_ptr() if init is not None else None
    a.o = o.data_ptr()
    a.final_state = final.data_ptr()
    return a


def fwd_workspace_bytes(args: "_lib.FwdArgs") -> int:
    lib = _lib.load()
    nbytes = ctypes.c_size_t(0)
    rc = lib.ngdn2_fwd_workspace_size(ctypes.byref(args), ctypes.byref(nbytes))
    _raise_for(rc, "ngdn2_fwd_workspace_size", chunk_size=args.chunk_size)
    return int(nbytes.value)


class FwdCall:
    """One validated forward call bound to its tensors.

    Holds the C-ABI argument struct, the outputs (``o``, ``final``) and the
    workspace, so the same call can be launched repeatedly (benchmarks,
    CUDA-graph capture) without re-validating or re-allocating. Launches go
    on the current CUDA stream of the inputs' device.
    """

    def __init__(self, q, k, v, g, b, w, mix_weights, query_banks, key_projections,
                 b_projections, w_projections, g_projections, n_queries_per_level,
                 firing_intervals, L, scale=None, initial_state=None, chunk_size=64,
                 promotion="learned", path="auto", workspace=None, gate=None, gate_polls=0):
        B, T, H, _, K = q.shape
        if chunk_size != 64:  # chunk.py:230-231
            raise ValueError(f"chunk_size must be 64 for GDN-2, got {chunk_size}")
        if promotion not in _lib.PROMOTION:
            raise KeyError(promotion)  # PROBES[promotion] in the reference
        if path not in _lib.PATHS:
            raise ValueError(f"path must be one of {sorted(_lib.PATHS)}, got {path!r}")
        if scale is None:
            scale = K ** -0.5
        V = v.shape[-1]
        firing = [int(x) for x in firing_intervals]
        nq = [int(x) for x in n_queries_per_level]
        for lvl in range(1, L):
            n = K if promotion == "merge" else nq[lvl - 1]
            if n < 16 or n & (n - 1):  # update_fwd.py:162-163
                raise ValueError(f"pairs per firing must be a power of two >= 16, got {n}")
        _require_cuda(q, k, v, g, b, w, mix_weights, initial_state)
        params, n_max = [], 1
        if L > 1:
            pdt = query_banks.dtype
            params = [t.to(q.device, pdt).contiguous() for t in
                      (query_banks, key_projections, b_projections, w_projections, g_projections)]
            _require_cuda(*params)
            n_max = query_banks.shape[2]
        init = initial_state.to(torch.float32).contiguous() if initial_state is not None else None
        self.device = q.device
        self.T = T
        self.o = torch.empty(B, T, H, V, dtype=q.dtype, device=q.device)
        self.final = torch.empty(B, H, L, K, V, dtype=torch.float32, device=q.device)
        self.init = init
        self._keep = (q, k, v, g, b, w, mix_weights, params, init)
        self.path = None
        self.args = None
        if T == 0:
            return
        lib = _lib.load()
        self.args = _build_fwd_args(q, k, v, g, b, w, mix_weights, params, n_max, nq, firing, L,
                                    scale, init, self.o, self.final, chunk_size, promotion, path)
        sel = lib.ngdn2_fwd_select_path(ctypes.byref(self.args))
        _raise_for(sel if sel < 0 else 0, "ngdn2_fwd_select_path", chunk_size=chunk_size)
        self.path = _lib.PATH_NAMES.get(sel)
        need = fwd_workspace_bytes(self.args)
        if workspace is None or workspace.numel() < need:
            workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=q.device)
        self.workspace = workspace
        self.args.workspace = workspace.data_ptr()
        self.args.workspace_bytes = workspace.numel()
        # Every forward reports into its device's sticky status word.
        self._status = _DeviceStatus.get(q.device)
        self.args.status = self._status.word.data_ptr()
        if gate is not None:
            _require_cuda(gate)
            if gate.dtype != torch.int32 or gate.numel() < 1:
                raise TypeError("gate must be an int32 CUDA tensor")
            self._keep = self._keep + (gate,)
            self.args.gate = gate.data_ptr()
            self.args.gate_polls = int(gate_polls)

    @property
    def num_launches(self) -> int:
        if self.args is None:
            return 0
        return _lib.load().ngdn2_fwd_num_launches(ctypes.byref(self.args))

    def launch(self, stage: int = 0):
        """Run the forward (stage 0) or one of its stages (1 = prep, 2 = scan)."""
        if self.args is None:
            self.final.copy_(self.init if self.init is not None else torch.zeros_like(self.final))
            return self.o, self.final
        self._status.poll()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        rc = _lib.load().ngdn2_fwd_stage(ctypes.byref(self.args), stage, ctypes.c_void_p(stream))
        _raise_for(rc, "ngdn2_fwd", chunk_size=self.args.chunk_size)
        _LAST_PATH[0] = self.path
        self._status.after_launch()
        return self.o, self.final

    def check(self, sync: bool = True):
        """Raise ``KernelStatusError`` if a forward on this call's device
        reported a device status (a bounded wait gave up, or the start gate
        stayed closed); ``sync`` waits for the device first."""
        if self.args is not None:
            self._status.check(sync=sync)


def chunk_nested_gdn2_fwd(
    q, k, v, g, b, w, mix_weights, query_banks, key_projections, b_projections,
    w_projections, g_projections, n_queries_per_level, firing_intervals, L,
    scale=None, initial_state=None, output_final_state=False, chunk_size=64,
    return_aux=False, promotion="learned", *, path="auto", workspace=None,
):
    """Chunkwise NestedGDN-2 forward (chunk.py:159-304).

    Args and returns as the reference: q [B, T, H, L, K]; k, g, b
    [B, T, H, K]; v, w [B, T, H, V]; mix_weights [B, T, H, L];
    query_banks [L-1, H, N, K]; key_projections [L-1, H, K, V];
    b/g_projections [L-1, H, V, K]; w_projections [L-1, H, V, V];
    n_queries_per_level [L-1] ints; firing_intervals [L] ints; initial_state
    [B, H, L, K, V] or None. Returns ``(o, final_state)`` with o in q's dtype
    and final_state fp32 (None unless ``output_final_state``); with
    ``return_aux`` also a dict, which here holds only ``scale`` and the
    per-level ``finals``: the backward (chunk_nested_gdn2_bwd) recomputes
    its intermediates instead of keeping the reference's aux tensors.

    Keyword-only extras: ``path`` ("auto", "simt" or "tc") picks the kernel
    family; ``workspace`` is an optional preallocated uint8 CUDA tensor.

    Device-side failures (a bounded wait that gave up) are reported through
    a sticky per-device status word: the next forward on the device raises
    ``KernelStatusError``, and so does ``check_status()`` at any time.
    """
    call = FwdCall(q, k, v, g, b, w, mix_weights, query_banks, key_projections, b_projections,
                   w_projections, g_projections, n_queries_per_level, firing_intervals, L,
                   scale=scale, initial_state=initial_state, chunk_size=chunk_size,
                   promotion=promotion, path=path, workspace=workspace)
    o, final = call.launch()
    final_state = final if output_final_state else None
    if not return_aux:
        return o, final_state
    aux = dict(scale=scale if scale is not None else q.shape[-1] ** -0.5,
               finals=list(final.unbind(2)))
    return o, final_state, aux


def chunk_nested_gdn2_bwd(q, k, v, g, b, w, mix_weights, query_banks, key_projections,
                          b_projections, w_projections, g_projections, n_queries_per_level,
                          firing_intervals, L, do, d_final=None, scale=None, initial_state=None,
                          chunk_size=64, promotion="learned", workspace=None):
    """Gradients of ``sum(o * do) + sum(final_state * d_final)`` with respect
    to every differentiable input (the job of chunk.py:368-564 behind
    ChunkNestedGDN2Function.backward, chunk.py:650-719).

    Runs ``ngdn2_bwd``: a checkpointing re-run of the forward on CUDA cores,
    then the reverse scan and the per-chunk gradients, all fp32. Returns
    ``(dq, dk, dv, dg, db, dw, dmix, dquery_banks, dkey_projections,
    db_projections, dw_projections, dg_projections, dinitial_state)`` in the
    dtypes of the corresponding inputs (``dinitial_state`` is None without an
    initial state).
    """
    B, T, H, _, K = q.shape
    V = v.shape[-1]
    if chunk_size != 64:  # chunk.py:230-231
        raise ValueError(f"chunk_size must be 64 for GDN-2, got {chunk_size}")
    if promotion not in _lib.PROMOTION:
        raise KeyError(promotion)
    if scale is None:
        scale = K ** -0.5
    _require_cuda(q, k, v, g, b, w, mix_weights, do, initial_state, d_final)
    firing = [int(x) for x in firing_intervals]
    nq = [int(x) for x in n_queries_per_level]
    dev = q.device
    f32 = dict(dtype=torch.float32, device=dev)
    dq = torch.zeros(B, T, H, L, K, **f32)
    dk, dg, db = (torch.zeros(B, T, H, K, **f32) for _ in range(3))
    dv, dw = (torch.zeros(B, T, H, V, **f32) for _ in range(2))
    dmix = torch.zeros(B, T, H, L, **f32)
    raw = (query_banks, key_projections, b_projections, w_projections, g_projections)
    dparams = [torch.zeros(t.shape, **f32) for t in raw]
    dinit = torch.zeros(B, H, L, K, V, **f32) if initial_state is not None else None
    if T > 0:
        params, n_max = [], 1
        if L > 1:
            params = [t.to(dev, query_banks.dtype).contiguous() for t in raw]
            n_max = query_banks.shape[2]
        init = (initial_state.to(torch.float32).contiguous()
                if initial_state is not None else None)
        # The forward's o and final_state are not used by the backward; do
        # stands in for o so the argument struct validates.
        fa = _build_fwd_args(q, k, v, g, b, w, mix_weights, params, n_max, nq, firing, L,
                             scale, init, do, dq, chunk_size, promotion, "simt")
        a = _lib.BwdArgs()
        a.abi_version = _lib.ABI_VERSION
        a.fwd = fa
        _fill_tok(a, "d_o", do, 4)
        dfin = d_final.to(torch.float32).contiguous() if d_final is not None else None
        a.d_final = dfin.data_ptr() if dfin is not None else None
        a.dq, a.dk, a.dv, a.dg = dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dg.data_ptr()
        a.db, a.dw, a.dmix = db.data_ptr(), dw.data_ptr(), dmix.data_ptr()
        if L > 1:
            (a.dquery_banks, a.dkey_projections, a.db_projections, a.dw_projections,
             a.dg_projections) = (t.data_ptr() for t in dparams)
        a.dinitial_state = dinit.data_ptr() if dinit is not None else None
        lib = _lib.load()
        nbytes = ctypes.c_size_t(0)
        rc = lib.ngdn2_bwd_workspace_size(ctypes.byref(a), ctypes.byref(nbytes))
        _raise_for(rc, "ngdn2_bwd_workspace_size", chunk_size=chunk_size)
        if workspace is None or workspace.numel() < nbytes.value:
            workspace = torch.empty(max(int(nbytes.value), 1), dtype=torch.uint8, device=dev)
        a.workspace, a.workspace_bytes = workspace.data_ptr(), workspace.numel()
        stream = torch.cuda.current_stream(dev).cuda_stream
        rc = lib.ngdn2_bwd(ctypes.byref(a), ctypes.c_void_p(stream))
        _raise_for(rc, "ngdn2_bwd", chunk_size=chunk_size)
    elif dinit is not None and d_final is not None:
        dinit.copy_(d_final)
    out = [dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype), dg.to(g.dtype), db.to(b.dtype),
           dw.to(w.dtype), dmix.to(mix_weights.dtype)]
    out += [d.to(t.dtype) for d, t in zip(dparams, raw)]
    out.append(dinit.to(initial_state.dtype) if dinit is not None else None)
    return tuple(out)


class ChunkNestedGDN2Function(torch.autograd.Function):
    """Autograd node for the whole op (chunk.py:567-719). The forward runs the
    fast path and keeps only its inputs; the backward recomputes what it needs
    (chunk_nested_gdn2_bwd)."""

    @staticmethod
    def forward(ctx, q, k, v, g, b, w, mix_weights, query_banks, key_projections,
                b_projections, w_projections, g_projections, n_queries_per_level,
                firing_intervals, L, scale, initial_state, output_final_state,
                chunk_size, promotion):
        o, final_state = chunk_nested_gdn2_fwd(
            q, k, v, g, b, w, mix_weights, query_banks, key_projections, b_projections,
            w_projections, g_projections, n_queries_per_level, firing_intervals, L,
            scale=scale, initial_state=initial_state, output_final_state=True,
            chunk_size=chunk_size, promotion=promotion)
        ctx.save_for_backward(q, k, v, g, b, w, mix_weights, query_banks, key_projections,
                              b_projections, w_projections, g_projections, initial_state)
        ctx.meta = ([int(x) for x in n_queries_per_level], [int(x) for x in firing_intervals],
                    L, scale, chunk_size, promotion)
        return o, (final_state if output_final_state else None)

    @staticmethod
    def backward(ctx, do, dfinal):
        (q, k, v, g, b, w, mix, qb, kp, bp, wp, gp, init) = ctx.saved_tensors
        nq, firing, L, scale, chunk_size, promotion = ctx.meta
        if do is None:
            do = torch.zeros(*q.shape[:3], v.shape[-1], dtype=q.dtype, device=q.device)
        grads = chunk_nested_gdn2_bwd(
            q, k, v, g, b, w, mix, qb, kp, bp, wp, gp, nq, firing, L, do.contiguous(),
            d_final=dfinal, scale=scale, initial_state=init, chunk_size=chunk_size,
            promotion=promotion)
        return (*grads[:12], None, None, None, None, grads[12], None, None, None)


def chunk_nested_gdn2(q, k, v, g, b, w, mix_weights, query_banks, key_projections,
                      b_projections, w_projections, g_projections, n_queries_per_level,
                      firing_intervals, L, scale=None, initial_state=None,
                      output_final_state=False, chunk_size=64, promotion="learned"):
    """Chunkwise NestedGDN-2 (chunk.py:722-766). Signature matches the naive op."""
    return ChunkNestedGDN2Function.apply(
        q, k, v, g, b, w, mix_weights, query_banks, key_projections, b_projections,
        w_projections, g_projections, n_queries_per_level, firing_intervals, L, scale,
        initial_state, output_final_state, chunk_size, promotion)


def update_state_bwd(states, keys, values, g, b, w, d_states, d_final, has_init=False,
                     block_v=16):
    """Backward of ``update_state`` (update_bwd.py:167-263): the gradients of
    ``sum(states * d_states) + sum(final * d_final)``.

    states [B, NG, H, K, V] (from the forward); keys [B, NF, H, N, K] (may be
    a broadcast view); values, w [B, NF, H, N, V]; g [B, NF, H, K]; b
    [B, NF, H, N, K]; d_states like states; d_final [B, H, K, V]. Returns a
    dict with float32 ``dkeys``, ``dvalues``, ``dg``, ``db``, ``dw`` and, when
    ``has_init``, ``dinit`` -- as the reference.
    """
    B, NF, H, N, K = keys.shape
    NG = states.shape[1]
    V = values.shape[-1]
    # update_bwd.py:197-206, same checks and order.
    if N < 16 or N & (N - 1):
        raise ValueError(f"pairs per firing must be a power of two >= 16, got {N}")
    if block_v < 16 or block_v & (block_v - 1):
        raise ValueError(f"block_v must be a power of two >= 16, got {block_v}")
    if V % block_v:
        raise ValueError(f"V={V} must be divisible by block_v={block_v}")
    if keys.stride(-1) != 1:
        raise ValueError("keys must be unit-stride along K")
    if not (NG - 1 <= NF <= NG):
        raise ValueError(f"NF={NF} inconsistent with NG={NG}")
    _require_cuda(states, keys, values, g, b, w, d_states, d_final)
    dt = values.dtype
    if keys.dtype != dt:
        keys = keys.to(dt)
    values, b, w = (t.to(dt).contiguous() for t in (values, b, w))
    g = g.contiguous()
    states, d_states, d_final = (t.to(torch.float32).contiguous()
                                 for t in (states, d_states, d_final))
    f32 = dict(dtype=torch.float32, device=values.device)
    out = {"dkeys": torch.zeros(B, NF, H, N, K, **f32),
           "dvalues": torch.zeros(B, NF, H, N, V, **f32),
           "dg": torch.zeros(B, NF, H, K, **f32),
           "db": torch.zeros(B, NF, H, N, K, **f32),
           "dw": torch.zeros(B, NF, H, N, V, **f32)}
    dinit = torch.zeros(B, H, K, V, **f32) if has_init else None
    a = _lib.UpdateBwdArgs()
    a.abi_version = _lib.ABI_VERSION
    a.B, a.NF, a.NG, a.H, a.K, a.V, a.N = B, NF, NG, H, K, V, N
    a.block_v = block_v
    a.dtype, a.g_dtype = _code(values), _code(g)
    a.has_init = int(bool(has_init))
    a.states = states.data_ptr()
    a.keys = keys.data_ptr()
    for i, st in enumerate(keys.stride()):
        a.keys_stride[i] = st
    a.values, a.g, a.b, a.w = values.data_ptr(), g.data_ptr(), b.data_ptr(), w.data_ptr()
    a.d_states, a.d_final = d_states.data_ptr(), d_final.data_ptr()
    (a.dkeys, a.dvalues, a.dg, a.db, a.dw) = (out[n].data_ptr() for n in
                                              ("dkeys", "dvalues", "dg", "db", "dw"))
    a.dinit = dinit.data_ptr() if dinit is not None else None
    lib = _lib.load()
    nbytes = ctypes.c_size_t(0)
    rc = lib.ngdn2_update_bwd_workspace_size(ctypes.byref(a), ctypes.byref(nbytes))
    _raise_for(rc, "ngdn2_update_bwd_workspace_size", N=N, block_v=block_v, V=V, NF=NF, NG=NG)
    ws = torch.empty(max(int(nbytes.value), 1), dtype=torch.uint8, device=values.device)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    stream = torch.cuda.current_stream(values.device).cuda_stream
    rc = lib.ngdn2_update_state_bwd(ctypes.byref(a), ctypes.c_void_p(stream))
    _raise_for(rc, "ngdn2_update_state_bwd", N=N, block_v=block_v, V=V, NF=NF, NG=NG)
    if has_init:
        out["dinit"] = dinit
    return out


def update_state(keys, values, g, b, w, n_groups, initial_state=None, block_v=16):
    """Run one level's write scan over all groups (update_fwd.py:131-204).

    keys [B, NF, H, N, K] (may be a broadcast view; read by stride);
    values, w [B, NF, H, N, V]; g [B, NF, H, K]; b [B, NF, H, N, K].
    Returns states [B, NG, H, K, V] (the state entering each group) and the
    final state [B, H, K, V], both float32.
    """
    B, NF, H, N, K = keys.shape
    V = values.shape[-1]
    # update_fwd.py:162-171, same checks and order.
    if N < 16 or N & (N - 1):
        raise ValueError(f"pairs per firing must be a power of two >= 16, got {N}")
    if block_v < 16 or block_v & (block_v - 1):
        raise ValueError(f"block_v must be a power of two >= 16, got {block_v}")
    if V % block_v:
        raise ValueError(f"V={V} must be divisible by block_v={block_v}")
    if keys.stride(-1) != 1:
        raise ValueError("keys must be unit-stride along K")
    if not (n_groups - 1 <= NF <= n_groups):
        raise ValueError(f"NF={NF} inconsistent with n_groups={n_groups}")
    _require_cuda(keys, values, g, b, w, initial_state)
    dt = values.dtype
    if keys.dtype != dt:
        keys = keys.to(dt)
    values, b, w = (t.to(dt).contiguous() for t in (values, b, w))
    g = g.contiguous()
    states = values.new_empty(B, n_groups, H, K, V, dtype=torch.float32)
    final = values.new_empty(B, H, K, V, dtype=torch.float32)
    init = initial_state.to(torch.float32).contiguous() if initial_state is not None else None
    a = _lib.UpdateArgs()
    a.abi_version = _lib.ABI_VERSION
    a.B, a.NF, a.NG, a.H, a.K, a.V, a.N = B, NF, n_groups, H, K, V, N
    a.block_v = block_v
    a.dtype, a.g_dtype = _code(values), _code(g)
    a.keys = keys.data_ptr()
    for i, s in enumerate(keys.stride()):
        a.keys_stride[i] = s
    a.values, a.g, a.b, a.w = values.data_ptr(), g.data_ptr(), b.data_ptr(), w.data_ptr()
    a.initial_state = init.data_ptr() if init is not None else None
    a.states, a.final_state = states.data_ptr(), final.data_ptr()
    stream = torch.cuda.current_stream(values.device).cuda_stream
    rc = _lib.load().ngdn2_update_state(ctypes.byref(a), ctypes.c_void_p(stream))
    _raise_for(rc, "ngdn2_update_state", N=N, block_v=block_v, V=V, NF=NF, NG=n_groups)
    return states, final


def step_nested_gdn2(q, k, v, g, b, w, mix_weights, state, position, query_banks,
                     key_projections, b_projections, w_projections, g_projections,
                     n_queries_per_level, firing_intervals, L, scale=None, chunk_size=64,
                     promotion="learned", *, out_state=None, workspace=None):
    """One decode token for every batch row (naive.py:42-134,
    ``naive_step_nested_gdn2``): level 0 writes, every level is read and
    mixed, then each level whose firing this token completes promotes,
    bottom-up. Level 0 writes before the read, levels above after, so a
    firing is first visible at the next token.

    Args as the reference: q [B, H, L, K]; k, g, b [B, H, K]; v, w [B, H, V];
    mix_weights [B, H, L]; state [B, H, L, K, V] float32; position an int or a
    [B] integer tensor (rows at different positions fire on different
    tokens); the rest as for ``chunk_nested_gdn2``. ``out_state`` may be
    ``state`` itself to update in place.

    Returns ``(o, state)``: o [B, H, V] in q's dtype, the new state float32.
    """
    if promotion not in _lib.PROMOTION:
        raise KeyError(promotion)  # PROBES[promotion] in the reference
    B, H, _, K = q.shape
    V = v.shape[-1]
    if scale is None:
        scale = K ** -0.5
    firing = [int(x) for x in firing_intervals]
    nq = [int(x) for x in n_queries_per_level]
    for lvl in range(1, L):
        n = K if promotion == "merge" else nq[lvl - 1]
        if n < 16 or n & (n - 1):
            raise ValueError(f"pairs per firing must be a power of two >= 16, got {n}")
    _require_cuda(q, k, v, g, b, w, mix_weights, state)
    params, n_max = [], 1
    if L > 1:
        pdt = query_banks.dtype
        params = [t.to(q.device, pdt).contiguous() for t in
                  (query_banks, key_projections, b_projections, w_projections, g_projections)]
        _require_cuda(*params)
        n_max = query_banks.shape[2]
    state_in = state.to(torch.float32).contiguous()
    new = torch.empty_like(state_in) if out_state is None else out_state
    o = torch.empty(B, H, V, dtype=q.dtype, device=q.device)
    a = _lib.StepArgs()
    a.abi_version = _lib.ABI_VERSION
    a.B, a.H, a.K, a.V, a.L = B, H, K, V, L
    a.chunk_size = int(chunk_size)
    a.promotion = _lib.PROMOTION[promotion]
    a.dtype = _code(o)
    a.param_dtype = _code(params[0]) if params else _lib.F32
    a.scale = float(scale)
    a.n_max = n_max
    for i, n in enumerate(nq):
        a.n_queries[i] = n
    for i, f in enumerate(firing):
        a.firing[i] = f
    _fill_tok(a, "q", q, 4)
    for name, t in (("k", k), ("v", v), ("g", g), ("b", b), ("w", w), ("mix", mix_weights)):
        _fill_tok(a, name, t, 3)
    if params:
        (a.query_banks, a.key_projections, a.b_projections, a.w_projections,
         a.g_projections) = (p.data_ptr() for p in params)
    pos = None
    if torch.is_tensor(position):
        pos = position.to(q.device, torch.int64).contiguous()
        a.positions = pos.data_ptr()
    else:
        a.position = int(position)
    a.state_in = state_in.data_ptr()
    a.state_out = new.data_ptr()
    a.o = o.data_ptr()
    lib = _lib.load()
    need = ctypes.c_size_t(0)
    _raise_for(lib.ngdn2_step_workspace_size(ctypes.byref(a), ctypes.byref(need)), "ngdn2_step")
    if need.value and (workspace is None or workspace.numel() < need.value):
        workspace = torch.empty(need.value, dtype=torch.uint8, device=q.device)
    if need.value:
        a.workspace = workspace.data_ptr()
        a.workspace_bytes = workspace.numel()
    stream = torch.cuda.current_stream(q.device).cuda_stream
    _raise_for(lib.ngdn2_step(ctypes.byref(a), ctypes.c_void_p(stream)), "ngdn2_step")
    return o, new
