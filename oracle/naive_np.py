"""Numpy restatement of the reference's nested GDN-2 oracle.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): never imported by the
product path.

Every function follows one reference function and cites it by file:line
within the reference project (awehrs/nested_recurrent_memory):

* ``nested_gdn2/ops/naive.py``   -- update step, token step, recurrent and
  chunkwise forwards;
* ``nested_gdn2/ops/probe.py``   -- the ``learned`` and ``merge`` probes;
* ``nested_gdn2/ops/chunk.py``   -- schedule arithmetic (groups, firings,
  source index);
* ``tests/ops/_update_ref.py``   -- the group scan over the update step.

Arithmetic runs in ``dtype`` (float64 by default, which makes the oracle a
stricter checker than the fp32 torch original; float32 reproduces the
reference's own precision for the CPU baseline).

Layouts are the reference's: per-token tensors are ``[B, T, H, ...]``,
states ``[B, H, L, K, V]``.
"""

from __future__ import annotations

import numpy as np

# probe.py:28-31 -- gate logit offsets.
B_LOGIT_INIT = -4.0
W_LOGIT_INIT = 0.0
G_LOGIT_INIT = -4.0


# ----------------------------------------------------------------------------
# Schedule arithmetic (chunk.py:26-55)
# ----------------------------------------------------------------------------


def n_groups(n_chunks: int, firing_interval: int) -> int:
    """Runs of ``firing_interval`` chunks covering ``n_chunks`` (chunk.py:26-31)."""
    return (n_chunks + firing_interval - 1) // firing_interval


def n_firings(n_chunks: int, firing_interval: int) -> int:
    """One firing per complete run (chunk.py:34-36)."""
    return n_chunks // firing_interval


def source_index(firing_below: int, firing_here: int, n_chunks: int) -> list[int]:
    """Group of the level below read by each firing of this level (chunk.py:39-55)."""
    return [((i + 1) * firing_here) // firing_below
            for i in range(n_firings(n_chunks, firing_here))]


# ----------------------------------------------------------------------------
# Elementwise helpers with torch's semantics
# ----------------------------------------------------------------------------


def _sigmoid(x):
    return 0.5 * (1.0 + np.tanh(0.5 * x))


def _softplus(x):
    # torch.nn.functional.softplus (beta=1, threshold=20): x above 20 is
    # returned as is; below, log1p(exp(x)) evaluated stably.
    return np.where(x > 20.0, x, np.logaddexp(0.0, x))


def _normalize(x, eps=1e-12):
    # torch.nn.functional.normalize(x, dim=-1): x / max(||x||_2, eps).
    n = np.sqrt((x * x).sum(-1, keepdims=True))
    return x / np.maximum(n, eps)


# ----------------------------------------------------------------------------
# Probes (probe.py)
# ----------------------------------------------------------------------------


def gates(values, b_proj, w_proj, g_proj):
    """Gates projected from the values being written (probe.py:34-66).

    values [..., H, N, V]; b_proj [H, V, K]; w_proj [H, V, V]; g_proj [H, V, K].
    Returns b [..., H, N, K], w [..., H, N, V], g [..., H, K] (mean over N).
    """
    b = np.einsum("hvk,...hnv->...hnk", b_proj, values)
    w = np.einsum("hvu,...hnv->...hnu", w_proj, values)
    g = np.einsum("hvk,...hnv->...hnk", g_proj, values)
    b = _sigmoid(b + B_LOGIT_INIT)
    w = _sigmoid(w + W_LOGIT_INIT)
    g = -_softplus(g + G_LOGIT_INIT).mean(axis=-2)
    return b, w, g


def probe_learned(state_below, query_bank, key_proj, b_proj, w_proj, g_proj, n_queries):
    """Learned query bank reads the level below (probe.py:69-102).

    state_below [..., H, K, V]; query_bank [H, N_MAX, K] (rows past
    ``n_queries`` ignored); key_proj [H, K, V].
    Returns keys [..., H, n, K] (unit norm), values [..., H, n, V], b, w, g.
    """
    q = query_bank[:, :n_queries]
    values = np.einsum("hnk,...hkv->...hnv", q, state_below)
    u = np.einsum("hkv,...hnv->...hnk", key_proj, values)
    keys = _normalize(u)
    b, w, g = gates(values, b_proj, w_proj, g_proj)
    return keys, values, b, w, g


def probe_merge(state_below, query_bank, key_proj, b_proj, w_proj, g_proj, n_queries):
    """Identity addresses: each row of the level below written whole (probe.py:105-136).

    The bank, key projection and ``n_queries`` are ignored; always K pairs.
    """
    K = state_below.shape[-2]
    keys = np.broadcast_to(np.eye(K, dtype=state_below.dtype),
                           state_below.shape[:-2] + (K, K))
    b, w, g = gates(state_below, b_proj, w_proj, g_proj)
    return keys, state_below, b, w, g


PROBES = {"learned": probe_learned, "merge": probe_merge}


# ----------------------------------------------------------------------------
# Update (naive.py:7-39) and the group scan (tests/ops/_update_ref.py:34-51)
# ----------------------------------------------------------------------------


def update_step(state, keys, values, b, w, g):
    """One firing: decay, erase at the keys, write the values (naive.py:7-39).

    state [..., K, V]; keys, b [..., N, K]; values, w [..., N, V]; g [..., K].
    All N pairs act on the pre-firing state. Unfactored, as in the reference.
    """
    S = state * np.exp(g)[..., :, None]
    kb = keys * b
    gram = np.einsum("...nk,...nj->...kj", keys, kb)
    return (S - np.einsum("...kj,...jv->...kv", gram, S)
            + np.einsum("...nk,...nv->...kv", keys, values * w))


def update_scan(keys, values, g, b, w, n_groups, initial_state=None):
    """The write scan of ``update_state`` (update_fwd.py:131-204), as the
    reference tests restate it (tests/ops/_update_ref.py:34-51).

    keys, b [B, NF, H, N, K]; values, w [B, NF, H, N, V]; g [B, NF, H, K].
    Returns states [B, NG, H, K, V] (the state entering each group) and the
    final state [B, H, K, V].
    """
    B, NF, H, _, K = keys.shape
    V = values.shape[-1]
    S = (np.array(initial_state, dtype=values.dtype) if initial_state is not None
         else np.zeros((B, H, K, V), dtype=values.dtype))
    states = []
    for j in range(n_groups):
        states.append(S)
        if j < NF:
            S = update_step(S, keys[:, j], values[:, j], b[:, j], w[:, j], g[:, j])
    return np.stack(states, axis=1), S


# ----------------------------------------------------------------------------
# Token step and token-recurrent forward (naive.py:42-223)
# ----------------------------------------------------------------------------


def step(q, k, v, g, b, w, mix_weights, state, position,
         query_banks, key_projections, b_projections, w_projections, g_projections,
         n_queries_per_level, firing_intervals, L, scale=None, chunk_size=64,
         promotion="learned", dtype=np.float64):
    """One token (naive.py:42-134): level 0 writes, every level is read and
    mixed, then each level whose firing this token completes promotes,
    bottom-up.

    q [B, H, L, K]; k, g, b [B, H, K]; v, w [B, H, V]; mix [B, H, L];
    state [B, H, L, K, V]; position an int or [B] ints.
    Returns o [B, H, V] and the new state.
    """
    f = lambda x: np.asarray(x, dtype=dtype)  # noqa: E731
    q, k, v, g, b, w, mix_weights = map(f, (q, k, v, g, b, w, mix_weights))
    if scale is None:
        scale = q.shape[-1] ** -0.5
    S = [f(state)[:, :, lvl] for lvl in range(L)]
    S[0] = update_step(S[0], k[:, :, None], v[:, :, None], b[:, :, None], w[:, :, None], g)
    reads = np.einsum("bhlk,bhlkv->bhlv", q * scale, np.stack(S, axis=2))
    o = (reads * mix_weights[..., None]).sum(2)

    Bsz = k.shape[0]
    pos = (np.asarray(position, dtype=np.int64) if np.ndim(position)
           else np.full(Bsz, int(position), dtype=np.int64))
    end = pos + 1
    at_boundary = end % chunk_size == 0
    chunk = end // chunk_size
    for lvl in range(1, L):
        fire = at_boundary & (chunk % int(firing_intervals[lvl]) == 0)
        idx = np.nonzero(fire)[0]
        if idx.size == 0:
            continue
        keys, vals, bp, wp, gp = PROBES[promotion](
            S[lvl - 1][idx],
            f(query_banks[lvl - 1]), f(key_projections[lvl - 1]),
            f(b_projections[lvl - 1]), f(w_projections[lvl - 1]),
            f(g_projections[lvl - 1]), int(n_queries_per_level[lvl - 1]))
        new = S[lvl].copy()
        new[idx] = update_step(S[lvl][idx], keys, vals, bp, wp, gp)
        S[lvl] = new
    return o, np.stack(S, axis=2)


def recurrent_forward(q, k, v, g, b, w, mix_weights, query_banks, key_projections,
                      b_projections, w_projections, g_projections,
                      n_queries_per_level, firing_intervals, L, scale=None,
                      initial_state=None, output_final_state=False, chunk_size=1,
                      promotion="learned", dtype=np.float64):
    """Token-by-token forward (naive.py:137-223)."""
    B, T, H, K = np.shape(k)
    V = np.shape(v)[-1]
    state = (np.array(initial_state, dtype=dtype) if initial_state is not None
             else np.zeros((B, H, L, K, V), dtype=dtype))
    outs = []
    for t in range(T):
        o_t, state = step(q[:, t], k[:, t], v[:, t], g[:, t], b[:, t], w[:, t],
                          mix_weights[:, t], state, t, query_banks, key_projections,
                          b_projections, w_projections, g_projections,
                          n_queries_per_level, firing_intervals, L, scale=scale,
                          chunk_size=chunk_size, promotion=promotion, dtype=dtype)
        outs.append(o_t)
    return np.stack(outs, axis=1), (state if output_final_state else None)


# ----------------------------------------------------------------------------
# Chunkwise forward (naive.py:226-420)
# ----------------------------------------------------------------------------


def chunk_forward(q, k, v, g, b, w, mix_weights, query_banks, key_projections,
                  b_projections, w_projections, g_projections,
                  n_queries_per_level, firing_intervals, L, scale=None,
                  initial_state=None, output_final_state=False, chunk_size=64,
                  promotion="learned", dtype=np.float64):
    """Chunkwise nested GDN-2 forward, the reference oracle's algorithm
    (naive.py:226-420), restated one chunk at a time so that the per-channel
    decay tensor is [B, H, C, C, K] for one chunk instead of for all of them.

    q [B, T, H, L, K]; k, g, b [B, T, H, K]; v, w [B, T, H, V];
    mix_weights [B, T, H, L]; query_banks [L-1, H, N_MAX, K];
    key_projections [L-1, H, K, V]; b/g_projections [L-1, H, V, K];
    w_projections [L-1, H, V, V]; initial_state [B, H, L, K, V] or None.
    Returns o [B, T, H, V] (in ``dtype``) and the final state or None.
    """
    f = lambda x: np.asarray(x, dtype=dtype)  # noqa: E731
    BT = chunk_size
    # naive.py:293-296 -- [B, H, T, ...] layout.
    q = f(q).transpose(0, 2, 1, 3, 4)
    k, v, g, b, w = (f(x).transpose(0, 2, 1, 3) for x in (k, v, g, b, w))
    mix = f(mix_weights).transpose(0, 2, 1, 3)
    B, H, T, K = k.shape
    V = v.shape[-1]
    if scale is None:
        scale = q.shape[-1] ** -0.5  # naive.py:288-289

    # naive.py:302-312 -- zero-pad T to a multiple of BT; the padded tail
    # neither decays (g = 0) nor writes (k = 0), and its chunk still fires.
    pad = (BT - T % BT) % BT
    if pad:
        q = np.pad(q, ((0, 0), (0, 0), (0, pad), (0, 0), (0, 0)))
        k, v, g, b, w = (np.pad(x, ((0, 0), (0, 0), (0, pad), (0, 0))) for x in (k, v, g, b, w))
        mix = np.pad(mix, ((0, 0), (0, 0), (0, pad), (0, 0)))
    NT = q.shape[2] // BT
    q = q * scale  # naive.py:314

    strict = np.tril(np.ones((BT, BT), dtype=bool), -1)   # naive.py:337-340
    causal = np.tril(np.ones((BT, BT), dtype=bool), 0)    # naive.py:355-358
    eye = np.eye(BT, dtype=dtype)

    if initial_state is not None:                          # naive.py:360-363
        S = [f(initial_state)[:, :, lvl].copy() for lvl in range(L)]
    else:
        S = [np.zeros((B, H, K, V), dtype=dtype) for _ in range(L)]
    o = np.zeros((B, H, NT * BT, V), dtype=dtype)

    for n in range(NT):                                    # naive.py:367
        sl = slice(n * BT, (n + 1) * BT)
        q0, kn, vn, gn, bn, wn = q[:, :, sl, 0], k[:, :, sl], v[:, :, sl], g[:, :, sl], b[:, :, sl], w[:, :, sl]
        gc = np.cumsum(gn, axis=2)                         # naive.py:329-330
        gl = gc[:, :, -1]
        kgb = kn * np.exp(gc) * bn                         # naive.py:332-333
        decay = np.exp(np.minimum(gc[:, :, :, None, :] - gc[:, :, None, :, :], 0.0))  # naive.py:335-336,354
        t_low = np.einsum("bhik,bhjk,bhijk->bhij", bn * kn, kn, decay)  # naive.py:341-344
        t_low = np.where(strict, t_low, 0.0)
        # naive.py:346-351 -- [U | W] = (I + T_lower)^-1 [w*v | k_g_b].
        sol = np.linalg.solve(eye + t_low, np.concatenate([wn * vn, kgb], axis=-1))
        u_wy, w_wy = sol[..., :V], sol[..., V:]
        k_tail = kn * np.exp(gl[:, :, None, :] - gc)       # naive.py:352

        v_new = u_wy - w_wy @ S[0]                         # naive.py:376
        a_qk = np.where(causal, np.einsum("bhik,bhjk,bhijk->bhij", q0, kn, decay), 0.0)  # :377-378
        reads = [a_qk @ v_new + (q0 * np.exp(gc)) @ S[0]]   # naive.py:379
        for lvl in range(1, L):                             # naive.py:382-385
            reads.append(q[:, :, sl, lvl] @ S[lvl])
        o[:, :, sl] = sum(mix[:, :, sl, lvl, None] * reads[lvl] for lvl in range(L))  # :387-390

        S[0] = S[0] * np.exp(gl)[..., None] + np.swapaxes(k_tail, -1, -2) @ v_new  # :392

        for lvl in range(1, L):                             # naive.py:394-415
            if (n + 1) % int(firing_intervals[lvl]) != 0:
                continue
            keys, vals, bp, wp, gp = PROBES[promotion](
                S[lvl - 1], f(query_banks[lvl - 1]), f(key_projections[lvl - 1]),
                f(b_projections[lvl - 1]), f(w_projections[lvl - 1]),
                f(g_projections[lvl - 1]), int(n_queries_per_level[lvl - 1]))
            S[lvl] = update_step(S[lvl], keys, vals, bp, wp, gp)

    o = o[:, :, :T].transpose(0, 2, 1, 3)                  # naive.py:417
    final = np.stack(S, axis=2) if output_final_state else None
    return o, final
