"""Differentiable torch restatement of the reference's chunkwise nested GDN-2
oracle, for the backward's parity checks.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): never imported by the
product path. Gradients come from torch autograd through this restatement,
which is how the reference checks its own backward
(tests/ops/test_chunk.py:62-83: autograd through ``naive_chunk_nested_gdn2``).

Follows, by file:line within the reference project:

* ``nested_gdn2/ops/naive.py:7-39``    -- ``naive_update_step``;
* ``nested_gdn2/ops/naive.py:226-420`` -- ``naive_chunk_nested_gdn2``;
* ``nested_gdn2/ops/probe.py:34-136``  -- ``_gates``, ``probe_learned``,
  ``probe_merge``;
* ``tests/ops/_update_ref.py:34-51``   -- the group scan over the update step.

Arithmetic runs in ``dtype`` (float64 by default). Layouts are the
reference's: per-token tensors ``[B, T, H, ...]`` (q ``[B, T, H, L, K]``),
states ``[B, H, L, K, V]``. The forward is pinned to the numpy oracle and the
gradients to golden vectors produced by autograd through the reference's own
oracle (``tests/golden/make_golden_bwd.py``).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

# probe.py:28-31
B_LOGIT_INIT = -4.0
W_LOGIT_INIT = 0.0
G_LOGIT_INIT = -4.0


def gates(values, b_proj, w_proj, g_proj):
    """probe.py:34-66. values [..., N, V]; projections [V, K] / [V, V] / [V, K]
    of one head. Returns b [..., N, K], w [..., N, V], g [..., K]."""
    b = torch.sigmoid(values @ b_proj + B_LOGIT_INIT)
    w = torch.sigmoid(values @ w_proj + W_LOGIT_INIT)
    g = -F.softplus(values @ g_proj + G_LOGIT_INIT).mean(dim=-2)
    return b, w, g


def probe(promotion, state_below, query_bank, key_proj, b_proj, w_proj, g_proj, n_queries):
    """probe.py:69-136 for one head. state_below [B, K, V]; query_bank
    [N_max, K]; key_proj [K, V]. Returns keys [B, N, K], values [B, N, V],
    b, w, g."""
    if promotion == "merge":
        K = state_below.shape[-2]
        keys = torch.eye(K, dtype=state_below.dtype).expand(state_below.shape[0], K, K)
        values = state_below
    else:
        values = query_bank[:n_queries] @ state_below          # probe.py:97-98
        u = values @ key_proj.transpose(0, 1)                    # probe.py:99
        keys = F.normalize(u, dim=-1)                            # probe.py:100
    b, w, g = gates(values, b_proj, w_proj, g_proj)
    return keys, values, b, w, g


def update_step(state, keys, values, b, w, g):
    """naive.py:7-39: S' = e^g S - (K^T (K*b)) e^g S + K^T (V*w), per batch row.
    state [B, K, V]; keys/b [B, N, K]; values/w [B, N, V]; g [B, K]."""
    S = state * g.exp().unsqueeze(-1)
    gram = keys.transpose(-1, -2) @ (keys * b)
    return S - gram @ S + keys.transpose(-1, -2) @ (values * w)


def update_scan(keys, values, g, b, w, n_groups, initial_state=None):
    """tests/ops/_update_ref.py:34-51 (the reference's group loop over
    naive_update_step), differentiable. keys/b [B, NF, H, N, K]; values/w
    [B, NF, H, N, V]; g [B, NF, H, K]. Returns states [B, NG, H, K, V] (the
    state entering each group) and the final state [B, H, K, V]."""
    B, NF, H, _, K = keys.shape
    V = values.shape[-1]
    S = initial_state if initial_state is not None else torch.zeros(
        B, H, K, V, dtype=values.dtype)
    states = []
    for j in range(n_groups):
        states.append(S)
        if j < NF:
            S = torch.stack([update_step(S[:, h], keys[:, j, h], values[:, j, h], b[:, j, h],
                                         w[:, j, h], g[:, j, h]) for h in range(H)], dim=1)
    return torch.stack(states, dim=1), S


def chunk_forward(q, k, v, g, b, w, mix_weights, query_banks, key_projections, b_projections,
                  w_projections, g_projections, n_queries_per_level, firing_intervals, L,
                  scale=None, initial_state=None, promotion="learned", chunk_size=64,
                  dtype=torch.float64):
    """naive.py:226-420 (chunkwise forward, chunk_size 64), differentiable.

    Returns (o [B, T, H, V], final_state [B, H, L, K, V]) in ``dtype``.
    """
    B, T, H, _, K = q.shape
    V = v.shape[-1]
    C = chunk_size
    if scale is None:
        scale = K ** -0.5
    cast = lambda x: x.to(dtype)  # noqa: E731
    q, k, v, g, b, w, mix = (cast(x) for x in (q, k, v, g, b, w, mix_weights))
    qb, kp, bp, wp, gp = (cast(x) for x in (query_banks, key_projections, b_projections,
                                            w_projections, g_projections))
    NT = (T + C - 1) // C
    pad = NT * C - T
    if pad:   # naive.py:302-312: tokens past T are zeros
        pz = lambda x: F.pad(x, (0, 0) * (x.dim() - 2) + (0, pad))  # noqa: E731
        q, k, v, g, b, w, mix = (pz(x) for x in (q, k, v, g, b, w, mix))
    # [B, H, NT, C, ...]
    ch = lambda x: x.transpose(1, 2).reshape(B, H, NT, C, *x.shape[3:])  # noqa: E731
    q, k, v, g, b, w, mix = (ch(x) for x in (q, k, v, g, b, w, mix))
    q = q * scale
    q0 = q[..., 0, :]
    G = g.cumsum(-2)                                              # naive.py:329
    G_last = G[..., -1, :]
    dec = (G.unsqueeze(-2) - G.unsqueeze(-3)).clamp(max=0).exp()  # [.., i, j, K]
    strict = torch.tril(torch.ones(C, C, dtype=torch.bool), -1)
    causal = torch.tril(torch.ones(C, C, dtype=torch.bool), 0)
    A_kk = torch.einsum("...ik,...jk,...ijk->...ij", b * k, k, dec) * strict
    A = torch.eye(C, dtype=dtype) + A_kk
    rhs = torch.cat([w * v, k * b * G.exp()], dim=-1)
    UW = torch.linalg.solve_triangular(A, rhs, upper=False, unitriangular=True)
    U, W = UW[..., :V], UW[..., V:]
    Kt = k * (G_last.unsqueeze(-2) - G).exp()
    A_qk = torch.einsum("...ik,...jk,...ijk->...ij", q0, k, dec) * causal
    QG = q0 * G.exp()

    if initial_state is not None:
        S = [cast(initial_state[:, :, l]) for l in range(L)]
    else:
        S = [torch.zeros(B, H, K, V, dtype=dtype) for _ in range(L)]
    outs = []
    for n in range(NT):
        v_new = U[:, :, n] - W[:, :, n] @ S[0]                   # naive.py:376
        reads = [A_qk[:, :, n] @ v_new + QG[:, :, n] @ S[0]]     # naive.py:377-379
        for l in range(1, L):                                     # naive.py:381-385
            reads.append(q[:, :, n, :, l, :] @ S[l])
        mixn = mix[:, :, n]
        outs.append(sum(r * mixn[..., l:l + 1] for l, r in enumerate(reads)))
        S[0] = S[0] * G_last[:, :, n].exp().unsqueeze(-1) + Kt[:, :, n].transpose(-1, -2) @ v_new
        for l in range(1, L):                                     # naive.py:394-415
            if (n + 1) % int(firing_intervals[l]) != 0:
                continue
            new = []
            for h in range(H):
                keys, vals, bp_, wp_, gg = probe(
                    promotion, S[l - 1][:, h], qb[l - 1, h], kp[l - 1, h], bp[l - 1, h],
                    wp[l - 1, h], gp[l - 1, h], int(n_queries_per_level[l - 1]))
                new.append(update_step(S[l][:, h], keys, vals, bp_, wp_, gg))
            S[l] = torch.stack(new, dim=1)
    o = torch.stack(outs, dim=2).reshape(B, H, NT * C, V)[:, :, :T].transpose(1, 2)
    return o, torch.stack(S, dim=2)
