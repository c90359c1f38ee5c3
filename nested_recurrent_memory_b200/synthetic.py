"""Seeded synthetic inputs for the nested GDN-2 forward.

Two recipes, both generated on the CPU in fp32 with a private
``torch.Generator`` (so results do not depend on the device or on global RNG
state) and then cast:

* ``op_inputs`` follows the reference op tests' recipe
  (tests/ops/_op_inputs.py:11-77): q ~ N(0,1) un-normalised, k L2-normalised,
  v * 0.5, g = logsigmoid(N(0,1)), b, w ~ U(0,1), mix = softmax, projections
  scaled by K^-1/2 / V^-1/2.
* ``config_inputs`` follows the benchmark configurations: q, k ~ N(0,1)
  L2-normalised, v ~ N(0,1), beta = sigmoid(N(0,1)) per token and head
  broadcast to b [.., K] and w [.., V], g = logsigmoid(N(0,1) + 3) per token
  and head broadcast to [.., K], mix = softmax(N(0,1)) over levels, query banks
  ~ N(0, 1/K), key projections ~ N(0, 1/V), gate projections zero (so the
  upper levels' gates are the probe's offsets, probe.py:28-31) unless
  ``gate_proj_std`` is given.

Both return a dict keyed by the reference op's argument names
(chunk.py:722-743) plus ``L``.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

__all__ = ["op_inputs", "config_inputs", "CONFIGS"]


def _randn(gen, *shape):
    return torch.randn(*shape, generator=gen, dtype=torch.float32, device=gen.device)


def _promo_params(gen, L, H, N, K, V, gate_std):
    n = max(L - 1, 0)
    qb = _randn(gen, n, H, N, K) * K ** -0.5
    kp = _randn(gen, n, H, K, V) * V ** -0.5
    if gate_std is None:
        bp = torch.zeros(n, H, V, K, device=gen.device)
        wp = torch.zeros(n, H, V, V, device=gen.device)
        gp = torch.zeros(n, H, V, K, device=gen.device)
    else:
        bp = _randn(gen, n, H, V, K) * gate_std
        wp = _randn(gen, n, H, V, V) * gate_std
        gp = _randn(gen, n, H, V, K) * gate_std
    return qb, kp, bp, wp, gp


def op_inputs(B, T, H, K, V, L, N_MAX, *, firing_intervals=None,
              n_queries_per_level=None, dtype=torch.float32, seed=42,
              device="cpu"):
    """The reference op tests' input recipe (tests/ops/_op_inputs.py:11-77)."""
    gen = torch.Generator().manual_seed(seed)
    q = _randn(gen, B, T, H, L, K)
    k = F.normalize(_randn(gen, B, T, H, K), dim=-1)
    v = _randn(gen, B, T, H, V) * 0.5
    g = F.logsigmoid(_randn(gen, B, T, H, K))
    b = torch.rand(B, T, H, K, generator=gen)
    w = torch.rand(B, T, H, V, generator=gen)
    mix = torch.softmax(_randn(gen, B, T, H, L), dim=-1)
    qb, kp, bp, wp, gp = _promo_params(gen, L, H, N_MAX, K, V, V ** -0.5)
    if n_queries_per_level is None:
        n_queries_per_level = [N_MAX] * (L - 1)
    if firing_intervals is None:
        firing_intervals = [1] + [2 ** i for i in range(1, L)]
    out = dict(q=q, k=k, v=v, g=g, b=b, w=w, mix_weights=mix, query_banks=qb,
               key_projections=kp, b_projections=bp, w_projections=wp,
               g_projections=gp)
    out = {n: t.to(dtype).to(device) for n, t in out.items()}
    out["n_queries_per_level"] = torch.tensor(list(n_queries_per_level), dtype=torch.int32)
    out["firing_intervals"] = torch.tensor(list(firing_intervals), dtype=torch.int32)
    out["L"] = L
    return out


def config_inputs(B, T, H, K, V, L, m, firing_intervals, *, dtype=torch.bfloat16,
                  seed=0, device="cpu", gate_proj_std=None, dense_gates=True,
                  gen_device="cpu"):
    """The benchmark configurations' input recipe (see module docstring).

    ``dense_gates=False`` returns b, w, g as stride-0 broadcast views of the
    per-token, per-head scalars instead of materialised tensors.
    ``gen_device`` is where the random numbers are drawn (a CUDA generator
    is much faster at benchmark sizes; its stream differs from the CPU one).
    """
    gen = torch.Generator(device=gen_device).manual_seed(seed)
    q = F.normalize(_randn(gen, B, T, H, L, K), dim=-1)
    k = F.normalize(_randn(gen, B, T, H, K), dim=-1)
    v = _randn(gen, B, T, H, V)
    beta = torch.sigmoid(_randn(gen, B, T, H))
    g = F.logsigmoid(_randn(gen, B, T, H) + 3.0)
    mix = torch.softmax(_randn(gen, B, T, H, L), dim=-1)
    qb, kp, bp, wp, gp = _promo_params(gen, L, H, m, K, V, gate_proj_std)
    cast = lambda t: t.to(dtype).to(device)  # noqa: E731
    out = dict(q=cast(q), k=cast(k), v=cast(v), mix_weights=cast(mix),
               query_banks=cast(qb), key_projections=cast(kp),
               b_projections=cast(bp), w_projections=cast(wp),
               g_projections=cast(gp))
    beta_c, g_c = cast(beta), cast(g)
    b_ = beta_c.unsqueeze(-1).expand(B, T, H, K)
    w_ = beta_c.unsqueeze(-1).expand(B, T, H, V)
    g_ = g_c.unsqueeze(-1).expand(B, T, H, K)
    if dense_gates:
        b_, w_, g_ = b_.contiguous(), w_.contiguous(), g_.contiguous()
    out.update(b=b_, w=w_, g=g_)
    out["n_queries_per_level"] = torch.tensor([m] * (L - 1), dtype=torch.int32)
    out["firing_intervals"] = torch.tensor(list(firing_intervals), dtype=torch.int32)
    out["L"] = L
    return out


# The benchmark configurations: (B, T, H, K, V, L, m, firing, dtype).
CONFIGS = {
    "config0": (1, 1024, 4, 64, 64, 2, 64, (1, 4), torch.float32),
    "config1": (8, 8192, 16, 128, 128, 3, 64, (1, 4, 16), torch.bfloat16),
    "config2_flat": (16, 4096, 16, 128, 128, 1, 64, (1,), torch.bfloat16),
    "config2_nested": (16, 4096, 16, 128, 128, 3, 64, (1, 4, 16), torch.bfloat16),
    "config3": (1, 65536, 32, 128, 128, 4, 128, (1, 4, 16, 64), torch.bfloat16),
}
