"""Generate golden gradients from the reference's own pure-torch oracle.

Run once, in a checkout that has the reference project next to it:

    python tests/golden/make_golden_bwd.py /path/to/nested_recurrent_memory

Like ``make_golden.py`` it imports ``nested_gdn2.ops.naive`` (and the probes)
from the reference through stub parent packages, then takes torch autograd
through ``naive_chunk_nested_gdn2`` -- the check the reference applies to its
own backward (tests/ops/test_chunk.py:62-83, 94-111) -- on seeded fp32 CPU
inputs, and writes ``bwd_*.npz`` next to this script: the op inputs, the
upstream gradients ``d_o`` and ``d_final``, and ``grad_<input>`` for every
differentiable input (``grad_initial_state`` when one is given); and
``bwdupd_scan.npz`` for the write scan's backward (update_state_bwd).
"""

from __future__ import annotations

import pathlib
import sys

import numpy as np
import torch

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(HERE.parents[1]))

from make_golden import _import_reference  # noqa: E402

from nested_recurrent_memory_b200.synthetic import op_inputs  # noqa: E402

LEAVES = ("q", "k", "v", "g", "b", "w", "mix_weights", "query_banks", "key_projections",
          "b_projections", "w_projections", "g_projections")

# (name, B, T, H, K, V, L, N_MAX, firing, n_queries, promotion, with_init)
CASES = [
    ("bwd_l2_learned_init", 1, 128, 2, 32, 32, 2, 16, (1, 2), None, "learned", True),
    ("bwd_l3_learned_queries", 2, 256, 1, 32, 32, 3, 32, (1, 2, 4), (32, 16), "learned", False),
    ("bwd_l3_merge_init", 1, 256, 1, 32, 32, 3, 16, (1, 2, 4), None, "merge", True),
    ("bwd_l1", 1, 128, 2, 32, 16, 1, 16, (1,), None, "learned", True),
]


def update_case(naive):
    """update_state_bwd's contract (update_bwd.py:167-263): autograd through
    the reference's group scan over naive_update_step, in float64 as
    tests/ops/test_update_bwd.py:36-48 does. NG = NF + 1 (ragged) with an
    initial state."""
    gen = torch.Generator().manual_seed(21)
    B, NF, NG, H, K, V, N = 2, 4, 5, 2, 16, 32, 16
    r = lambda *s: torch.randn(*s, generator=gen, dtype=torch.float64)  # noqa: E731
    leaves = dict(keys=torch.nn.functional.normalize(r(B, NF, H, N, K), dim=-1),
                  values=r(B, NF, H, N, V) * V ** -0.5,
                  g=-torch.nn.functional.softplus(r(B, NF, H, K)),
                  b=torch.sigmoid(r(B, NF, H, N, K)), w=torch.sigmoid(r(B, NF, H, N, V)))
    init = r(B, H, K, V) * K ** -0.5
    leaves = {k: t.requires_grad_(True) for k, t in leaves.items()}
    init.requires_grad_(True)
    S, states = init, []
    for j in range(NG):
        states.append(S)
        if j < NF:
            S = naive.naive_update_step(S, leaves["keys"][:, j], leaves["values"][:, j],
                                        leaves["b"][:, j], leaves["w"][:, j], leaves["g"][:, j])
    states = torch.stack(states, 1)
    d_states = r(B, NG, H, K, V)
    d_final = r(B, H, K, V)
    ((states * d_states).sum() + (S * d_final).sum()).backward()
    arrays = {k: t.detach().numpy() for k, t in leaves.items()}
    arrays.update(initial_state=init.detach().numpy(), n_groups=NG, out_states=states.detach().numpy(),
                  out_final=S.detach().numpy(), d_states=d_states.numpy(), d_final=d_final.numpy())
    for k, t in leaves.items():
        arrays[f"grad_{k}"] = t.grad.numpy()
    arrays["grad_initial_state"] = init.grad.numpy()
    np.savez_compressed(HERE / "bwdupd_scan.npz", **arrays)
    print("bwdupd_scan", {k: v.shape for k, v in arrays.items() if k.startswith("grad_")})


def main(ref_root: str):
    naive, _ = _import_reference(ref_root)
    update_case(naive)
    for (name, B, T, H, K, V, L, N, firing, nq, promo, with_init) in CASES:
        inp = op_inputs(B, T, H, K, V, L, N, firing_intervals=firing, n_queries_per_level=nq,
                        seed=13)
        L = inp.pop("L")
        gen = torch.Generator().manual_seed(17)
        init = torch.randn(B, H, L, K, V, generator=gen) * 0.1 if with_init else None
        d_o = torch.randn(B, T, H, V, generator=gen)
        d_final = torch.randn(B, H, L, K, V, generator=gen) * 0.1
        leaves = {n: inp[n].detach().clone().requires_grad_(True) for n in LEAVES}
        args = dict(inp, **leaves)
        init_leaf = init.clone().requires_grad_(True) if init is not None else None
        o, s = naive.naive_chunk_nested_gdn2(
            **args, L=L, initial_state=init_leaf, output_final_state=True, chunk_size=64,
            promotion=promo)
        ((o * d_o).sum() + (s * d_final).sum()).backward()
        arrays = {n: (t.numpy() if torch.is_tensor(t) else np.asarray(t)) for n, t in inp.items()}
        arrays.update(L=L, promotion=promo, d_o=d_o.numpy(), d_final=d_final.numpy(),
                      out_o=o.detach().numpy(), out_final=s.detach().numpy())
        for n in LEAVES:
            gr = leaves[n].grad
            arrays[f"grad_{n}"] = (torch.zeros_like(leaves[n]) if gr is None else gr).numpy()
        if init is not None:
            arrays["initial_state"] = init.numpy()
            arrays["grad_initial_state"] = init_leaf.grad.numpy()
        np.savez_compressed(HERE / f"{name}.npz", **arrays)
        print(name, {k: v.shape for k, v in arrays.items() if k.startswith("grad_")})


if __name__ == "__main__":
    main(sys.argv[1])
