"""Generate golden vectors from the reference's own pure-torch oracle.

Run once, in a checkout that has the reference project next to it:

    python tests/golden/make_golden.py /path/to/nested_recurrent_memory

It imports ``nested_gdn2.ops.naive`` and ``nested_gdn2.ops.probe`` from the
reference through stub parent packages (the reference's package ``__init__``
imports its HF model, which needs a newer flash-linear-attention than this
image has; the two op modules need torch only), runs them on seeded CPU
inputs and writes ``*.npz`` files next to this script. The tests only read
the ``.npz`` files; the reference is not needed at test time.

Each file holds the op inputs under their reference argument names, the
scalar arguments, and the reference outputs under ``out_*``.
"""

from __future__ import annotations

import os
import pathlib
import sys
import types

import numpy as np
import torch

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from nested_recurrent_memory_b200.synthetic import config_inputs, op_inputs  # noqa: E402

# (name, B, T, H, K, V, L, N_MAX, firing, n_queries, promotion, with_init)
CHUNK_CASES = [
    ("chunk_l2_learned", 1, 128, 2, 32, 32, 2, 16, (1, 2), None, "learned", False),
    ("chunk_l3_learned_init", 2, 128, 1, 32, 32, 3, 16, (1, 2, 4), None, "learned", True),
    ("chunk_l3_merge", 1, 256, 1, 32, 32, 3, 16, (1, 2, 4), None, "merge", False),
    ("chunk_l3_queries", 1, 256, 1, 32, 32, 3, 32, (1, 2, 4), (32, 16), "learned", False),
    ("chunk_l1", 1, 128, 2, 32, 32, 1, 16, (1,), None, "learned", True),
    ("chunk_ragged_t100", 1, 100, 1, 32, 32, 3, 16, (1, 1, 2), None, "learned", False),
    ("chunk_k64", 1, 128, 1, 64, 64, 2, 16, (1, 1), None, "merge", True),
]


PER_TOKEN = ("q", "k", "v", "g", "b", "w", "mix_weights")


def _import_reference(ref_root: str):
    os.environ["PYTHONDONTWRITEBYTECODE"] = "1"
    sys.dont_write_bytecode = True
    for name, sub in (("nested_gdn2", ""), ("nested_gdn2.ops", "ops")):
        mod = types.ModuleType(name)
        mod.__path__ = [os.path.join(ref_root, "nested_gdn2", sub)]
        sys.modules[name] = mod
    import nested_gdn2.ops.naive as naive
    import nested_gdn2.ops.probe as probe
    return naive, probe


def _np(d):
    return {k: (v.detach().cpu().numpy() if torch.is_tensor(v) else np.asarray(v))
            for k, v in d.items()}


def chunk_cases(naive):
    for (name, B, T, H, K, V, L, N, firing, nq, promo, init) in CHUNK_CASES:
        inp = op_inputs(B, T, H, K, V, L, N, firing_intervals=firing,
                        n_queries_per_level=nq, seed=7)
        L = inp.pop("L")
        init_t = None
        if init:
            gen = torch.Generator().manual_seed(11)
            init_t = torch.randn(B, H, L, K, V, generator=gen) * 0.1
        # naive.py:307 pads g along H rather than T (three pad pairs on a 4-D
        # tensor), so the reference oracle raises for T % 64 != 0. Zero-pad
        # the per-token inputs to whole chunks here, which is what its padding
        # intends (a zero token neither decays nor writes), and cut o back.
        pad = (-T) % 64
        padded = {n: (torch.nn.functional.pad(t, (0, 0) * (t.dim() - 2) + (0, pad))
                      if n in PER_TOKEN else t) for n, t in inp.items()}
        o, s = naive.naive_chunk_nested_gdn2(
            **padded, L=L, initial_state=init_t, output_final_state=True,
            chunk_size=64, promotion=promo)
        o = o[:, :T]
        rec_o, rec_s = naive.naive_recurrent_nested_gdn2(
            **inp, L=L, initial_state=init_t, output_final_state=True,
            chunk_size=64, promotion=promo)
        arrays = _np(inp)
        if init_t is not None:
            arrays["initial_state"] = init_t.numpy()
        arrays.update(L=L, promotion=promo, out_o=o.numpy(), out_final=s.numpy(),
                      out_rec_o=rec_o.numpy(), out_rec_final=rec_s.numpy())
        np.savez_compressed(HERE / f"{name}.npz", **arrays)
        print(name, {k: v.shape for k, v in arrays.items() if hasattr(v, "shape")})


def config0_case(naive):
    """Config 0 cut to T=256 and one head to keep the fixture small; the
    recipe and every other shape are the config's."""
    inp = config_inputs(1, 256, 1, 64, 64, 2, 64, (1, 4), dtype=torch.float32, seed=0)
    L = inp.pop("L")
    o, s = naive.naive_chunk_nested_gdn2(**inp, L=L, output_final_state=True, chunk_size=64)
    arrays = _np(inp)
    arrays.update(L=L, promotion="learned", out_o=o.numpy(), out_final=s.numpy())
    np.savez_compressed(HERE / "config0_t256_h1.npz", **arrays)


def update_case(naive):
    """update_state's contract: the group scan over naive_update_step
    (tests/ops/_update_ref.py:34-51), in float64 as the reference tests run it."""
    gen = torch.Generator().manual_seed(3)
    B, NF, NG, H, K, V, N = 2, 4, 5, 2, 16, 32, 16
    r = lambda *s: torch.randn(*s, generator=gen, dtype=torch.float64)  # noqa: E731
    keys = torch.nn.functional.normalize(r(B, NF, H, N, K), dim=-1)
    values = r(B, NF, H, N, V) * V ** -0.5
    g = -torch.nn.functional.softplus(r(B, NF, H, K))
    b = torch.sigmoid(r(B, NF, H, N, K))
    w = torch.sigmoid(r(B, NF, H, N, V))
    init = r(B, H, K, V) * K ** -0.5
    S = init
    states = []
    for j in range(NG):
        states.append(S)
        if j < NF:
            S = naive.naive_update_step(S, keys[:, j], values[:, j], b[:, j], w[:, j], g[:, j])
    np.savez_compressed(
        HERE / "update_scan.npz", keys=keys.numpy(), values=values.numpy(),
        g=g.numpy(), b=b.numpy(), w=w.numpy(), initial_state=init.numpy(),
        n_groups=NG, out_states=torch.stack(states, 1).numpy(), out_final=S.numpy())


def probe_case(probe):
    gen = torch.Generator().manual_seed(5)
    B, NF, H, K, V, N = 2, 3, 2, 16, 16, 8
    r = lambda *s: torch.randn(*s, generator=gen)  # noqa: E731
    args = dict(state_below=r(B, NF, H, K, V) * K ** -0.5,
                query_bank=r(H, 2 * N, K) * K ** -0.5, key_proj=r(H, K, V) * V ** -0.5,
                b_proj=r(H, V, K) * V ** -0.5, w_proj=r(H, V, V) * V ** -0.5,
                g_proj=r(H, V, K) * V ** -0.5)
    out = {}
    for arm in ("learned", "merge"):
        res = probe.PROBES[arm](**args, n_queries=N, out_dtype=torch.float32)
        for nm, t in zip(("keys", "values", "b", "w", "g"), res):
            out[f"out_{arm}_{nm}"] = t.contiguous().numpy()
    np.savez_compressed(HERE / "probes.npz", n_queries=N, **_np(args), **out)


def main():
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("NGDN2_REFERENCE", "")
    if not ref_root:
        raise SystemExit("usage: make_golden.py <reference checkout>")
    torch.set_num_threads(4)
    naive, probe = _import_reference(ref_root)
    chunk_cases(naive)
    config0_case(naive)
    update_case(naive)
    probe_case(probe)


if __name__ == "__main__":
    main()
