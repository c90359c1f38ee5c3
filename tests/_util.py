"""Shared helpers for the tests: golden-file loading and error measures."""

from __future__ import annotations

import pathlib

import numpy as np

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"

OP_ARGS = ("q", "k", "v", "g", "b", "w", "mix_weights", "query_banks", "key_projections",
           "b_projections", "w_projections", "g_projections", "n_queries_per_level",
           "firing_intervals")

# Parity bars. fp32 inputs: max |got - ref| <= 1e-4 * max |ref| (relative to
# the tensor's scale). bf16/fp16 operands with fp32 accumulation: 2e-2.
FP32_REL = 1e-4
LOWP_REL = 2e-2


def load_case(name):
    d = dict(np.load(GOLDEN / f"{name}.npz"))
    args = {k: d[k] for k in OP_ARGS}
    extra = dict(L=int(d["L"]), promotion=str(d["promotion"]),
                 initial_state=d.get("initial_state"))
    return args, extra, d


def chunk_case_names():
    return sorted(p.stem for p in GOLDEN.glob("chunk_*.npz")) + ["config0_t256_h1"]


def rel_err(got, ref):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    scale = max(np.abs(ref).max(), 1e-30)
    return float(np.abs(got - ref).max() / scale)
