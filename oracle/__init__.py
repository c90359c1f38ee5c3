"""CPU oracle for the nested-GDN forward hot path.

TEST INFRASTRUCTURE ONLY. Nothing in the product imports this package: only
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` use it, and only as the checker (or, for the baseline, as the
timed CPU restatement of the reference algorithm).

``naive_np`` is a numpy restatement of the reference's pure-torch oracle
(``nested_gdn2/ops/naive.py``) and its promotion probes
(``nested_gdn2/ops/probe.py``). Parity of this restatement is pinned against
golden vectors produced by the reference itself (``tests/golden/``).
``naive_torch`` is a differentiable torch restatement of the chunkwise oracle
(imported as ``oracle.naive_torch``); the backward's parity tests take
autograd through it, and its gradients are pinned to golden gradients taken
by autograd through the reference's oracle (``tests/golden/bwd_*.npz``).
"""

from .naive_np import (  # noqa: F401
    B_LOGIT_INIT,
    G_LOGIT_INIT,
    W_LOGIT_INIT,
    chunk_forward,
    gates,
    n_firings,
    n_groups,
    probe_learned,
    probe_merge,
    recurrent_forward,
    source_index,
    step,
    update_scan,
    update_step,
)
