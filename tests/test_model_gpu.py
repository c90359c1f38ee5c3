"""The full-model harness (nested_recurrent_memory_b200/model.py) with this
package's op against the same model, same weights and inputs, whose token
mixer runs the CPU oracle instead: only the op differs between the two runs,
so the logits must agree within the op's own tolerance (fp32 1e-4 on the
CUDA-core path, 2e-2 with bf16 weights on the tensor-core path)."""

import pytest
import torch

import oracle
from _util import FP32_REL, LOWP_REL, rel_err
from nested_recurrent_memory_b200.model import ModelConfig, NestedGDN2ForCausalLM

pytestmark = pytest.mark.gpu


def oracle_op(q, k, v, g, b, w, mix_weights, query_banks, key_projections, b_projections,
              w_projections, g_projections, n_queries_per_level, firing_intervals, L, scale=None,
              initial_state=None, output_final_state=False, chunk_size=64, promotion="learned"):
    f = lambda t: t.detach().float().cpu().numpy()  # noqa: E731
    o, s = oracle.chunk_forward(
        f(q), f(k), f(v), f(g), f(b), f(w), f(mix_weights), f(query_banks), f(key_projections),
        f(b_projections), f(w_projections), f(g_projections), list(n_queries_per_level),
        list(firing_intervals), L, scale=scale,
        initial_state=None if initial_state is None else f(initial_state),
        output_final_state=True, promotion=promotion)
    return (torch.as_tensor(o, dtype=torch.float32).to(q.device, q.dtype),
            torch.as_tensor(s, dtype=torch.float32, device=q.device))


def _logits_both(cfg, dtype, B, T, seed):
    torch.manual_seed(seed)
    model = NestedGDN2ForCausalLM(cfg).cuda().to(dtype)
    ids = torch.randint(0, cfg.vocab_size, (B, T), generator=torch.Generator().manual_seed(seed)).cuda()
    with torch.no_grad():
        ours = model(ids).float()
        for layer in model.layers:
            layer.attn.op = oracle_op
        ref = model(ids).float()
    torch.cuda.synchronize()
    return ours.cpu().numpy(), ref.cpu().numpy()


@pytest.mark.parametrize("promotion", ["learned", "merge"])
def test_small_model_fp32_cuda_core_path(promotion):
    cfg = ModelConfig(vocab_size=256, hidden_size=128, num_hidden_layers=2, num_heads=2,
                      head_dim=64, num_levels=3, firing_intervals=(1, 2, 4),
                      n_queries_per_level=(16, 16), promotion=promotion)
    ours, ref = _logits_both(cfg, torch.float32, 2, 256, 0)
    assert rel_err(ours, ref) < FP32_REL


def test_bf16_model_tensor_core_path():
    cfg = ModelConfig(vocab_size=512, hidden_size=256, num_hidden_layers=2, num_heads=2,
                      head_dim=128, num_levels=3, firing_intervals=(1, 4, 16),
                      n_queries_per_level=(64, 64))
    ours, ref = _logits_both(cfg, torch.bfloat16, 1, 1024, 1)
    assert rel_err(ours, ref) < LOWP_REL


def test_config4_shapes_run():
    """BASELINE config 4's architecture (12 layers, d 1024, 8 x 128 heads,
    L 3, m 64, vocab 32000) on one short sequence: finite logits."""
    torch.manual_seed(2)
    model = NestedGDN2ForCausalLM(ModelConfig()).cuda().to(torch.bfloat16)
    ids = torch.randint(0, 32000, (1, 512), device="cuda")
    with torch.no_grad():
        logits = model(ids)
    assert logits.shape == (1, 512, 32000)
    assert torch.isfinite(logits.float()).all()
