"""Full-model forward harness: the NestedGDN-2 language model around this
package's op (the caller side of the hot path).

A plain-torch restatement of the reference's layer and model,
nested_gdn2/layers/nested_gdn2.py:28-237 (``NestedGDN2Attention``) and
nested_gdn2/models/modeling_nested_gdn2.py:43-160 (block, model, LM head),
with the same parameter names and shapes so that a reference state dict
loads unchanged. fla's modules that the reference imports are restated from
their published definitions: ``ShortConvolution`` (depthwise causal
convolution with SiLU), ``RMSNorm``, ``FusedRMSNormGated`` (RMSNorm times a
sigmoid gate) and ``GatedMLP`` (SwiGLU, intermediate size
256 * ceil(hidden * ratio * 2/3 / 256)). Dense layers run as torch (cuBLAS)
GEMMs; the token mixer's op is ``chunk_nested_gdn2`` from this package
(hand-written sm_100a kernels) unless another op with the same signature is
passed in. Forward only, no decode cache.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn as nn
import torch.nn.functional as F

from .ops import chunk_nested_gdn2

__all__ = ["ModelConfig", "NestedGDN2Attention", "NestedGDN2Block", "NestedGDN2ForCausalLM"]


@dataclass
class ModelConfig:
    """The fields of NestedGDN2Config (configuration_nested_gdn2.py:14-47)
    that the forward reads; defaults are BASELINE config 4's."""
    vocab_size: int = 32000
    hidden_size: int = 1024
    num_hidden_layers: int = 12
    num_heads: int = 8
    head_dim: int = 128
    expand_v: float = 1.0
    conv_size: int = 4
    hidden_ratio: int = 4
    intermediate_size: int | None = None
    norm_eps: float = 1e-5
    initializer_range: float = 0.02
    num_levels: int = 3
    firing_intervals: tuple = (1, 4, 16)
    n_queries_per_level: tuple = field(default_factory=lambda: (64, 64))
    promotion: str = "learned"
    read_mix: str = "softmax"
    max_horizon: int | None = None


class ShortConvolution(nn.Module):
    """Depthwise causal 1-D convolution over time followed by SiLU (fla's
    ShortConvolution with activation="silu", no bias)."""

    def __init__(self, channels: int, kernel_size: int):
        super().__init__()
        self.kernel_size = kernel_size
        self.weight = nn.Parameter(torch.empty(channels, 1, kernel_size))

    def forward(self, x):  # [B, T, C]
        T = x.shape[1]
        y = F.conv1d(x.transpose(1, 2), self.weight, padding=self.kernel_size - 1,
                     groups=self.weight.shape[0])[..., :T]
        return F.silu(y).transpose(1, 2)


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)
        return (y * self.weight.float()).to(x.dtype)


class GatedRMSNorm(RMSNorm):
    """RMSNorm over the last dimension times sigmoid(gate) (fla's
    FusedRMSNormGated with activation="sigmoid")."""

    def forward(self, x, gate):
        return (super().forward(x).float() * torch.sigmoid(gate.float())).to(x.dtype)


class GatedMLP(nn.Module):
    """SwiGLU channel mixer (fla's GatedMLP, hidden_act="swish")."""

    def __init__(self, hidden: int, ratio: int, intermediate: int | None):
        super().__init__()
        if intermediate is None:
            intermediate = int(hidden * ratio * 2 / 3)
            intermediate = 256 * ((intermediate + 255) // 256)
        self.gate_proj = nn.Linear(hidden, intermediate, bias=False)
        self.up_proj = nn.Linear(hidden, intermediate, bias=False)
        self.down_proj = nn.Linear(intermediate, hidden, bias=False)

    def forward(self, x):
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class NestedGDN2Attention(nn.Module):
    """The token-mixing layer (nested_gdn2.py:28-237), short convolutions on."""

    def __init__(self, cfg: ModelConfig, op=None):
        super().__init__()
        self.cfg = cfg
        self.op = op or chunk_nested_gdn2
        self.L = L = cfg.num_levels
        H, K = cfg.num_heads, cfg.head_dim
        V = int(cfg.head_dim * cfg.expand_v)
        self.H, self.K, self.V = H, K, V
        self.key_dim, self.value_dim = H * K, H * V
        d = cfg.hidden_size
        self.q_proj = nn.Linear(d, L * self.key_dim, bias=False)
        self.k_proj = nn.Linear(d, self.key_dim, bias=False)
        self.v_proj = nn.Linear(d, self.value_dim, bias=False)
        self.q_conv1d = ShortConvolution(L * self.key_dim, cfg.conv_size)
        self.k_conv1d = ShortConvolution(self.key_dim, cfg.conv_size)
        self.v_conv1d = ShortConvolution(self.value_dim, cfg.conv_size)
        self.f_proj = nn.Sequential(nn.Linear(d, V, bias=False), nn.Linear(V, self.key_dim, bias=False))
        self.b_proj = nn.Linear(d, self.key_dim, bias=False)
        self.w_proj = nn.Linear(d, self.value_dim, bias=False)
        # nested_gdn2.py:66-71
        self.A_log = nn.Parameter(torch.log(torch.empty(H, dtype=torch.float32).uniform_(1, 16)))
        dt = torch.exp(torch.rand(self.key_dim) * (math.log(0.1) - math.log(0.001))
                       + math.log(0.001)).clamp(min=1e-4)
        self.dt_bias = nn.Parameter(dt + torch.log(-torch.expm1(-dt)))
        # nested_gdn2.py:73-92
        n_max = max(cfg.n_queries_per_level) if L > 1 else 1
        self.b_projections = nn.Parameter(torch.randn(L - 1, H, V, K) * V ** -0.5)
        self.w_projections = nn.Parameter(torch.randn(L - 1, H, V, V) * V ** -0.5)
        self.g_projections = nn.Parameter(torch.randn(L - 1, H, V, K) * V ** -0.5)
        self.query_banks = nn.Parameter(torch.randn(L - 1, H, n_max, K) * K ** -0.5)
        self.key_projections = nn.Parameter(torch.randn(L - 1, H, K, V) * V ** -0.5)
        self.n_queries_per_level = tuple(cfg.n_queries_per_level)
        self.firing_intervals = tuple(cfg.firing_intervals)
        self.mix_proj = nn.Linear(d, H * L, bias=False)
        self.g_proj = nn.Sequential(nn.Linear(d, V, bias=False), nn.Linear(V, self.value_dim, bias=True))
        self.o_norm = GatedRMSNorm(V, cfg.norm_eps)
        self.o_proj = nn.Linear(self.value_dim, d, bias=False)

    def forward(self, x, initial_state=None):
        """x [B, T, d] -> (output [B, T, d], final state [B, H, L, K, V])."""
        B, T, _ = x.shape
        H, K, V, L = self.H, self.K, self.V, self.L
        q = self.q_conv1d(self.q_proj(x)).reshape(B, T, L, H, K).transpose(2, 3)
        k = self.k_conv1d(self.k_proj(x)).reshape(B, T, H, K)
        v = self.v_conv1d(self.v_proj(x)).reshape(B, T, H, V)
        q = F.normalize(q, dim=-1).to(v.dtype)
        k = F.normalize(k, dim=-1).to(v.dtype)
        # nested_gdn2.py:142-150: per-channel log-decay in fp32, gates.
        g0 = F.softplus(self.f_proj(x).float() + self.dt_bias).reshape(B, T, H, K)
        g0 = -self.A_log.float().exp()[:, None] * g0
        if self.cfg.max_horizon:
            g0 = g0.clamp(max=-1.0 / self.cfg.max_horizon)
        b0 = self.b_proj(x).sigmoid().reshape(B, T, H, K)
        w0 = self.w_proj(x).sigmoid().reshape(B, T, H, V)
        logits = self.mix_proj(x).reshape(B, T, H, L)
        mix = (logits.sigmoid() if self.cfg.read_mix == "sigmoid" else logits.softmax(-1)).to(v.dtype)
        o, state = self.op(
            q=q, k=k, v=v, g=g0, b=b0, w=w0, mix_weights=mix,
            query_banks=self.query_banks, key_projections=self.key_projections,
            b_projections=self.b_projections, w_projections=self.w_projections,
            g_projections=self.g_projections, n_queries_per_level=self.n_queries_per_level,
            firing_intervals=self.firing_intervals, L=L, initial_state=initial_state,
            output_final_state=True, chunk_size=64, promotion=self.cfg.promotion)
        o = self.o_norm(o, self.g_proj(x).reshape(B, T, H, V))
        return self.o_proj(o.reshape(B, T, H * V)), state


class NestedGDN2Block(nn.Module):
    """Pre-norm token mixing and channel mixing with residuals
    (modeling_nested_gdn2.py:43-67)."""

    def __init__(self, cfg: ModelConfig, op=None):
        super().__init__()
        self.attn_norm = RMSNorm(cfg.hidden_size, cfg.norm_eps)
        self.attn = NestedGDN2Attention(cfg, op)
        self.mlp_norm = RMSNorm(cfg.hidden_size, cfg.norm_eps)
        self.mlp = GatedMLP(cfg.hidden_size, cfg.hidden_ratio, cfg.intermediate_size)

    def forward(self, h):
        a, _ = self.attn(self.attn_norm(h))
        h = h + a
        return h + self.mlp(self.mlp_norm(h))


class NestedGDN2ForCausalLM(nn.Module):
    """Embedding -> blocks -> RMSNorm -> LM head (modeling_nested_gdn2.py:93-160,
    203-268); weights N(0, initializer_range) as ``_init_weights``
    (modeling_nested_gdn2.py:76-90), except the layer's own A_log, dt_bias
    and promotion parameters."""

    def __init__(self, cfg: ModelConfig, op=None):
        super().__init__()
        self.cfg = cfg
        self.embeddings = nn.Embedding(cfg.vocab_size, cfg.hidden_size)
        self.layers = nn.ModuleList(NestedGDN2Block(cfg, op) for _ in range(cfg.num_hidden_layers))
        self.norm = RMSNorm(cfg.hidden_size, cfg.norm_eps)
        self.lm_head = nn.Linear(cfg.hidden_size, cfg.vocab_size, bias=False)
        for m in self.modules():
            if isinstance(m, (nn.Linear, nn.Embedding, ShortConvolution)):
                nn.init.normal_(m.weight, mean=0.0, std=cfg.initializer_range)
                if getattr(m, "bias", None) is not None:
                    nn.init.zeros_(m.bias)

    def forward(self, input_ids):
        h = self.embeddings(input_ids)
        for layer in self.layers:
            h = layer(h)
        return self.lm_head(self.norm(h))
