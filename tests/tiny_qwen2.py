"""Test scaffolding: a small Qwen2 causal LM with the reference's module tree
and parameter names (model/qwen2.py:91-123 RMSNorm, :769-794 MLP, :796-913
decoder layer, :915-931 backbone, :1160-1170 LM head), so the runner tests
can load the state dict that the reference model ran with.  The attention
class is injected: this package's Qwen2Attention, or a weight-only stand-in
for the swap test.
"""

from __future__ import annotations

from types import SimpleNamespace

import torch
import torch.nn as nn
import torch.nn.functional as F


class RMSNorm(nn.Module):
    def __init__(self, hidden_size: int, eps: float) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size))
        self.variance_epsilon = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        dt = x.dtype
        stat = torch.float32 if dt in (torch.float16, torch.bfloat16) else dt
        xs = x.to(stat)
        normed = xs * torch.rsqrt(xs.square().mean(dim=-1, keepdim=True) + self.variance_epsilon)
        return self.weight.to(dt) * normed.to(dt)


class MLP(nn.Module):
    def __init__(self, hidden: int, inter: int) -> None:
        super().__init__()
        self.gate_proj = nn.Linear(hidden, inter, bias=False)
        self.up_proj = nn.Linear(hidden, inter, bias=False)
        self.down_proj = nn.Linear(inter, hidden, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class DecoderLayer(nn.Module):
    def __init__(self, config, attn_cls) -> None:
        super().__init__()
        self.self_attn = attn_cls(config)
        self.mlp = MLP(config.hidden_size, config.intermediate_size)
        self.input_layernorm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(config.hidden_size, config.rms_norm_eps)


class Backbone(nn.Module):
    def __init__(self, config, attn_cls) -> None:
        super().__init__()
        self.config = config
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_size)
        self.layers = nn.ModuleList([DecoderLayer(config, attn_cls) for _ in range(config.num_hidden_layers)])
        self.norm = RMSNorm(config.hidden_size, config.rms_norm_eps)


class CausalLM(nn.Module):
    def __init__(self, config, attn_cls) -> None:
        super().__init__()
        self.model = Backbone(config, attn_cls)
        self.lm_head = nn.Linear(config.hidden_size, config.vocab_size, bias=False)


class WeightsOnlyAttention(nn.Module):
    """The reference attention's parameters (qkv_proj.{q,k,v}_proj with bias,
    o_proj) and nothing else: what swap_attention must carry over."""

    def __init__(self, config) -> None:
        super().__init__()
        h = config.hidden_size
        d = h // config.num_attention_heads
        self.qkv_proj = nn.Module()
        self.qkv_proj.q_proj = nn.Linear(h, config.num_attention_heads * d)
        self.qkv_proj.v_proj = nn.Linear(h, config.num_key_value_heads * d)
        self.qkv_proj.k_proj = nn.Linear(h, config.num_key_value_heads * d)
        self.o_proj = nn.Linear(h, h, bias=False)


def make_config(values: dict) -> SimpleNamespace:
    return SimpleNamespace(**values)
