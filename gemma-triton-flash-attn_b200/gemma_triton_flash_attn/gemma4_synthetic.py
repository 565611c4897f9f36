"""Random-init Gemma-4-E2B-shaped decoder whose attention dispatches through
transformers' attention registry.

The stock transformers Gemma-4 config has one head count for every layer, so
the E2B mix of global layers (head_dim 512, 32 query / 4 KV heads) and
sliding layers (head_dim 256, 16 / 8 heads, window 512) is not expressible
with it. This module is a small HF-style decoder with exactly that layer mix:
pre-norm residual blocks with RMSNorm, rotary position embeddings, q/k
RMSNorm, a gated-GELU MLP and tied embeddings. Each attention layer calls
``ALL_ATTENTION_FUNCTIONS[config.attn_implementation]`` the way transformers'
own attention modules do, with q/k/v as (B, H, N, D) views of (B, N, H, D)
storage, ``scaling`` and ``sliding_window``; ``register_triton_attention()``
makes "triton_gqa" resolve to this library's adapter. The role mirrors the
reference's hand-built stack (flash_attn/gemma4_e2e.py).

Weights are random (no checkpoint is available offline); the decoder exists to
drive the attention path at the real shapes, end to end.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

__all__ = ["Gemma4SyntheticConfig", "Gemma4SyntheticDecoder"]


@dataclass
class Gemma4SyntheticConfig:
    vocab_size: int = 32768
    hidden_size: int = 2048
    num_layers: int = 35
    global_every: int = 5          # layers 4, 9, 14, ... are global
    global_heads: int = 32
    global_kv_heads: int = 4
    global_head_dim: int = 512
    local_heads: int = 16
    local_kv_heads: int = 8
    local_head_dim: int = 256
    sliding_window: int = 512
    intermediate_size: int = 8192
    rope_theta_local: float = 10_000.0
    rope_theta_global: float = 1_000_000.0
    rms_eps: float = 1e-6
    attn_implementation: str = "triton_gqa"

    def is_global(self, layer: int) -> bool:
        return (layer + 1) % self.global_every == 0


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.weight = nn.Parameter(torch.zeros(dim))
        self.eps = eps

    def forward(self, x):
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)
        return (y * (1.0 + self.weight.float())).to(x.dtype)


def _rope(x, cos, sin):
    """Rotate-half rotary embedding on the last dim; x is (B, N, H, D)."""
    d = x.shape[-1] // 2
    x1, x2 = x[..., :d], x[..., d:]
    return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1)


def _rope_tables(n, dim, theta, device, dtype):
    inv = 1.0 / (theta ** (torch.arange(0, dim, 2, device=device, dtype=torch.float32) / dim))
    ang = torch.arange(n, device=device, dtype=torch.float32)[:, None] * inv[None, :]
    return ang.cos().to(dtype)[None, :, None, :], ang.sin().to(dtype)[None, :, None, :]


class Attention(nn.Module):
    def __init__(self, cfg: Gemma4SyntheticConfig, layer: int):
        super().__init__()
        self.is_global = cfg.is_global(layer)
        self.num_heads = cfg.global_heads if self.is_global else cfg.local_heads
        self.num_kv_heads = cfg.global_kv_heads if self.is_global else cfg.local_kv_heads
        self.head_dim = cfg.global_head_dim if self.is_global else cfg.local_head_dim
        self.sliding_window = None if self.is_global else cfg.sliding_window
        self.rope_theta = cfg.rope_theta_global if self.is_global else cfg.rope_theta_local
        self.is_causal = True
        self.scaling = self.head_dim ** -0.5
        self.cfg = cfg
        h = cfg.hidden_size
        self.q_proj = nn.Linear(h, self.num_heads * self.head_dim, bias=False)
        self.k_proj = nn.Linear(h, self.num_kv_heads * self.head_dim, bias=False)
        self.v_proj = nn.Linear(h, self.num_kv_heads * self.head_dim, bias=False)
        self.o_proj = nn.Linear(self.num_heads * self.head_dim, h, bias=False)
        self.q_norm = RMSNorm(self.head_dim, cfg.rms_eps)
        self.k_norm = RMSNorm(self.head_dim, cfg.rms_eps)

    def forward(self, x, rope):
        from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

        b, n, _ = x.shape
        q = self.q_norm(self.q_proj(x).view(b, n, self.num_heads, self.head_dim))
        k = self.k_norm(self.k_proj(x).view(b, n, self.num_kv_heads, self.head_dim))
        v = self.v_proj(x).view(b, n, self.num_kv_heads, self.head_dim)
        cos, sin = rope
        q, k = _rope(q, cos, sin), _rope(k, cos, sin)
        attn = ALL_ATTENTION_FUNCTIONS[self.cfg.attn_implementation]
        out, _ = attn(self, q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), None,
                      dropout=0.0, scaling=self.scaling, sliding_window=self.sliding_window)
        return self.o_proj(out.reshape(b, n, -1))


class Block(nn.Module):
    def __init__(self, cfg: Gemma4SyntheticConfig, layer: int):
        super().__init__()
        self.attn_norm = RMSNorm(cfg.hidden_size, cfg.rms_eps)
        self.attn = Attention(cfg, layer)
        self.mlp_norm = RMSNorm(cfg.hidden_size, cfg.rms_eps)
        self.gate_proj = nn.Linear(cfg.hidden_size, cfg.intermediate_size, bias=False)
        self.up_proj = nn.Linear(cfg.hidden_size, cfg.intermediate_size, bias=False)
        self.down_proj = nn.Linear(cfg.intermediate_size, cfg.hidden_size, bias=False)

    def forward(self, x, rope):
        x = x + self.attn(self.attn_norm(x), rope)
        h = self.mlp_norm(x)
        return x + self.down_proj(F.gelu(self.gate_proj(h), approximate="tanh") * self.up_proj(h))


class Gemma4SyntheticDecoder(nn.Module):
    def __init__(self, cfg: Gemma4SyntheticConfig):
        super().__init__()
        self.cfg = cfg
        self.embed = nn.Embedding(cfg.vocab_size, cfg.hidden_size)
        self.layers = nn.ModuleList(Block(cfg, i) for i in range(cfg.num_layers))
        self.norm = RMSNorm(cfg.hidden_size, cfg.rms_eps)

    @torch.no_grad()
    def init_weights(self, seed: int = 0, std: float = 0.02):
        """Seeded N(0, std) matrices (drawn on the parameters' device); norm gains stay 0."""
        gens = {}
        for p in self.parameters():
            if p.dim() >= 2:
                g = gens.setdefault(p.device, torch.Generator(device=p.device).manual_seed(seed))
                p.copy_(torch.randn(p.shape, generator=g, device=p.device, dtype=torch.float32).mul_(std))
        return self

    def forward(self, input_ids):
        b, n = input_ids.shape
        x = self.embed(input_ids) * (self.cfg.hidden_size ** 0.5)
        dt, dev = x.dtype, x.device
        ropes = {}
        for layer in self.layers:
            a = layer.attn
            key = (a.head_dim, a.rope_theta)
            if key not in ropes:
                ropes[key] = _rope_tables(n, a.head_dim, a.rope_theta, dev, dt)
            x = layer(x, ropes[key])
        x = self.norm(x)
        return x @ self.embed.weight.t()
