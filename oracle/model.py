"""CPU fp32 restatement of duoan/mega-trading's ``TradingModel`` and train step.

TEST INFRASTRUCTURE ONLY (tests/, __graft_entry__.smoke(), bench.py CPU legs).

Follows ``src/mega_trading/model.py``: tied token embedding / output head
(:51, :69-71), pre-norm decoder blocks (:184-186), GQA attention with RoPE
tables cast to the activation dtype (:218-237, :286-294), SwiGLU MLP
(:249-256), ``F.rms_norm`` (:266-269), N(0, 0.02) init (:319-326),
``forward_with_loss`` = mean next-token CE (:84-132).  The train step follows
``trainer.py:324-345`` (forward, CE, backward, fused AdamW ``:537-545``).
Parameter names match the reference so state dicts move between the two.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn

from . import ops


@dataclass(frozen=True)
class ModelConfig:
    vocab_size: int = 21504
    block_size: int = 2048
    hidden_dim: int = 768
    layers: int = 12
    attention_heads: int = 12
    kv_heads: int = 4
    intermediate_dim: int = 2048
    rope_theta: float = 500_000.0
    norm_eps: float = 1e-5

    @property
    def head_dim(self) -> int:
        return self.hidden_dim // self.attention_heads

    def matmul_params(self) -> int:
        """Parameters that take part in a GEMM per token (tied head counted once)."""
        h, i, d = self.hidden_dim, self.intermediate_dim, self.head_dim
        per_layer = h * h * 2 + 2 * h * self.kv_heads * d + 3 * h * i
        return self.layers * per_layer + self.vocab_size * h

    def train_flops_per_token(self, seq_len: int) -> float:
        """6 * matmul params + causal attention (fwd + bwd = 3.5 x fwd)."""
        attn = self.layers * 3.5 * 4 * self.attention_heads * self.head_dim * (seq_len + 1) / 2
        return 6.0 * self.matmul_params() + attn


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.rms_norm(x, self.weight, self.eps)


class Attention(nn.Module):
    def __init__(self, cfg: ModelConfig) -> None:
        super().__init__()
        d = cfg.head_dim
        self.heads, self.kv_heads, self.head_dim = cfg.attention_heads, cfg.kv_heads, d
        self.q_proj = nn.Linear(cfg.hidden_dim, cfg.attention_heads * d, bias=False)
        self.k_proj = nn.Linear(cfg.hidden_dim, cfg.kv_heads * d, bias=False)
        self.v_proj = nn.Linear(cfg.hidden_dim, cfg.kv_heads * d, bias=False)
        self.o_proj = nn.Linear(cfg.hidden_dim, cfg.hidden_dim, bias=False)
        cos, sin = ops.rope_tables(d, cfg.block_size, cfg.rope_theta)
        self.register_buffer("cos", cos, persistent=False)
        self.register_buffer("sin", sin, persistent=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, T, H = x.shape
        q = self.q_proj(x).view(B, T, self.heads, self.head_dim).transpose(1, 2)
        k = self.k_proj(x).view(B, T, self.kv_heads, self.head_dim).transpose(1, 2)
        v = self.v_proj(x).view(B, T, self.kv_heads, self.head_dim).transpose(1, 2)
        cos = self.cos[:, :, :T].to(q.dtype)
        sin = self.sin[:, :, :T].to(q.dtype)
        q, k = ops.rotate(q, cos, sin), ops.rotate(k, cos, sin)
        o = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=self.heads != self.kv_heads)
        return self.o_proj(o.transpose(1, 2).contiguous().view(B, T, H))


class SwiGLU(nn.Module):
    def __init__(self, cfg: ModelConfig) -> None:
        super().__init__()
        self.w1 = nn.Linear(cfg.hidden_dim, cfg.intermediate_dim, bias=False)
        self.w2 = nn.Linear(cfg.intermediate_dim, cfg.hidden_dim, bias=False)
        self.w3 = nn.Linear(cfg.hidden_dim, cfg.intermediate_dim, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.w2(F.silu(self.w1(x)) * self.w3(x))


class Block(nn.Module):
    def __init__(self, cfg: ModelConfig) -> None:
        super().__init__()
        self.attention_norm = RMSNorm(cfg.hidden_dim, cfg.norm_eps)
        self.attention = Attention(cfg)
        self.ffn_norm = RMSNorm(cfg.hidden_dim, cfg.norm_eps)
        self.feed_forward = SwiGLU(cfg)

    def forward(self, h: torch.Tensor) -> torch.Tensor:
        h = h + self.attention(self.attention_norm(h))
        return h + self.feed_forward(self.ffn_norm(h))


class TradingModelRef(nn.Module):
    """fp32 restatement of the reference ``TradingModel`` (dropout 0)."""

    def __init__(self, cfg: ModelConfig) -> None:
        super().__init__()
        self.cfg = cfg
        self.token_embedding = nn.Embedding(cfg.vocab_size, cfg.hidden_dim)
        self.blocks = nn.ModuleList([Block(cfg) for _ in range(cfg.layers)])
        self.norm = RMSNorm(cfg.hidden_dim, cfg.norm_eps)
        self.output = nn.Linear(cfg.hidden_dim, cfg.vocab_size, bias=False)
        self.apply(_init_weights)
        self.output.weight = self.token_embedding.weight

    def hidden_states(self, input_ids: torch.Tensor) -> torch.Tensor:
        h = self.token_embedding(input_ids)
        for block in self.blocks:
            h = block(h)
        return self.norm(h)

    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        return self.output(self.hidden_states(input_ids))

    def forward_with_loss(self, input_ids: torch.Tensor, labels: torch.Tensor, *, ignore_index: int = -100):
        normed = self.hidden_states(input_ids)
        flat = normed.reshape(-1, normed.shape[-1])
        return ops.linear_cross_entropy(flat, self.output.weight, labels.reshape(-1), ignore_index), None


def _init_weights(module: nn.Module) -> None:
    if isinstance(module, (nn.Linear, nn.Embedding)):
        nn.init.normal_(module.weight, mean=0.0, std=0.02)


def make_optimizer(model: nn.Module, lr: float = 2e-4, weight_decay: float = 0.01) -> torch.optim.Optimizer:
    """AdamW with the reference's rtx settings (configs/rtx.yaml, trainer.py:537-545)."""
    return torch.optim.AdamW(model.parameters(), lr=lr, betas=(0.9, 0.999), eps=1e-8, weight_decay=weight_decay)


def train_step(model: TradingModelRef, opt: torch.optim.Optimizer, input_ids: torch.Tensor,
               labels: torch.Tensor) -> torch.Tensor:
    """One full step: forward, mean CE, backward, AdamW update."""
    loss, _ = model.forward_with_loss(input_ids, labels)
    loss.backward()
    opt.step()
    opt.zero_grad(set_to_none=True)
    return loss.detach()


def seq_flops(cfg: ModelConfig, seq_len: int) -> float:
    return cfg.train_flops_per_token(seq_len) * seq_len


def _check() -> None:  # pragma: no cover - documentation aid
    assert math.isclose(ModelConfig().matmul_params(), 92_012_544, rel_tol=0, abs_tol=0)
