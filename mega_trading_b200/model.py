"""Llama-style order-flow model on the sm_100a operators.

Same architecture and parameter names as the reference ``TradingModel``
(duoan/mega-trading ``src/mega_trading/model.py:20-331``), so state dicts move
between the two.  Every transformer operator on the hot path runs on this
package's kernels: RMSNorm (fp32 residual in, bf16 out), RoPE, causal GQA
attention (tcgen05), the SwiGLU gate and the fused linear + cross-entropy
(tcgen05, logits never in HBM).  The dense projections are library (cuBLAS)
bf16 GEMMs with fp32 accumulation, as in the reference.

Precision follows the reference's Accelerate bf16 autocast (``trainer.py:336``,
``:1009-1023``): fp32 master weights, bf16 GEMM operands, fp32 residual stream.
The bf16 operands are :class:`~mega_trading_b200.optim.PackedWeights` copies in
the layouts the GEMMs read (q/k/v stacked, gate/up interleaved); the fused
optimizer (``optim.AdamWShadow``) rewrites them as it updates the weights, so
the forward does no casting.  Dropout is 0 (the reference's rtx
configuration, ``configs/rtx.yaml``).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn

from .kernels import triton_attention as _attn
from .kernels import triton_ops as _ops
from .kernels.fused_blocks import (GATE_BLOCK, qkv_proj_rope_attention, qkv_rope_attention,
                                   qkv_rope_gemm_supported, swiglu_mlp, swiglu_mlp_supported, swiglu_packed)
from .kernels.fused_ce import fused_linear_cross_entropy
from .optim import PackedWeights


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

    @property
    def repeats(self) -> int:
        return self.attention_heads // self.kv_heads

    def matmul_params(self) -> int:
        h, i, d = self.hidden_dim, self.intermediate_dim, self.head_dim
        per_layer = h * h * 2 + 2 * h * self.kv_heads * d + 3 * h * i
        return self.layers * per_layer + self.vocab_size * h

    def train_flops_per_token(self, seq_len: int) -> float:
        """6 x GEMM parameters + causal attention (forward + backward = 3.5 x forward)."""
        attn = self.layers * 3.5 * 4 * self.attention_heads * self.head_dim * (seq_len + 1) / 2
        return 6.0 * self.matmul_params() + attn


# BASELINE configurations (model part)
CONFIGS = {
    "demo": ModelConfig(block_size=512, hidden_dim=256, layers=4, attention_heads=8, kv_heads=2,
                        intermediate_dim=688, rope_theta=10_000.0),
    "gqa12": ModelConfig(),
    "large24": ModelConfig(block_size=4096, hidden_dim=1024, layers=24, attention_heads=16, kv_heads=4,
                           intermediate_dim=2816),
}

_BF16 = torch.bfloat16


def _w(p: torch.Tensor) -> torch.Tensor:
    return p if p.dtype == _BF16 else p.to(_BF16)


def _packed(module: nn.Module, key: str, params: list[nn.Parameter], kind: str = "single") -> PackedWeights:
    """The module's cached bf16 copy of ``params`` (rebuilt if the parameters were replaced)."""
    pw = module.__dict__.get(key)
    if pw is None or len(pw.params) != len(params) or any(a is not b for a, b in zip(pw.params, params)) \
            or pw.kind != kind:
        pw = PackedWeights(params, kind, block_rows=GATE_BLOCK)
        module.__dict__[key] = pw
    return pw


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x: torch.Tensor, out_dtype: torch.dtype = _BF16) -> torch.Tensor:
        return _ops.rms_norm(x, self.weight, eps=self.eps, out_dtype=out_dtype)


class LlamaAttention(nn.Module):
    def __init__(self, cfg: ModelConfig) -> None:
        super().__init__()
        d = cfg.head_dim
        self.heads, self.kv_heads, self.head_dim, self.repeats = cfg.attention_heads, cfg.kv_heads, d, cfg.repeats
        self.q_proj = nn.Linear(cfg.hidden_dim, cfg.attention_heads * d, bias=False)
        self.k_proj = nn.Linear(cfg.hidden_dim, cfg.kv_heads * d, bias=False)
        self.v_proj = nn.Linear(cfg.hidden_dim, cfg.kv_heads * d, bias=False)
        self.o_proj = nn.Linear(cfg.hidden_dim, cfg.hidden_dim, bias=False)
        positions = torch.arange(cfg.block_size, dtype=torch.float32)
        inv_freq = 1.0 / (cfg.rope_theta ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
        freqs = torch.outer(positions, inv_freq)
        # tables rounded to the activation dtype, as model.py:290-291 does per call
        self.register_buffer("cos", freqs.cos().to(_BF16), persistent=False)
        self.register_buffer("sin", freqs.sin().to(_BF16), persistent=False)

    def packed_weights(self) -> list[PackedWeights]:
        return [_packed(self, "_qkv_bf16", [self.q_proj.weight, self.k_proj.weight, self.v_proj.weight], "rows"),
                _packed(self, "_o_bf16", [self.o_proj.weight])]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, T, H = x.shape
        # one projection GEMM against [q_proj; k_proj; v_proj]; RoPE + attention
        # read the packed output in place and write one packed gradient
        pw_qkv, pw_o = self.packed_weights()
        w_qkv = pw_qkv.get()
        if qkv_rope_gemm_supported(self.heads, self.kv_heads, self.head_dim, H):
            # RoPE in the projection GEMM's epilogue (tcgen05)
            o = qkv_proj_rope_attention(x, w_qkv, self.cos, self.sin, self.heads, self.kv_heads, self.head_dim)
        else:
            qkv = F.linear(x, w_qkv)
            o = qkv_rope_attention(qkv, self.cos, self.sin, self.heads, self.kv_heads, self.head_dim)
        # o is stored [B, T, H, D]: the transpose is free
        return F.linear(o.transpose(1, 2).reshape(B, T, H), pw_o.get())

    def forward_unfused(self, x: torch.Tensor) -> torch.Tensor:
        """Operator-by-operator path through the reference API mirror (same math)."""
        B, T, H = x.shape
        q = F.linear(x, _w(self.q_proj.weight)).view(B, T, self.heads, self.head_dim).transpose(1, 2)
        k = F.linear(x, _w(self.k_proj.weight)).view(B, T, self.kv_heads, self.head_dim).transpose(1, 2)
        v = F.linear(x, _w(self.v_proj.weight)).view(B, T, self.kv_heads, self.head_dim).transpose(1, 2)
        q, k = _ops.triton_apply_rope(q, k, self.cos[:T], self.sin[:T])
        o = _attn.triton_attention(q, k, v, repeats=self.repeats)
        return F.linear(o.transpose(1, 2).reshape(B, T, H), _w(self.o_proj.weight))


class SwiGLU(nn.Module):
    def __init__(self, cfg: ModelConfig) -> None:
        super().__init__()
        self.w1 = nn.Linear(cfg.hidden_dim, cfg.intermediate_dim, bias=False)
        self.w2 = nn.Linear(cfg.intermediate_dim, cfg.hidden_dim, bias=False)
        self.w3 = nn.Linear(cfg.hidden_dim, cfg.intermediate_dim, bias=False)

    def packed_weights(self) -> list[PackedWeights]:
        inter, hidden = self.w1.weight.shape
        # gate/up interleaved in GATE_BLOCK-row blocks for the fused GEMM, else stacked
        kind = "interleave" if swiglu_mlp_supported(inter, hidden) else "rows"
        return [_packed(self, "_w13_bf16", [self.w1.weight, self.w3.weight], kind),
                _packed(self, "_w2_bf16", [self.w2.weight])]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        pw13, pw2 = self.packed_weights()
        if pw13.kind == "interleave":
            # gate inside the projection GEMMs (tcgen05): w1 || w3 interleaved
            return swiglu_mlp(x, pw13.get(), pw2.get())
        # one GEMM against [w1; w3]; the gate reads [gate | up] in place
        gu = F.linear(x, pw13.get())
        return F.linear(swiglu_packed(gu), pw2.get())

    def forward_unfused(self, x: torch.Tensor) -> torch.Tensor:
        gate = F.linear(x, _w(self.w1.weight))
        up = F.linear(x, _w(self.w3.weight))
        return F.linear(_ops.triton_swiglu_gate(gate, up), _w(self.w2.weight))


class LlamaDecoderBlock(nn.Module):
    def __init__(self, cfg: ModelConfig) -> None:
        super().__init__()
        self.attention_norm = RMSNorm(cfg.hidden_dim, cfg.norm_eps)
        self.attention = LlamaAttention(cfg)
        self.ffn_norm = RMSNorm(cfg.hidden_dim, cfg.norm_eps)
        self.feed_forward = SwiGLU(cfg)

    def forward(self, h: torch.Tensor) -> torch.Tensor:
        h = h + self.attention(self.attention_norm(h))
        return h + self.feed_forward(self.ffn_norm(h))

    def forward_fused(self, h: torch.Tensor, x: torch.Tensor, next_norm: "RMSNorm") -> tuple[torch.Tensor, torch.Tensor]:
        """Same block with each residual add fused into the following RMSNorm.

        ``x`` is ``attention_norm(h)`` (already computed by the previous fused
        add); returns ``(h_out, next_norm(h_out))``."""
        h, x = _ops.add_rms_norm(self.attention(x), h, self.ffn_norm.weight, eps=self.ffn_norm.eps,
                                 out_dtype=_BF16)
        return _ops.add_rms_norm(self.feed_forward(x), h, next_norm.weight, eps=next_norm.eps, out_dtype=_BF16)


class TradingModelB200(nn.Module):
    """The reference ``TradingModel`` (dropout 0) on the sm_100a operators."""

    def __init__(self, cfg: ModelConfig) -> None:
        super().__init__()
        self.cfg = cfg
        self.token_embedding = nn.Embedding(cfg.vocab_size, cfg.hidden_dim)
        self.blocks = nn.ModuleList([LlamaDecoderBlock(cfg) for _ in range(cfg.layers)])
        self.norm = RMSNorm(cfg.hidden_dim, cfg.norm_eps)
        self.output = nn.Linear(cfg.hidden_dim, cfg.vocab_size, bias=False)
        self.apply(_init_weights)
        self.output.weight = self.token_embedding.weight

    def hidden_states(self, input_ids: torch.Tensor) -> torch.Tensor:
        if input_ids.ndim != 2:
            raise ValueError("input_ids must have shape [batch, time]")
        if input_ids.shape[1] > self.cfg.block_size:
            raise ValueError(f"sequence length {input_ids.shape[1]} exceeds block_size {self.cfg.block_size}")
        h = self.token_embedding(input_ids)  # fp32 residual stream
        if not self.blocks:
            return self.norm(h)
        # every residual add runs fused with the RMSNorm that follows it
        x = self.blocks[0].attention_norm(h)
        for i, block in enumerate(self.blocks):
            nxt = self.blocks[i + 1].attention_norm if i + 1 < len(self.blocks) else self.norm
            h, x = block.forward_fused(h, x, nxt)
        return x

    def packed_weights(self) -> list[PackedWeights]:
        """Every bf16 GEMM operand copy of the model (handed to ``optim.AdamWShadow``)."""
        out = [_packed(self, "_out_bf16", [self.output.weight])]
        for block in self.blocks:
            out += block.attention.packed_weights() + block.feed_forward.packed_weights()
        return out

    def forward(self, input_ids: torch.Tensor, labels: torch.Tensor | None = None) -> torch.Tensor:
        """Mean next-token loss when ``labels`` is given (the training entry), else logits."""
        if labels is not None:
            return self.forward_with_loss(input_ids, labels, return_logits=False)[0]
        return F.linear(self.hidden_states(input_ids), self.packed_weights()[0].get()).float()

    def forward_with_loss(self, input_ids: torch.Tensor, labels: torch.Tensor, *, return_logits: bool = False,
                          ignore_index: int = -100):
        """``(loss, logits | None)`` like the reference (model.py:84-132); the loss comes from the
        fused linear + cross-entropy unless logits are requested."""
        if labels.shape != input_ids.shape:
            raise ValueError("labels must match input_ids shape")
        normed = self.hidden_states(input_ids)
        pw_out = _packed(self, "_out_bf16", [self.output.weight])
        if not return_logits:
            flat = normed.reshape(-1, normed.shape[-1])
            # the kernels read the bf16 copy; dW lands in the fp32 (tied) weight unrounded
            return fused_linear_cross_entropy(flat, self.output.weight, labels.reshape(-1), ignore_index=ignore_index,
                                              compute_weight=pw_out.value()), None
        w_out = pw_out.get()
        logits = F.linear(normed, w_out).float()
        loss = F.cross_entropy(logits.reshape(-1, logits.shape[-1]), labels.reshape(-1), ignore_index=ignore_index)
        return loss, logits


def _init_weights(module: nn.Module) -> None:
    """N(0, 0.02) for linear and embedding weights (model.py:319-326)."""
    if isinstance(module, (nn.Linear, nn.Embedding)):
        nn.init.normal_(module.weight, mean=0.0, std=0.02)
