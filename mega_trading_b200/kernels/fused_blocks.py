"""Fused autograd nodes the B200 training model is built from.

``qkv_rope_attention`` takes the output of ONE projection GEMM against the
concatenated ``[q_proj; k_proj; v_proj]`` weights (``[B, T, (Hq + 2 Hkv) D]``),
applies RoPE to the q/k slices, runs causal GQA attention and returns O in the
``[B, T, Hq, D]`` physical layout (so ``O.transpose(1, 2).reshape(B, T, H)`` is
free).  Its backward writes dq, dk and dv straight into one packed
``[B, T, (Hq + 2 Hkv) D]`` gradient through strided views, so the backward of
the projection is again ONE GEMM and no gradient slices are copied or added;
the RoPE backward is folded into the attention backward's dq / dk epilogues.
Same math as the reference's q/k/v projections + ``RotaryEmbedding`` +
``triton_attention`` (``src/mega_trading/model.py:218-237, 286-294``).

``swiglu_packed`` is the SwiGLU gate on ``[N, 2I] = [gate | up]`` from one GEMM
against the concatenated ``[w1; w3]`` weights (``model.py:249-256``).
"""

from __future__ import annotations

import math

import torch

from .. import _lib
from . import triton_attention as _attn
from . import triton_ops as _ops


def _bthd(B: int, T: int, H: int, D: int, like: torch.Tensor) -> torch.Tensor:
    """Empty ``[B, H, T, D]`` view over ``[B, T, H, D]`` storage."""
    return torch.empty((B, T, H, D), device=like.device, dtype=like.dtype).transpose(1, 2)


def _split(qkv: torch.Tensor, hq: int, hkv: int, d: int):
    B, T, _ = qkv.shape
    q = qkv[..., : hq * d].view(B, T, hq, d).transpose(1, 2)
    k = qkv[..., hq * d:(hq + hkv) * d].view(B, T, hkv, d).transpose(1, 2)
    v = qkv[..., (hq + hkv) * d:].view(B, T, hkv, d).transpose(1, 2)
    return q, k, v


class _QKVRopeAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, cos, sin, hq, hkv, d):
        B, T, _ = qkv.shape
        q, k, v = _split(qkv, hq, hkv, d)
        q_rot = _bthd(B, T, hq, d, qkv)
        k_rot = _bthd(B, T, hkv, d, qkv)
        _ops._launch_rope(q, k, cos, sin, q_rot, k_rot, negate=False)
        scale = 1.0 / math.sqrt(d)
        o, lse = _attn._launch_fwd(q_rot, k_rot, v, hq // hkv, scale)
        ctx.save_for_backward(q_rot, k_rot, v, o, lse, cos, sin)
        ctx.dims = (hq, hkv, d)
        ctx.scale = scale
        return o

    @staticmethod
    def backward(ctx, grad_o):
        q_rot, k_rot, v, o, lse, cos, sin = ctx.saved_tensors
        hq, hkv, d = ctx.dims
        B, _, T, _ = q_rot.shape
        do = _attn._aligned_view(grad_o)
        dqkv = torch.empty((B, T, (hq + 2 * hkv) * d), device=q_rot.device, dtype=q_rot.dtype)
        dq, dk, dv = _split(dqkv, hq, hkv, d)
        # the RoPE backward runs inside the attention backward's dq / dk epilogues
        _attn._launch_bwd(q_rot, k_rot, v, o, lse, do, ctx.scale, dq=dq, dk=dk, dv=dv, rope=(cos, sin))
        return dqkv, None, None, None, None, None


def qkv_rope_attention(qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, heads: int, kv_heads: int,
                       head_dim: int) -> torch.Tensor:
    """Causal GQA attention of the RoPE-rotated q/k slices of a packed projection."""
    _lib.require_cuda_sm100(qkv, "qkv_rope_attention")
    if qkv.dim() != 3 or qkv.shape[-1] != (heads + 2 * kv_heads) * head_dim:
        raise ValueError("qkv must have shape [batch, time, (heads + 2 * kv_heads) * head_dim]")
    if qkv.dtype not in (torch.bfloat16, torch.float16) or not qkv.is_contiguous():
        raise ValueError("qkv must be a contiguous bf16/fp16 tensor")
    T = qkv.shape[1]
    cos2 = _ops._table_2d(cos, T, head_dim // 2, qkv.dtype)
    sin2 = _ops._table_2d(sin, T, head_dim // 2, qkv.dtype)
    return _QKVRopeAttention.apply(qkv, cos2, sin2, heads, kv_heads, head_dim)


class _SwiGLUPacked(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu):
        lib = _lib.load()
        inter = gu.shape[-1] // 2
        rows = gu.numel() // gu.shape[-1]
        y = torch.empty(gu.shape[:-1] + (inter,), device=gu.device, dtype=gu.dtype)
        st = lib.mt_swiglu_packed_fwd(gu.data_ptr(), y.data_ptr(), _lib.dtype_code(gu.dtype), rows, inter,
                                      _lib.stream_ptr(gu.device))
        _lib.check(st, "swiglu_packed forward")
        _lib.count(1)
        ctx.save_for_backward(gu)
        return y

    @staticmethod
    def backward(ctx, dy):
        lib = _lib.load()
        (gu,) = ctx.saved_tensors
        inter = gu.shape[-1] // 2
        rows = gu.numel() // gu.shape[-1]
        dy = dy.contiguous()
        dgu = torch.empty_like(gu)
        st = lib.mt_swiglu_packed_bwd(gu.data_ptr(), dy.data_ptr(), dgu.data_ptr(), _lib.dtype_code(gu.dtype), rows,
                                      inter, _lib.stream_ptr(gu.device))
        _lib.check(st, "swiglu_packed backward")
        _lib.count(1)
        return dgu


def swiglu_packed(gu: torch.Tensor) -> torch.Tensor:
    """``silu(gate) * up`` for ``gu = [gate | up]`` along the last dimension."""
    _lib.require_cuda_sm100(gu, "swiglu_packed")
    if gu.shape[-1] % 16 != 0 or not gu.is_contiguous() or gu.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("gu must be contiguous bf16/fp16 with a last dimension that is a multiple of 16")
    return _SwiGLUPacked.apply(gu)
