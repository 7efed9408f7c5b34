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
``qkv_proj_rope_attention`` also owns the projection: a tcgen05 GEMM whose
epilogue applies RoPE, so the rotated q/k are written once, straight from the
accumulator.

``swiglu_packed`` is the SwiGLU gate on ``[N, 2I] = [gate | up]`` from one GEMM
against the concatenated ``[w1; w3]`` weights (``model.py:249-256``).

``swiglu_mlp`` is the whole SwiGLU MLP ``w2(silu(w1 x) * w3 x)`` with the gate
inside two tcgen05 GEMMs: the gate/up projection writes the saved activation
and the W2 input in one pass, and the W2 input-gradient GEMM writes the packed
gate/up gradient directly, so neither the gate output nor its gradient makes
an extra HBM round trip.
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


def qkv_rope_gemm_supported(heads: int, kv_heads: int, head_dim: int, hidden: int) -> bool:
    return (heads + 2 * kv_heads) * head_dim % 256 == 0 and head_dim in (32, 64) and hidden % 8 == 0


def _qkv_rope_gemm(x2, w, cos2, sin2, seq, rot_cols, head_dim):
    lib = _lib.load()
    m, hidden = x2.shape
    n = w.shape[0]
    qkv = torch.empty((m, n), device=x2.device, dtype=x2.dtype)
    status = _lib.status_word(x2.device)
    st = lib.mt_qkv_rope_gemm(x2.data_ptr(), w.data_ptr(), qkv.data_ptr(), cos2.data_ptr(), sin2.data_ptr(),
                              cos2.stride(0), _lib.dtype_code(x2.dtype), m, hidden, n, rot_cols, seq, head_dim,
                              status.data_ptr(), _lib.stream_ptr(x2.device))
    _lib.check(st, "qkv_rope_gemm")
    return qkv


class _QKVProjRopeAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, cos2, sin2, hq, hkv, d):
        B, T, H = x.shape
        x2 = x.reshape(B * T, H).contiguous()
        qkv = _qkv_rope_gemm(x2, w, cos2, sin2, T, (hq + hkv) * d, d).view(B, T, -1)
        q_rot, k_rot, v = _split(qkv, hq, hkv, d)
        scale = 1.0 / math.sqrt(d)
        o, lse = _attn._launch_fwd(q_rot, k_rot, v, hq // hkv, scale)
        ctx.save_for_backward(x2, w, q_rot, k_rot, v, o, lse, cos2, sin2)
        ctx.dims = (hq, hkv, d)
        ctx.scale = scale
        return o

    @staticmethod
    def backward(ctx, grad_o):
        x2, w, q_rot, k_rot, v, o, lse, cos2, sin2 = ctx.saved_tensors
        hq, hkv, d = ctx.dims
        B, _, T, _ = q_rot.shape
        do = _attn._aligned_view(grad_o)
        n = (hq + 2 * hkv) * d
        dqkv = torch.empty((B, T, n), device=q_rot.device, dtype=q_rot.dtype)
        dq, dk, dv = _split(dqkv, hq, hkv, d)
        _attn._launch_bwd(q_rot, k_rot, v, o, lse, do, ctx.scale, dq=dq, dk=dk, dv=dv, rope=(cos2, sin2))
        d2 = dqkv.view(B * T, n)
        return d2.mm(w).view(B, T, -1), d2.t().mm(x2), None, None, None, None, None


def qkv_proj_rope_attention(x: torch.Tensor, w_qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, heads: int,
                            kv_heads: int, head_dim: int) -> torch.Tensor:
    """Causal GQA attention of ``x`` projected by ``w_qkv = [Wq; Wk; Wv]`` with RoPE in the GEMM epilogue."""
    _lib.require_cuda_sm100(x, "qkv_proj_rope_attention")
    if x.dim() != 3 or w_qkv.shape != ((heads + 2 * kv_heads) * head_dim, x.shape[-1]):
        raise ValueError("x must be [batch, time, hidden] and w_qkv [(heads + 2 * kv_heads) * head_dim, hidden]")
    if not qkv_rope_gemm_supported(heads, kv_heads, head_dim, x.shape[-1]):
        raise ValueError("qkv_proj_rope_attention needs (heads + 2 kv_heads) head_dim a multiple of 256")
    if x.dtype not in (torch.bfloat16, torch.float16) or w_qkv.dtype != x.dtype:
        raise ValueError("x and w_qkv must share a 16-bit dtype")
    T = x.shape[1]
    cos2 = _ops._table_2d(cos, T, head_dim // 2, x.dtype).contiguous()
    sin2 = _ops._table_2d(sin, T, head_dim // 2, x.dtype).contiguous()
    return _QKVProjRopeAttention.apply(x, w_qkv.contiguous(), cos2, sin2, heads, kv_heads, head_dim)


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
        return dgu


def swiglu_packed(gu: torch.Tensor) -> torch.Tensor:
    """``silu(gate) * up`` for ``gu = [gate | up]`` along the last dimension."""
    _lib.require_cuda_sm100(gu, "swiglu_packed")
    if gu.shape[-1] % 16 != 0 or not gu.is_contiguous() or gu.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("gu must be contiguous bf16/fp16 with a last dimension that is a multiple of 16")
    return _SwiGLUPacked.apply(gu)


GATE_BLOCK = 128  # interleave block of the fused gate/up weight


def interleave_gate_up(w1: torch.Tensor, w3: torch.Tensor) -> torch.Tensor:
    """``[2I, H]`` weight holding w1 and w3 in alternating blocks of 128 rows."""
    inter, hidden = w1.shape
    blocks = inter // GATE_BLOCK
    return torch.stack([w1.reshape(blocks, GATE_BLOCK, hidden), w3.reshape(blocks, GATE_BLOCK, hidden)],
                       dim=1).reshape(2 * inter, hidden)


def swiglu_mlp_supported(inter: int, hidden: int) -> bool:
    return inter % 256 == 0 and hidden % 8 == 0


class _SwiGLUMLP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w13, w2):
        lib = _lib.load()
        hidden = x.shape[-1]
        inter = w13.shape[0] // 2
        x2 = x.reshape(-1, hidden).contiguous()
        m = x2.shape[0]
        gu = torch.empty((m, 2 * inter), device=x.device, dtype=x.dtype)
        y = torch.empty((m, inter), device=x.device, dtype=x.dtype)
        status = _lib.status_word(x.device)
        st = lib.mt_swiglu_gemm_fwd(x2.data_ptr(), w13.data_ptr(), gu.data_ptr(), y.data_ptr(),
                                    _lib.dtype_code(x.dtype), m, hidden, inter, status.data_ptr(),
                                    _lib.stream_ptr(x.device))
        _lib.check(st, "swiglu_gemm forward")
        out = torch.nn.functional.linear(y, w2)
        ctx.save_for_backward(x2, w13, w2, gu, y)
        return out.view(*x.shape[:-1], w2.shape[0])

    @staticmethod
    def backward(ctx, dout):
        lib = _lib.load()
        x2, w13, w2, gu, y = ctx.saved_tensors
        hidden = x2.shape[1]
        inter = gu.shape[1] // 2
        d2 = dout.reshape(-1, w2.shape[0]).contiguous()
        dw2 = d2.t().mm(y)
        w2t = w2.t().contiguous()
        dgu = torch.empty_like(gu)
        status = _lib.status_word(gu.device)
        st = lib.mt_swiglu_gemm_bwd(d2.data_ptr(), w2t.data_ptr(), gu.data_ptr(), dgu.data_ptr(),
                                    _lib.dtype_code(gu.dtype), gu.shape[0], w2.shape[0], inter, status.data_ptr(),
                                    _lib.stream_ptr(gu.device))
        _lib.check(st, "swiglu_gemm backward")
        dx = dgu.mm(w13)
        dw13 = dgu.t().mm(x2)
        return dx.view(*dout.shape[:-1], hidden), dw13, dw2


def swiglu_mlp(x: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor) -> torch.Tensor:
    """``w2(silu(w1 x) * w3 x)`` for ``w13 = interleave_gate_up(w1, w3)`` (16-bit, same dtype as x)."""
    _lib.require_cuda_sm100(x, "swiglu_mlp")
    inter, hidden = w13.shape[0] // 2, x.shape[-1]
    if w13.shape != (2 * inter, hidden) or w2.shape != (hidden, inter):
        raise ValueError("w13 must be [2I, H] and w2 [H, I]")
    if not swiglu_mlp_supported(inter, hidden):
        raise ValueError("swiglu_mlp needs I a multiple of 256 and H a multiple of 8")
    if x.dtype not in (torch.bfloat16, torch.float16) or w13.dtype != x.dtype or w2.dtype != x.dtype:
        raise ValueError("x, w13 and w2 must share a 16-bit dtype")
    return _SwiGLUMLP.apply(x, w13.contiguous(), w2.contiguous())

