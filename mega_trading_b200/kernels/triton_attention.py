"""B200 (sm_100a) causal grouped-query attention.

Drop-in mirror of ``mega_trading.kernels.triton_attention`` (duoan/mega-trading,
``src/mega_trading/kernels/triton_attention.py:12-111``): same function name,
signature, validation messages and autograd contract.  Forward and backward
are tcgen05/TMEM/TMA kernels for every shape with head_dim 32 or 64 in bf16 or
fp16 (the reference's Triton backward only covers one shape and otherwise
materialises fp32 T x T tensors, ``triton_attention.py:85-111``).
"""

from __future__ import annotations

import math
import warnings

import torch

from .. import _lib

__all__ = ["triton_attention", "attention"]

_SUPPORTED = {torch.bfloat16, torch.float16}


def _launch_fwd(q, k, v, repeats: int, scale: float):
    lib = _lib.load()
    B, Hq, T, D = q.shape
    Hkv = k.shape[1]
    o = torch.empty_like(q)
    lse = torch.empty((B, Hq, T), device=q.device, dtype=torch.float32)
    ws = torch.empty((int(lib.mt_attention_fwd_workspace_bytes(B, Hq, T, D)),), device=q.device, dtype=torch.uint8)
    status = _lib.status_word(q.device)
    tok = _lib.timer.start("attention_fwd", q.device, main_kernel=True)
    st = lib.mt_attention_fwd(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(), _lib.dtype_code(q.dtype),
        B, Hq, Hkv, T, D, _lib.i64_array(q.stride()), _lib.i64_array(k.stride()), _lib.i64_array(v.stride()),
        _lib.i64_array(o.stride()), float(scale), ws.data_ptr(), ws.numel(), status.data_ptr(),
        _lib.stream_ptr(q.device),
    )
    _lib.timer.stop(tok)
    _lib.check(st, "attention forward")
    return o, lse


def _launch_bwd(q, k, v, o, lse, do, scale: float, dq=None, dk=None, dv=None, rope=None):
    """Attention backward; with ``rope=(cos, sin)`` ([T, D/2] tables in q's dtype) q / k are the
    rotated inputs and dq / dk come back as the gradients of the un-rotated ones."""
    lib = _lib.load()
    B, Hq, T, D = q.shape
    Hkv = k.shape[1]
    dq = torch.empty_like(q) if dq is None else dq
    dk = torch.empty_like(k) if dk is None else dk
    dv = torch.empty_like(v) if dv is None else dv
    ws_bytes = int(lib.mt_attention_bwd_workspace_bytes(B, Hq, T, D))
    ws = torch.empty((max(ws_bytes, 16),), device=q.device, dtype=torch.uint8)
    status = _lib.status_word(q.device)
    tok = _lib.timer.start("attention_bwd", q.device, main_kernel=True)
    common = (
        q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(), do.data_ptr(), dq.data_ptr(),
        dk.data_ptr(), dv.data_ptr(), _lib.dtype_code(q.dtype), B, Hq, Hkv, T, D,
        _lib.i64_array(q.stride()), _lib.i64_array(k.stride()), _lib.i64_array(v.stride()),
        _lib.i64_array(o.stride()), _lib.i64_array(do.stride()), _lib.i64_array(dq.stride()),
        _lib.i64_array(dk.stride()), _lib.i64_array(dv.stride()), float(scale),
    )
    tail = (ws.data_ptr(), ws.numel(), status.data_ptr(), _lib.stream_ptr(q.device))
    if rope is None:
        st = lib.mt_attention_bwd(*common, *tail)
    else:
        cos, sin = rope
        if cos.dtype != q.dtype or sin.dtype != q.dtype or cos.stride(-1) != 1 or sin.stride() != cos.stride():
            raise ValueError("RoPE tables must be [T, D/2] in the query dtype with unit inner stride")
        st = lib.mt_attention_rope_bwd(*common, cos.data_ptr(), sin.data_ptr(), cos.stride(0), *tail)
    _lib.timer.stop(tok)
    _lib.check(st, "attention backward")
    return dq, dk, dv


#: number of inputs whose layout the TMA tensor maps cannot take (inner stride
#: not 1, an outer stride not a multiple of 8 elements, or a base address not
#: 16-byte aligned) and which were therefore copied to a contiguous tensor
layout_copies = 0


def _aligned_view(t: torch.Tensor) -> torch.Tensor:
    """Return ``t`` if the kernels accept its layout, else a contiguous copy
    (counted in ``layout_copies``; the first one also warns)."""
    global layout_copies
    s = t.stride()
    ok = s[3] == 1 and all(x % 8 == 0 and x > 0 for x in s[:3]) and t.data_ptr() % 16 == 0
    if ok:
        return t
    if layout_copies == 0:
        warnings.warn(f"triton_attention: an input with strides {tuple(s)} is copied to a contiguous tensor "
                      "(the sm_100a kernels read unit inner stride, outer strides that are multiples of 8 "
                      "elements and 16-byte aligned bases); see layout_copies", stacklevel=4)
    layout_copies += 1
    return t.contiguous()


class _CausalAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, query, key, value, repeats):
        q = _aligned_view(query)
        k = _aligned_view(key)
        v = _aligned_view(value)
        scale = 1.0 / math.sqrt(q.shape[-1])
        o, lse = _launch_fwd(q, k, v, repeats, scale)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.scale = scale
        return o

    @staticmethod
    def backward(ctx, grad_output):
        q, k, v, o, lse = ctx.saved_tensors
        do = _aligned_view(grad_output)
        dq, dk, dv = _launch_bwd(q, k, v, o, lse, do, ctx.scale)
        return dq, dk, dv, None


def triton_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, *, repeats: int) -> torch.Tensor:
    """Causal grouped-query attention on sm_100a (query [B,Hq,T,D], key/value [B,Hkv,T,D])."""
    if query.device.type != "cuda":
        raise RuntimeError("triton attention backend requires CUDA tensors")
    if query.dtype not in {torch.float16, torch.bfloat16, torch.float32}:
        raise RuntimeError("triton attention supports float16, bfloat16, and float32 tensors")
    if key.shape[1] * repeats != query.shape[1]:
        raise ValueError("query heads must equal key/value heads multiplied by repeats")
    if key.shape != value.shape:
        raise ValueError("key and value must have the same shape")
    if query.shape[0] != key.shape[0] or query.shape[2:] != key.shape[2:]:
        raise ValueError("query, key, and value must agree on batch, sequence, and head dimensions")
    _lib.require_cuda_sm100(query, "triton_attention")
    if query.dtype not in _SUPPORTED:
        raise RuntimeError("the sm_100a attention kernels take float16 or bfloat16 tensors")
    if key.dtype != query.dtype or value.dtype != query.dtype:
        raise RuntimeError("query, key and value must share one dtype")
    if query.shape[-1] not in (32, 64):
        raise RuntimeError("the sm_100a attention kernels support head_dim 32 or 64")
    return _CausalAttention.apply(query, key, value, int(repeats))


attention = triton_attention
