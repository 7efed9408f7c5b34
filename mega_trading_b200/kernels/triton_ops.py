"""B200 (sm_100a) implementations of the reference's non-attention operators.

Drop-in mirror of ``mega_trading.kernels.triton_ops`` (duoan/mega-trading,
``src/mega_trading/kernels/triton_ops.py``): same function names, argument
meaning, return values and autograd behaviour, backed by the hand-written CUDA
kernels in ``libmtb200.so`` instead of Triton.  Differences, all deliberate:

* There is no CPU / torch fallback: non-CUDA tensors raise ``RuntimeError``
  (the reference silently falls back, ``triton_ops.py:13-14, 52-53, 59-60``).
* Math is fp32 inside every kernel with one rounding per output.
* ``triton_fused_linear_cross_entropy`` returns an fp32 loss (the reference
  returns ``hidden.dtype``, ``triton_ops.py:401``) and needs no host sync for
  the valid-row count.
"""

from __future__ import annotations

import torch

from .. import _lib

__all__ = [
    "triton_rms_norm",
    "triton_add_rms_norm",
    "triton_apply_rope",
    "triton_swiglu_gate",
    "triton_fused_linear_cross_entropy",
    "rms_norm",
    "add_rms_norm",
]


def _require(t: torch.Tensor, op: str) -> None:
    _lib.require_cuda_sm100(t, op)


def _dev_stream(t: torch.Tensor) -> int:
    return _lib.stream_ptr(t.device)


# ---------------------------------------------------------------------------
# RMSNorm  (reference: triton_ops.py:11-15, :133-184)
# ---------------------------------------------------------------------------
def _rms_fwd(x: torch.Tensor, w: torch.Tensor, eps: float, out_dtype: torch.dtype) -> tuple[torch.Tensor, torch.Tensor]:
    lib = _lib.load()
    dim = x.shape[-1]
    rows = x.numel() // dim if dim else 0
    y = torch.empty(x.shape, device=x.device, dtype=out_dtype)
    rstd = torch.empty((rows,), device=x.device, dtype=torch.float32)
    st = lib.mt_rms_norm_fwd(
        x.data_ptr(), _lib.dtype_code(x.dtype), w.data_ptr(), _lib.dtype_code(w.dtype), y.data_ptr(),
        _lib.dtype_code(out_dtype), rstd.data_ptr(), rows, dim, float(eps), _dev_stream(x),
    )
    _lib.check(st, "rms_norm forward")
    return y, rstd


def _rms_bwd(x, w, rstd, dy, dx_dtype, residual_grad=None, branch_dtype=None):
    """dx (and dw); with ``branch_dtype`` also dx rounded to that dtype, written by the same kernel."""
    lib = _lib.load()
    dim = x.shape[-1]
    rows = x.numel() // dim
    dx = torch.empty(x.shape, device=x.device, dtype=dx_dtype)
    dx2 = None
    dw = torch.empty(w.shape, device=w.device, dtype=w.dtype)
    ws_bytes = int(lib.mt_rms_norm_bwd_workspace_bytes(rows, dim))
    ws = torch.empty((max(ws_bytes, 4),), device=x.device, dtype=torch.uint8)
    if residual_grad is None:
        st = lib.mt_rms_norm_bwd(
            x.data_ptr(), _lib.dtype_code(x.dtype), w.data_ptr(), _lib.dtype_code(w.dtype), rstd.data_ptr(),
            dy.data_ptr(), _lib.dtype_code(dy.dtype), dx.data_ptr(), _lib.dtype_code(dx_dtype), dw.data_ptr(),
            _lib.dtype_code(w.dtype), ws.data_ptr(), ws.numel(), rows, dim, _dev_stream(x),
        )
        _lib.check(st, "rms_norm backward")
    elif branch_dtype is None or branch_dtype == dx_dtype:
        st = lib.mt_add_rms_norm_bwd(
            x.data_ptr(), _lib.dtype_code(x.dtype), w.data_ptr(), _lib.dtype_code(w.dtype), rstd.data_ptr(),
            residual_grad.data_ptr(), _lib.dtype_code(residual_grad.dtype), dy.data_ptr(), _lib.dtype_code(dy.dtype),
            dx.data_ptr(), _lib.dtype_code(dx_dtype), dw.data_ptr(), _lib.dtype_code(w.dtype), ws.data_ptr(),
            ws.numel(), rows, dim, _dev_stream(x),
        )
        _lib.check(st, "add_rms_norm backward")
    else:
        if branch_dtype != dy.dtype:
            raise ValueError("the branch gradient takes the dtype of the normalised-output gradient")
        dx2 = torch.empty(x.shape, device=x.device, dtype=branch_dtype)
        st = lib.mt_add_rms_norm_bwd_dual(
            x.data_ptr(), _lib.dtype_code(x.dtype), w.data_ptr(), _lib.dtype_code(w.dtype), rstd.data_ptr(),
            residual_grad.data_ptr(), _lib.dtype_code(residual_grad.dtype), dy.data_ptr(), _lib.dtype_code(dy.dtype),
            dx.data_ptr(), _lib.dtype_code(dx_dtype), dx2.data_ptr(), dw.data_ptr(), _lib.dtype_code(w.dtype),
            ws.data_ptr(), ws.numel(), rows, dim, _dev_stream(x),
        )
        _lib.check(st, "add_rms_norm backward (dual)")
    if branch_dtype is not None:
        return dx, dw, (dx if dx2 is None else dx2)
    return dx, dw


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden, weight, eps, out_dtype):
        x = hidden.contiguous()
        w = weight.contiguous()
        y, rstd = _rms_fwd(x, w, eps, out_dtype)
        ctx.save_for_backward(x, w, rstd)
        ctx.in_dtype = hidden.dtype
        return y

    @staticmethod
    def backward(ctx, grad_output):
        x, w, rstd = ctx.saved_tensors
        dx, dw = _rms_bwd(x, w, rstd, grad_output.contiguous(), ctx.in_dtype)
        return dx, dw, None, None


def rms_norm(hidden: torch.Tensor, weight: torch.Tensor, *, eps: float, out_dtype: torch.dtype | None = None):
    """RMSNorm with an optional output dtype (e.g. fp32 residual in, bf16 out)."""
    _require(hidden, "rms_norm")
    if hidden.shape[-1] != weight.numel():
        raise ValueError("weight must have one entry per hidden feature")
    return _RMSNorm.apply(hidden, weight, float(eps), out_dtype or hidden.dtype)


def triton_rms_norm(hidden: torch.Tensor, weight: torch.Tensor, *, eps: float) -> torch.Tensor:
    """RMSNorm: ``hidden * rsqrt(mean(hidden^2) + eps) * weight`` (sm_100a kernels)."""
    return rms_norm(hidden, weight, eps=eps)


# ---------------------------------------------------------------------------
# Fused residual add + RMSNorm  (reference: triton_ops.py:18-42, :217-291)
# ---------------------------------------------------------------------------
class _AddRMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden, residual, weight, eps, out_dtype):
        lib = _lib.load()
        x = hidden.contiguous()
        r = residual.contiguous()
        w = weight.contiguous()
        dim = x.shape[-1]
        rows = x.numel() // dim if dim else 0
        new_res = torch.empty_like(r)  # residual dtype (may be wider than hidden's)
        normed = torch.empty(x.shape, device=x.device, dtype=out_dtype)
        rstd = torch.empty((rows,), device=x.device, dtype=torch.float32)
        st = lib.mt_add_rms_norm_fwd(
            x.data_ptr(), r.data_ptr(), _lib.dtype_code(x.dtype), w.data_ptr(), _lib.dtype_code(w.dtype),
            new_res.data_ptr(), _lib.dtype_code(r.dtype), normed.data_ptr(), _lib.dtype_code(out_dtype),
            rstd.data_ptr(), rows, dim, float(eps), _dev_stream(x),
        )
        _lib.check(st, "add_rms_norm forward")
        ctx.save_for_backward(new_res, w, rstd)
        ctx.hidden_dtype = hidden.dtype
        return new_res.view(residual.shape), normed.view(hidden.shape)

    @staticmethod
    def backward(ctx, grad_new_residual, grad_normed):
        new_res, w, rstd = ctx.saved_tensors
        if grad_new_residual is None:
            grad_new_residual = torch.zeros_like(new_res)
        if grad_normed is None:
            grad_normed = torch.zeros(new_res.shape, device=new_res.device, dtype=new_res.dtype)
        gn = grad_normed.contiguous()
        # both add inputs receive the same gradient (triton_ops.py:288-291); a
        # narrower hidden dtype gets its rounded copy from the same kernel
        branch = ctx.hidden_dtype if ctx.hidden_dtype == gn.dtype else None
        dx, dw, dh = _rms_bwd(new_res, w, rstd, gn, new_res.dtype,
                              residual_grad=grad_new_residual.to(new_res.dtype).contiguous(),
                              branch_dtype=branch or new_res.dtype)
        if dh.dtype != ctx.hidden_dtype:
            dh = dh.to(ctx.hidden_dtype)
        return dh, dx, dw, None, None


def add_rms_norm(hidden, residual, weight, *, eps: float, out_dtype: torch.dtype | None = None):
    """Fused ``new_residual = hidden + residual`` and ``RMSNorm(new_residual)``.

    ``residual`` may be wider than ``hidden`` (fp32 residual stream, bf16 branch
    output); ``new_residual`` takes the residual's dtype."""
    _require(hidden, "add_rms_norm")
    _require(residual, "add_rms_norm")
    if hidden.shape != residual.shape:
        raise ValueError("hidden and residual must have the same shape")
    if hidden.shape[-1] != weight.numel():
        raise ValueError("weight must have one entry per hidden feature")
    return _AddRMSNorm.apply(hidden, residual, weight, float(eps), out_dtype or hidden.dtype)


def triton_add_rms_norm(hidden: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, *,
                        eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """Fused residual-add + RMSNorm; returns ``(new_residual, normed)``."""
    _require(hidden, "triton_add_rms_norm")
    if hidden.dtype != residual.dtype:
        raise ValueError("hidden and residual must have the same dtype")
    return add_rms_norm(hidden, residual, weight, eps=eps)


# ---------------------------------------------------------------------------
# RoPE  (reference: triton_ops.py:45-54, :187-214, :477-525)
# ---------------------------------------------------------------------------
def _table_2d(t: torch.Tensor, seq: int, half: int, dtype: torch.dtype) -> torch.Tensor:
    t = t.to(dtype=dtype)
    t = t.reshape(-1, t.shape[-2], t.shape[-1])[0] if t.dim() > 2 else t
    if t.shape[0] < seq or t.shape[1] != half:
        raise ValueError(f"rope table of shape {tuple(t.shape)} does not cover [{seq}, {half}]")
    return t[:seq]


def _launch_rope(query, key, cos2, sin2, q_out, k_out, negate: bool) -> None:
    lib = _lib.load()
    B, Hq, T, D = query.shape
    Hk = key.shape[1]
    st = lib.mt_rope(
        query.data_ptr(), key.data_ptr(), cos2.data_ptr(), sin2.data_ptr(), q_out.data_ptr(), k_out.data_ptr(),
        _lib.dtype_code(query.dtype), B, Hq, Hk, T, D,
        _lib.i64_array(query.stride()), _lib.i64_array(key.stride()), _lib.i64_array(q_out.stride()),
        _lib.i64_array(k_out.stride()), _lib.i64_array(cos2.stride()), _lib.i64_array(sin2.stride()),
        1 if negate else 0, _dev_stream(query),
    )
    _lib.check(st, "rope")


class _RoPE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, query, key, cos, sin):
        T, D = query.shape[-2], query.shape[-1]
        cos2 = _table_2d(cos, T, D // 2, query.dtype)
        sin2 = _table_2d(sin, T, D // 2, query.dtype)
        q_out = torch.empty_like(query)
        k_out = torch.empty_like(key)
        _launch_rope(query, key, cos2, sin2, q_out, k_out, negate=False)
        ctx.save_for_backward(cos2, sin2)
        return q_out, k_out

    @staticmethod
    def backward(ctx, grad_query, grad_key):
        cos2, sin2 = ctx.saved_tensors
        gq_out = torch.empty_like(grad_query)
        gk_out = torch.empty_like(grad_key)
        _launch_rope(grad_query, grad_key, cos2, sin2, gq_out, gk_out, negate=True)
        return gq_out, gk_out, None, None


def triton_apply_rope(query: torch.Tensor, key: torch.Tensor, cos: torch.Tensor,
                      sin: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Rotate interleaved pairs of ``query`` [B,Hq,T,D] and ``key`` [B,Hk,T,D] by the RoPE tables."""
    _require(query, "triton_apply_rope")
    _require(key, "triton_apply_rope")
    if query.dim() != 4 or key.dim() != 4:
        raise ValueError("query and key must have shape [batch, heads, time, head_dim]")
    if query.shape[-1] != key.shape[-1] or query.shape[-1] % 2 != 0:
        raise ValueError("query and key must share an even head dimension")
    if query.shape[0] != key.shape[0] or query.shape[2] != key.shape[2]:
        raise ValueError("query and key must agree on batch and sequence length")
    if key.dtype != query.dtype:
        raise ValueError("query and key must have the same dtype")
    return _RoPE.apply(query, key, cos, sin)


# ---------------------------------------------------------------------------
# SwiGLU gate  (reference: triton_ops.py:57-61, :431-474)
# ---------------------------------------------------------------------------
class _SwiGLUGate(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gate, up):
        lib = _lib.load()
        g = gate.contiguous()
        u = up.contiguous()
        y = torch.empty_like(g)
        st = lib.mt_swiglu_fwd(g.data_ptr(), u.data_ptr(), y.data_ptr(), _lib.dtype_code(g.dtype), g.numel(),
                               _dev_stream(g))
        _lib.check(st, "swiglu forward")
        ctx.save_for_backward(g, u)
        return y

    @staticmethod
    def backward(ctx, grad_output):
        lib = _lib.load()
        g, u = ctx.saved_tensors
        dy = grad_output.contiguous()
        dg = torch.empty_like(g)
        du = torch.empty_like(u)
        st = lib.mt_swiglu_bwd(g.data_ptr(), u.data_ptr(), dy.data_ptr(), dg.data_ptr(), du.data_ptr(),
                               _lib.dtype_code(g.dtype), g.numel(), _dev_stream(g))
        _lib.check(st, "swiglu backward")
        return dg, du


def triton_swiglu_gate(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """SwiGLU gate ``silu(gate) * up`` (silu rounded to ``up``'s dtype before the product)."""
    _require(gate, "triton_swiglu_gate")
    _require(up, "triton_swiglu_gate")
    if gate.shape != up.shape:
        raise ValueError("gate and up must have the same shape")
    if gate.dtype != up.dtype:
        raise ValueError("gate and up must have the same dtype")
    return _SwiGLUGate.apply(gate, up)


# ---------------------------------------------------------------------------
# Fused linear + cross-entropy  (reference: triton_ops.py:64-92, :294-411)
# ---------------------------------------------------------------------------
def triton_fused_linear_cross_entropy(hidden: torch.Tensor, weight: torch.Tensor, labels: torch.Tensor, *,
                                      ignore_index: int = -100) -> torch.Tensor:
    """Mean cross-entropy of ``hidden @ weight.T`` against ``labels`` without materialising logits."""
    if hidden.ndim != 2:
        raise ValueError("hidden must have shape [rows, hidden_dim]")
    if weight.ndim != 2 or weight.shape[1] != hidden.shape[1]:
        raise ValueError("weight must have shape [vocab, hidden_dim] matching hidden's last dim")
    if labels.ndim != 1 or labels.shape[0] != hidden.shape[0]:
        raise ValueError("labels must be a 1D tensor with one entry per hidden row")
    if labels.dtype not in {torch.int32, torch.int64}:
        raise ValueError("labels must be an integer tensor")
    _require(hidden, "triton_fused_linear_cross_entropy")
    _require(weight, "triton_fused_linear_cross_entropy")
    from .fused_ce import fused_linear_cross_entropy

    return fused_linear_cross_entropy(hidden, weight, labels, ignore_index=int(ignore_index))
