"""Fused linear + cross-entropy on sm_100a (autograd wrapper of the C ABI).

Reference: ``triton_fused_linear_cross_entropy`` / ``_TritonFusedLinearCrossEntropy``
(duoan/mega-trading ``src/mega_trading/kernels/triton_ops.py:64-92, :294-411``).
The forward keeps every logit tile in TMEM (tcgen05 GEMM + online logsumexp);
the backward recomputes the tiles on chip and multiplies the 16-bit logit
gradient straight out of shared memory into dH and dW (fp32 accumulation), so
no ``[N, V]`` tensor exists at any point.  The valid-row count stays on the
device (no ``.item()``), the loss is fp32, and ``dW`` comes back in the
weight's dtype (fp32 for fp32 master weights, as the reference accumulates
``grad_weight`` in ``weight.dtype``, ``triton_ops.py:352-357``).
"""

from __future__ import annotations

import torch

from .. import _lib

_COMPUTE = {torch.bfloat16, torch.float16}


class _FusedLinearCrossEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden, weight, labels, ignore_index, compute_weight):
        lib = _lib.load()
        cdtype = hidden.dtype if hidden.dtype in _COMPUTE else torch.bfloat16
        h = hidden.to(cdtype).contiguous()
        src = weight if compute_weight is None else compute_weight
        w = src.detach().to(cdtype).contiguous()
        lab = labels.contiguous()
        n, k = h.shape
        v = w.shape[0]
        dev = h.device
        loss = torch.empty((), device=dev, dtype=torch.float32)
        lse2 = torch.empty((n + 3,), device=dev, dtype=torch.float32)
        ws = torch.empty((int(lib.mt_fused_ce_workspace_bytes(n, v)),), device=dev, dtype=torch.uint8)
        tok = _lib.timer.start("fused_ce_fwd", dev)
        st = lib.mt_fused_ce_fwd(
            h.data_ptr(), w.data_ptr(), lab.data_ptr(), 1 if lab.dtype == torch.int64 else 0, int(ignore_index),
            _lib.dtype_code(cdtype), n, v, k, loss.data_ptr(), lse2.data_ptr(), ws.data_ptr(), ws.numel(),
            _lib.status_word(dev).data_ptr(), _lib.stream_ptr(dev),
        )
        _lib.timer.stop(tok)
        _lib.check(st, "fused linear cross-entropy forward")
        ctx.save_for_backward(h, w, lab, lse2)
        ctx.ignore_index = int(ignore_index)
        ctx.dtypes = (hidden.dtype, weight.dtype)
        return loss

    @staticmethod
    def backward(ctx, grad_output):
        lib = _lib.load()
        h, w, lab, lse2 = ctx.saved_tensors
        n, k = h.shape
        v = w.shape[0]
        dev = h.device
        need_h, need_w = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        dh = torch.empty((n, k), device=dev, dtype=ctx.dtypes[0]) if need_h else None
        dw = torch.empty((v, k), device=dev, dtype=ctx.dtypes[1]) if need_w else None
        if not (need_h or need_w):
            return None, None, None, None, None
        go = grad_output.detach().to(device=dev, dtype=torch.float32).reshape(1).contiguous()
        ws = torch.empty((max(int(lib.mt_fused_ce_bwd_workspace_bytes(n, v, k)), 256),), device=dev,
                         dtype=torch.uint8)
        tok = _lib.timer.start("fused_ce_bwd", dev)
        st = lib.mt_fused_ce_bwd(
            h.data_ptr(), w.data_ptr(), lab.data_ptr(), 1 if lab.dtype == torch.int64 else 0, ctx.ignore_index,
            _lib.dtype_code(h.dtype), n, v, k, lse2.data_ptr(), go.data_ptr(),
            dh.data_ptr() if dh is not None else None, _lib.dtype_code(ctx.dtypes[0]),
            dw.data_ptr() if dw is not None else None, _lib.dtype_code(ctx.dtypes[1]),
            ws.data_ptr(), ws.numel(), _lib.status_word(dev).data_ptr(), _lib.stream_ptr(dev),
        )
        _lib.timer.stop(tok)
        _lib.check(st, "fused linear cross-entropy backward")
        return dh, dw, None, None, None


def fused_linear_cross_entropy(hidden: torch.Tensor, weight: torch.Tensor, labels: torch.Tensor, *,
                               ignore_index: int = -100, compute_weight: torch.Tensor | None = None) -> torch.Tensor:
    """Mean CE of ``hidden @ weight.T`` vs ``labels`` (fp32 scalar; 0 if every label is ignored).

    ``compute_weight``: an optional 16-bit copy of ``weight`` (same values rounded,
    e.g. the optimizer-maintained GEMM operand) that the kernels read instead of
    casting ``weight``; the gradient still goes to ``weight`` in its own dtype."""
    if compute_weight is not None and compute_weight.shape != weight.shape:
        raise ValueError("compute_weight must have the weight's shape")
    return _FusedLinearCrossEntropy.apply(hidden, weight, labels, int(ignore_index), compute_weight)
