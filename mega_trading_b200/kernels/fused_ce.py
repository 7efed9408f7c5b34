"""Fused linear + cross-entropy on sm_100a (autograd wrapper of the C ABI).

Reference: ``triton_fused_linear_cross_entropy`` / ``_TritonFusedLinearCrossEntropy``
(duoan/mega-trading ``src/mega_trading/kernels/triton_ops.py:64-92, :294-411``).
The forward keeps every logit tile in TMEM (tcgen05 GEMM + online logsumexp);
the backward recomputes the tiles on chip, writes only the bf16 logit gradient
and finishes with the two library GEMMs dH = dZ W and dW = dZ^T H.  The
valid-row count stays on the device (no ``.item()``), and the loss is fp32.
"""

from __future__ import annotations

import torch

from .. import _lib

_COMPUTE = {torch.bfloat16, torch.float16}


class _FusedLinearCrossEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden, weight, labels, ignore_index):
        lib = _lib.load()
        cdtype = hidden.dtype if hidden.dtype in _COMPUTE else torch.bfloat16
        h = hidden.to(cdtype).contiguous()
        w = weight.to(cdtype).contiguous()
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
        _lib.count(3)
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
        if n == 0 or not (need_h or need_w):
            return (torch.zeros_like(h).to(ctx.dtypes[0]) if need_h else None,
                    torch.zeros_like(w).to(ctx.dtypes[1]) if need_w else None, None, None)
        ld = (v + 7) // 8 * 8
        dz = torch.empty((n, ld), device=dev, dtype=h.dtype)
        go = grad_output.detach().to(device=dev, dtype=torch.float32).reshape(1).contiguous()
        tok = _lib.timer.start("fused_ce_grad_logits", dev)
        st = lib.mt_fused_ce_grad_logits(
            h.data_ptr(), w.data_ptr(), lab.data_ptr(), 1 if lab.dtype == torch.int64 else 0, ctx.ignore_index,
            _lib.dtype_code(h.dtype), n, v, k, lse2.data_ptr(), go.data_ptr(), dz.data_ptr(), ld,
            _lib.status_word(dev).data_ptr(), _lib.stream_ptr(dev),
        )
        _lib.timer.stop(tok)
        _lib.check(st, "fused linear cross-entropy backward")
        _lib.count(1)
        dzv = dz[:, :v]
        dh = torch.mm(dzv, w).to(ctx.dtypes[0]) if need_h else None
        dw = torch.mm(dzv.t(), h).to(ctx.dtypes[1]) if need_w else None
        return dh, dw, None, None


def fused_linear_cross_entropy(hidden: torch.Tensor, weight: torch.Tensor, labels: torch.Tensor, *,
                               ignore_index: int = -100) -> torch.Tensor:
    """Mean CE of ``hidden @ weight.T`` vs ``labels`` (fp32 scalar; 0 if every label is ignored)."""
    return _FusedLinearCrossEntropy.apply(hidden, weight, labels, int(ignore_index))
