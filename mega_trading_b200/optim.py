"""Fused AdamW on fp32 master weights that also writes the 16-bit weight copies.

The reference steps ``torch.optim.AdamW(fused=True)`` (duoan/mega-trading
``src/mega_trading/trainer.py:535-545``) and its bf16 autocast casts every
weight again in every forward (``trainer.py:336``).  ``AdamWShadow`` keeps the
same update rule and state (``step``, ``exp_avg``, ``exp_avg_sq`` per
parameter) and, in the same kernel (``mt_adamw_step``), rounds each updated
weight into the bf16 copy the projection GEMMs read -- including the packed
layouts of :class:`PackedWeights` (q/k/v rows stacked, gate/up rows
interleaved in blocks) -- so the forward does no casting or packing.

:class:`PackedWeights` owns one such bf16 tensor built from one or more fp32
parameters.  ``get()`` returns it inside the autograd graph: the forward reads
it as is and the backward hands each parameter its fp32 slice of the
gradient.  The copy is reused across forwards only while a live
``AdamWShadow`` owns it, and then only until a parameter's version counter
moves (initialisation, ``load_state_dict``, in-place edits); without an owner
it is rebuilt with torch ops in every forward, because other optimizers may
update weights without advancing version counters (torch's fused AdamW does
not).
"""

from __future__ import annotations

import math
import weakref
from dataclasses import dataclass

import torch

from . import _lib

_BF16 = torch.bfloat16


@dataclass
class _Part:
    """Where one parameter's elements live in a packed copy: blocks of ``block``
    elements starting at ``start``, ``stride`` elements apart."""

    param: torch.nn.Parameter
    start: int
    block: int
    stride: int


class _PackedGrad(torch.autograd.Function):
    @staticmethod
    def forward(ctx, packed_obj, packed, *params):
        ctx.obj = packed_obj
        return packed.view_as(packed)

    @staticmethod
    def backward(ctx, grad):
        return (None, None, *ctx.obj.split_grad(grad))


class PackedWeights:
    """A bf16 copy of one or more fp32 parameters in the layout a GEMM reads.

    ``kind``: ``"rows"`` stacks the parameters' rows (q/k/v projection),
    ``"interleave"`` alternates blocks of ``block_rows`` rows of two
    parameters (gate/up projection), ``"single"`` is one parameter."""

    def __init__(self, params: list[torch.nn.Parameter], kind: str = "single", block_rows: int = 128) -> None:
        self.params = list(params)
        self.kind = kind
        self.block_rows = block_rows
        cols = self.params[0].shape[-1]
        if any(p.dim() != 2 or p.shape[1] != cols for p in self.params):
            raise ValueError("packed weights take 2-D parameters with one column count")
        if kind == "interleave" and (len(self.params) != 2 or self.params[0].shape != self.params[1].shape
                                     or self.params[0].shape[0] % block_rows):
            raise ValueError("interleaving takes two parameters of equal shape, rows a multiple of the block")
        self.rows = sum(p.shape[0] for p in self.params)
        self.cols = cols
        self.tensor: torch.Tensor | None = None
        self._versions: list[int] = []
        self._owner = None  # weak reference to the AdamWShadow that keeps this copy current

    def __getstate__(self):
        # a copy (deepcopy, pickle) is owned by no optimizer and rebuilds its tensor
        state = dict(self.__dict__)
        state.update(tensor=None, _versions=[], _owner=None)
        return state

    # -------- layout
    def parts(self) -> list[_Part]:
        out = []
        if self.kind == "interleave":
            blk = self.block_rows * self.cols
            for i, p in enumerate(self.params):
                out.append(_Part(p, i * blk, blk, 2 * blk))
        else:
            row = 0
            for p in self.params:
                n = p.numel()
                out.append(_Part(p, row * self.cols, n, n))
                row += p.shape[0]
        return out

    def pack(self) -> torch.Tensor:
        """The packed copy computed with torch ops (also the oracle of the layout)."""
        ps = [p.detach() for p in self.params]
        if self.kind == "interleave":
            a, b = ps
            r = self.block_rows
            w = torch.stack([a.reshape(-1, r, self.cols), b.reshape(-1, r, self.cols)], dim=1)
            return w.reshape(self.rows, self.cols).to(_BF16)
        return torch.cat(ps, dim=0).to(_BF16) if len(ps) > 1 else ps[0].to(_BF16)

    def split_grad(self, grad: torch.Tensor) -> list[torch.Tensor]:
        g = grad.float()
        if self.kind == "interleave":
            r = self.block_rows
            v = g.reshape(-1, 2, r, self.cols)
            return [v[:, i].reshape(self.params[i].shape) for i in range(2)]
        out, row = [], 0
        for p in self.params:
            out.append(g[row:row + p.shape[0]])
            row += p.shape[0]
        return out

    # -------- freshness
    @property
    def owned(self) -> bool:
        return self._owner is not None and self._owner() is not None

    def _stale(self) -> bool:
        t = self.tensor
        if t is None or t.device != self.params[0].device or not self.owned:
            return True
        return any(p._version != v for p, v in zip(self.params, self._versions))

    def refresh(self) -> None:
        with torch.no_grad():
            packed = self.pack()
            if self.tensor is None or self.tensor.device != packed.device:
                self.tensor = packed.contiguous()
            else:
                self.tensor.copy_(packed)
        self.mark_fresh()

    def mark_fresh(self) -> None:
        self._versions = [p._version for p in self.params]

    def get(self) -> torch.Tensor:
        """The packed bf16 weights as a differentiable function of the parameters."""
        if self._stale():
            self.refresh()
        if torch.is_grad_enabled() and any(p.requires_grad for p in self.params):
            return _PackedGrad.apply(self, self.tensor, *self.params)
        return self.tensor

    def value(self) -> torch.Tensor:
        """The current packed bf16 weights outside the autograd graph (for an operator
        that sends its weight gradient to the fp32 parameter itself)."""
        if self._stale():
            self.refresh()
        return self.tensor


class AdamWShadow(torch.optim.Optimizer):
    """``torch.optim.AdamW`` (decoupled weight decay) on fp32 CUDA parameters in one
    kernel launch per step, writing the bf16 copies of ``packed`` as it goes."""

    def __init__(self, params, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 1e-2, packed: list[PackedWeights] | None = None) -> None:
        if lr < 0 or eps < 0 or weight_decay < 0 or not (0 <= betas[0] < 1 and 0 <= betas[1] < 1):
            raise ValueError("invalid AdamW hyper-parameters")
        super().__init__(params, dict(lr=lr, betas=tuple(betas), eps=eps, weight_decay=weight_decay))
        self.packed = list(packed or [])
        owned = {id(p) for g in self.param_groups for p in g["params"]}
        for pw in self.packed:
            if any(id(p) not in owned for p in pw.params):
                raise ValueError("every parameter of a packed copy must be stepped by this optimizer")
            pw._owner = weakref.ref(self)
        self._table_key = None
        self._table = None

    def _shadow_map(self) -> dict[int, tuple[PackedWeights, _Part]]:
        out = {}
        for pw in self.packed:
            if pw._stale():
                pw.refresh()
            for part in pw.parts():
                out[id(part.param)] = (pw, part)
        return out

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        lib = _lib.load()
        shadows = self._shadow_map()
        for group in self.param_groups:
            beta1, beta2 = group["betas"]
            by_step: dict[int, list] = {}
            for p in group["params"]:
                if p.grad is None:
                    continue
                if p.dtype != torch.float32 or p.grad.dtype != torch.float32 or not p.is_cuda:
                    raise RuntimeError("AdamWShadow updates fp32 CUDA parameters with fp32 gradients")
                if p.grad.is_sparse:
                    raise RuntimeError("AdamWShadow does not take sparse gradients")
                st = self.state[p]
                if not st:
                    st["step"] = torch.tensor(0.0)
                    st["exp_avg"] = torch.zeros_like(p, memory_format=torch.contiguous_format)
                    st["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.contiguous_format)
                st["step"] += 1
                by_step.setdefault(int(st["step"].item()), []).append(p)
            for t, params in by_step.items():
                self._launch(lib, params, shadows, t, group["lr"], beta1, beta2, group["eps"],
                             group["weight_decay"])
        for pw in self.packed:
            pw.mark_fresh()
        return loss

    def _launch(self, lib, params, shadows, t, lr, beta1, beta2, eps, wd) -> None:
        rows, total = [], 0
        for p in params:
            g = p.grad
            if not (p.is_contiguous() and g.is_contiguous()):
                raise RuntimeError("AdamWShadow needs contiguous parameters and gradients")
            st = self.state[p]
            pw_part = shadows.get(id(p))
            if pw_part is not None:
                pw, part = pw_part
                if part.block >= 2 ** 32:
                    raise RuntimeError("shadow block too large")
                sh = pw.tensor.data_ptr() + 2 * part.start
                blk, stride = part.block, part.stride
            else:
                sh, blk, stride = 0, p.numel(), p.numel()
            rows.append([p.data_ptr(), g.data_ptr(), st["exp_avg"].data_ptr(), st["exp_avg_sq"].data_ptr(), sh,
                         p.numel(), blk, stride, total])
            total += p.numel()
        dev = params[0].device
        key = (dev, tuple(tuple(r) for r in rows))
        if key != self._table_key:
            # pinned + non_blocking: no host synchronisation; the caching host
            # allocator keeps the staging buffer until the copy has run
            self._table = torch.tensor(rows, dtype=torch.int64).pin_memory().to(dev, non_blocking=True)
            self._table_key = key
        bc1 = 1.0 - beta1 ** t
        bc2 = 1.0 - beta2 ** t
        st = lib.mt_adamw_step(self._table.data_ptr(), len(rows), total, _lib.dtype_code(_BF16), float(lr),
                               float(beta1), float(beta2), float(eps), float(wd), float(lr / bc1),
                               float(math.sqrt(bc2)), _lib.status_word(dev).data_ptr(), _lib.stream_ptr(dev))
        _lib.check(st, "adamw step")
