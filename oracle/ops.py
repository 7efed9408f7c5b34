"""CPU fp32 restatement of duoan/mega-trading's PyTorch operator path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this
package; the product path (``mega_trading_b200``) never does.

Each function restates the reference's torch implementation of one operator
(the path the reference itself takes on CPU, ``triton_ops.py:13-14, 52-53,
59-60, 90-91``) in float32, from inputs that were already rounded to the
device dtype.  Where the reference rounds an intermediate to the activation
dtype (the RoPE tables, the SwiGLU silu, the residual add), the restatement
rounds at the same place.  Pinned against the reference's own outputs by
``tests/golden/make_golden.py`` / ``tests/test_oracle_golden.py``.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def _f32(t: torch.Tensor) -> torch.Tensor:
    return t.detach().to(device="cpu", dtype=torch.float32)


def rms_norm(hidden: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """``F.rms_norm(hidden, (H,), weight, eps)`` in fp32 (model.py:266-269)."""
    return F.rms_norm(hidden, (hidden.shape[-1],), weight, eps=eps)


def add_rms_norm(hidden: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float,
                 act_dtype: torch.dtype | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """``new = hidden + residual`` (rounded to the activation dtype), ``RMSNorm(new)``
    (triton_ops.py:39-41)."""
    new = hidden + residual
    if act_dtype is not None and act_dtype != torch.float32:
        new = new + (new.detach().to(act_dtype).float() - new.detach())  # straight-through rounding
    return new, rms_norm(new, weight, eps)


def rope_tables(head_dim: int, length: int, theta: float) -> tuple[torch.Tensor, torch.Tensor]:
    """RoPE cos/sin tables [1, 1, T, D/2] (model.py:280-284)."""
    positions = torch.arange(length, dtype=torch.float32)
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    freqs = torch.outer(positions, inv_freq)
    return (freqs.cos().view(1, 1, length, head_dim // 2), freqs.sin().view(1, 1, length, head_dim // 2))


def rotate(value: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Interleaved-pair rotation (model.py:312-316)."""
    even = value[..., 0::2]
    odd = value[..., 1::2]
    return torch.stack((even * cos - odd * sin, even * sin + odd * cos), dim=-1).flatten(start_dim=-2)


def apply_rope(query: torch.Tensor, key: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
               table_dtype: torch.dtype | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """RoPE of q and k; the tables are first rounded to the activation dtype
    (model.py:290-291) when ``table_dtype`` is given."""
    T = query.shape[-2]
    cos = cos[..., :T, :]
    sin = sin[..., :T, :]
    if table_dtype is not None:
        cos = cos.to(table_dtype).float()
        sin = sin.to(table_dtype).float()
    return rotate(query, cos, sin), rotate(key, cos, sin)


def swiglu_gate(gate: torch.Tensor, up: torch.Tensor, act_dtype: torch.dtype | None = None) -> torch.Tensor:
    """``F.silu(gate) * up`` (model.py:255); with ``act_dtype`` the silu output is
    rounded to it first, as a bf16 ``F.silu`` does (triton_ops.py:781-782)."""
    s = F.silu(gate)
    if act_dtype is not None and act_dtype != torch.float32:
        s = s + (s.detach().to(act_dtype).float() - s.detach())
    return s * up


def causal_gqa_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, repeats: int) -> torch.Tensor:
    """Causal grouped-query attention with scale 1/sqrt(D): the math of
    ``F.scaled_dot_product_attention(is_causal=True, enable_gqa=True)``
    (model.py:228-235) and of the reference backward (triton_attention.py:88-111)."""
    if repeats > 1:
        key = key.repeat_interleave(repeats, dim=1)
        value = value.repeat_interleave(repeats, dim=1)
    T = query.shape[-2]
    scale = 1.0 / math.sqrt(query.shape[-1])
    scores = torch.matmul(query, key.transpose(-2, -1)) * scale
    mask = torch.ones((T, T), dtype=torch.bool).tril()
    scores = scores.masked_fill(~mask, float("-inf"))
    probs = torch.softmax(scores, dim=-1)
    return torch.matmul(probs, value)


def attention_lse(query: torch.Tensor, key: torch.Tensor, repeats: int) -> torch.Tensor:
    """Natural-log logsumexp of the scaled causal scores, [B, Hq, T]
    (the tensor saved for backward, triton_attention.py:34, :344-349)."""
    if repeats > 1:
        key = key.repeat_interleave(repeats, dim=1)
    T = query.shape[-2]
    scores = torch.matmul(query, key.transpose(-2, -1)) / math.sqrt(query.shape[-1])
    mask = torch.ones((T, T), dtype=torch.bool).tril()
    return torch.logsumexp(scores.masked_fill(~mask, float("-inf")), dim=-1)


def linear_cross_entropy(hidden: torch.Tensor, weight: torch.Tensor, labels: torch.Tensor,
                         ignore_index: int = -100) -> torch.Tensor:
    """Mean CE of ``hidden @ weight.T`` over non-ignored rows; zero (still on the
    graph) when every row is ignored (triton_ops.py:99-112)."""
    if int((labels != ignore_index).sum().item()) == 0:
        return (hidden.sum() + weight.sum()) * 0.0
    return F.cross_entropy(F.linear(hidden, weight), labels, ignore_index=ignore_index)


@torch.no_grad()
def linear_cross_entropy_grads(hidden: torch.Tensor, weight: torch.Tensor, labels: torch.Tensor,
                               ignore_index: int = -100, grad_output: float = 1.0,
                               chunk_rows: int = 8192) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """``(loss, d_hidden, d_weight)`` of :func:`linear_cross_entropy` in fp32, computed
    analytically over row chunks on the inputs' device: the reference's chunked
    recipe (triton_ops.py:359-389: logits of one chunk, softmax minus one-hot of
    the target scaled by 1/n_valid, ``grad_hidden = dZ W``, ``grad_weight += dZ^T H``)
    with the loss of triton_ops.py:99-112 (mean over non-ignored rows, 0 when
    every row is ignored).  For sizes whose full [N, V] logits do not fit."""
    h = hidden.float()
    w = weight.float()
    valid = labels != ignore_index
    n_valid = int(valid.sum().item())
    dh = torch.zeros_like(h)
    dw = torch.zeros_like(w)
    if n_valid == 0:
        return torch.zeros((), dtype=torch.float32, device=h.device), dh, dw
    scale = grad_output / n_valid
    total = torch.zeros((), dtype=torch.float64, device=h.device)
    for lo in range(0, h.shape[0], chunk_rows):
        hi = min(h.shape[0], lo + chunk_rows)
        z = h[lo:hi] @ w.t()
        lse = torch.logsumexp(z, dim=-1)
        lab = labels[lo:hi]
        ok = valid[lo:hi]
        safe = torch.where(ok, lab, torch.zeros_like(lab)).long()
        zy = z.gather(1, safe[:, None]).squeeze(1)
        total += ((lse - zy) * ok).double().sum()
        dz = torch.softmax(z, dim=-1)
        dz[torch.arange(hi - lo, device=z.device), safe] -= 1.0
        dz *= (ok.float() * scale)[:, None]
        dh[lo:hi] = dz @ w
        dw += dz.t() @ h[lo:hi]
    return (total / n_valid).float(), dh, dw


def max_rel_error(actual: torch.Tensor, expected: torch.Tensor) -> float:
    """Normwise max relative error ``max|a - b| / max|b|`` (the BASELINE metric)."""
    a = _f32(actual)
    b = _f32(expected)
    denom = float(b.abs().max())
    diff = float((a - b).abs().max())
    if denom == 0.0:
        return diff
    return diff / denom
