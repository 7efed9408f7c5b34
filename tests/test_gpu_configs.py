"""Operator parity at the BASELINE configurations themselves (full sizes).

* Config 1 -- causal GQA attention, B=16, Hq=16, Hkv=4, D=64,
  T in {1024, 2048, 4096}, q/k/v ~ N(0,1)*0.5, dO ~ N(0,1) from a seed,
  softmax scale 1/8; forward and backward run on the whole batch, and sampled
  (batch, kv-head) groups -- the kernels are independent per group -- are
  compared with the CPU fp32 oracle (each group: its 4 query heads, the kv
  head, O, dQ, dK, dV).  Also the model's strided [B, T, H, D] layout.
* Config 2 -- 65,536 tokens: the fused linear + cross-entropy (hidden 768,
  vocab 21,504, W ~ N(0, 0.02), hidden ~ N(0, 1) like the final RMSNorm's
  output, labels from the composite-token distribution), RMSNorm,
  add + RMSNorm (all-bf16 and the training step's bf16-branch/fp32-residual
  form), RoPE (config-3 heads 12/4, D=64, theta 5e5, model layout) and the
  SwiGLU gate (hidden 2048).  At these sizes the oracle's torch code runs in
  fp32 on the GPU with TF32 off (the CE oracle is the chunked analytic
  restatement, pinned against the reference's outputs on the CPU).

Tolerances (BASELINE): 2e-2 normwise max relative error for every output and
gradient, 1e-3 relative for the CE loss.
"""

from __future__ import annotations

import pytest
import torch

from oracle import ops as O

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _rel(actual: torch.Tensor, expected: torch.Tensor) -> float:
    """max|a - b| / max|b| computed on the device (the BASELINE metric)."""
    a = actual.detach().float()
    b = expected.detach().float().to(a.device)
    denom = float(b.abs().max())
    diff = float((a - b).abs().max())
    return diff / denom if denom else diff


def _check(actual, expected, name):
    err = _rel(actual, expected)
    assert err <= TOL, f"{name}: max relative error {err:.3e} > {TOL}"


@pytest.fixture
def no_tf32():
    old = (torch.backends.cuda.matmul.allow_tf32, torch.get_float32_matmul_precision())
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.set_float32_matmul_precision("highest")
    yield
    torch.backends.cuda.matmul.allow_tf32 = old[0]
    torch.set_float32_matmul_precision(old[1])


# ----------------------------------------------------------------------------- config 1
ATTN_GROUPS = [(0, 0), (7, 2), (15, 3)]  # (batch, kv head) pairs compared with the oracle


def _attention_config1(dev, T, layout, seed):
    from mega_trading_b200.kernels import triton_attention as A

    B, Hq, Hkv, D, rep = 16, 16, 4, 64, 4
    g = torch.Generator(device=dev).manual_seed(seed)

    def make(h, scale):
        if layout == "model":  # physical [B, T, H, D] viewed as [B, H, T, D] (model.py:220-222)
            return (torch.randn(B, T, h, D, generator=g, device=dev) * scale).to(torch.bfloat16).transpose(1, 2)
        return (torch.randn(B, h, T, D, generator=g, device=dev) * scale).to(torch.bfloat16)

    q, k, v = make(Hq, 0.5), make(Hkv, 0.5), make(Hkv, 0.5)
    do = torch.randn(B, Hq, T, D, generator=g, device=dev).to(torch.bfloat16)
    qd, kd, vd = (t.detach().requires_grad_(True) for t in (q, k, v))
    o = A.triton_attention(qd, kd, vd, repeats=rep)
    o.backward(do)
    torch.cuda.synchronize()
    from mega_trading_b200 import _lib

    assert _lib.read_status(dev) == 0
    for b, h in ATTN_GROUPS:
        hs = slice(h * rep, (h + 1) * rep)
        qo = q[b, hs].float().cpu()[None].requires_grad_(True)
        ko = k[b, h:h + 1].float().cpu()[None].requires_grad_(True)
        vo = v[b, h:h + 1].float().cpu()[None].requires_grad_(True)
        oo = O.causal_gqa_attention(qo, ko, vo, rep)
        oo.backward(do[b, hs].float().cpu()[None])
        tag = f"T={T} {layout} b={b} kv={h}"
        _check(o[b, hs], oo[0], f"{tag} O")
        _check(qd.grad[b, hs], qo.grad[0], f"{tag} dQ")
        _check(kd.grad[b, h], ko.grad[0, 0], f"{tag} dK")
        _check(vd.grad[b, h], vo.grad[0, 0], f"{tag} dV")


@pytest.mark.parametrize("T", [1024, 2048, 4096])
def test_attention_config1(cuda_device, T):
    _attention_config1(cuda_device, T, "contiguous", seed=1000 + T)


def test_attention_config1_model_layout(cuda_device):
    _attention_config1(cuda_device, 2048, "model", seed=77)


# ----------------------------------------------------------------------------- config 2
N2 = 65536


def _ce_config2(dev, ignore_every, weight_dtype):
    from mega_trading_b200 import _lib
    from mega_trading_b200.data import composite_tokens
    from mega_trading_b200.kernels import triton_ops as K

    H, V = 768, 21504
    g = torch.Generator(device=dev).manual_seed(2)
    hidden = torch.randn(N2, H, generator=g, device=dev).to(torch.bfloat16)
    weight = (torch.randn(V, H, generator=g, device=dev) * 0.02).to(weight_dtype)
    labels = composite_tokens(32, 2048, seed=5, device=dev).flatten()
    if ignore_every:
        labels[::ignore_every] = -100
    hd = hidden.detach().requires_grad_(True)
    wd = weight.detach().requires_grad_(True)
    loss = K.triton_fused_linear_cross_entropy(hd, wd, labels, ignore_index=-100)
    torch.cuda.synchronize()
    base = torch.cuda.memory_allocated(dev)
    torch.cuda.reset_peak_memory_stats(dev)
    (loss * 0.5).backward()
    torch.cuda.synchronize()
    assert _lib.read_status(dev) == 0
    # the backward never holds an [N, V] logit gradient (2.8 GB here): only dH, dW and
    # the workspace (row inputs, fp32 split partials) are allocated
    grads = hd.grad.numel() * hd.grad.element_size() + wd.grad.numel() * wd.grad.element_size()
    ws = int(_lib.load().mt_fused_ce_bwd_workspace_bytes(N2, V, H))
    delta = torch.cuda.max_memory_allocated(dev) - base
    assert delta <= grads + ws + (64 << 20), (delta, grads, ws)
    assert delta < N2 * V * 2 // 2, delta
    assert wd.grad.dtype == weight_dtype
    # oracle on the bf16-rounded operands, as the kernels see them
    lo, dho, dwo = O.linear_cross_entropy_grads(hidden.float(), weight.to(torch.bfloat16).float(), labels, -100,
                                                grad_output=0.5)
    rel = abs(float(loss.detach()) - float(lo)) / abs(float(lo))
    assert rel <= 1e-3, f"loss {float(loss.detach()):.6f} vs oracle {float(lo):.6f} (rel {rel:.2e})"
    _check(hd.grad, dho, "CE dH")
    _check(wd.grad, dwo, "CE dW")


def test_fused_ce_config2(cuda_device, no_tf32):
    _ce_config2(cuda_device, 0, torch.bfloat16)


def test_fused_ce_config2_ignored_rows(cuda_device, no_tf32):
    _ce_config2(cuda_device, 17, torch.bfloat16)


def _leaf(t):
    return t.detach().requires_grad_(True)


def test_rms_norm_config2(cuda_device):
    from mega_trading_b200.kernels import triton_ops as K

    g = torch.Generator(device=cuda_device).manual_seed(21)
    x = torch.randn(N2, 768, generator=g, device=cuda_device).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(768, generator=g, device=cuda_device)).to(torch.bfloat16)
    dy = torch.randn(N2, 768, generator=g, device=cuda_device).to(torch.bfloat16)
    xd, wd = _leaf(x), _leaf(w)
    y = K.triton_rms_norm(xd, wd, eps=1e-5)
    y.backward(dy)
    xo, wo = _leaf(x.float()), _leaf(w.float())
    yo = O.rms_norm(xo, wo, 1e-5)
    yo.backward(dy.float())
    _check(y, yo, "rms_norm y")
    _check(xd.grad, xo.grad, "rms_norm dx")
    _check(wd.grad, wo.grad, "rms_norm dw")


@pytest.mark.parametrize("mixed", [False, True])
def test_add_rms_norm_config2(cuda_device, mixed):
    """All-bf16 (the reference op) and the training step's bf16 branch + fp32 residual."""
    from mega_trading_b200.kernels import triton_ops as K

    g = torch.Generator(device=cuda_device).manual_seed(22)
    bf = torch.bfloat16
    x = torch.randn(N2, 768, generator=g, device=cuda_device).to(bf)
    r = torch.randn(N2, 768, generator=g, device=cuda_device)
    r = r if mixed else r.to(bf)
    w = 1 + 0.1 * torch.randn(768, generator=g, device=cuda_device)
    w = w if mixed else w.to(bf)
    gres = torch.randn(N2, 768, generator=g, device=cuda_device).to(r.dtype)
    gnorm = torch.randn(N2, 768, generator=g, device=cuda_device).to(bf)
    xd, rd, wd = _leaf(x), _leaf(r), _leaf(w)
    if mixed:
        new_res, normed = K.add_rms_norm(xd, rd, wd, eps=1e-5, out_dtype=bf)
    else:
        new_res, normed = K.triton_add_rms_norm(xd, rd, wd, eps=1e-5)
    torch.autograd.backward([new_res, normed], [gres, gnorm])
    xo, ro, wo = _leaf(x.float()), _leaf(r.float()), _leaf(w.float())
    nro, no = O.add_rms_norm(xo, ro, wo, 1e-5, act_dtype=None if mixed else bf)
    torch.autograd.backward([nro, no], [gres.float(), gnorm.float()])
    _check(new_res, nro, "add_rms_norm new_residual")
    _check(normed, no, "add_rms_norm normed")
    _check(xd.grad, xo.grad, "add_rms_norm d_hidden")
    _check(rd.grad, ro.grad, "add_rms_norm d_residual")
    _check(wd.grad, wo.grad, "add_rms_norm dw")


def test_rope_config2(cuda_device):
    """65,536 tokens as 32 sequences of 2048, config-3 heads, the model's [B, T, H, D] layout."""
    from mega_trading_b200.kernels import triton_ops as K

    B, T, Hq, Hk, D = 32, 2048, 12, 4, 64
    g = torch.Generator(device=cuda_device).manual_seed(23)
    bf = torch.bfloat16
    q = torch.randn(B, T, Hq, D, generator=g, device=cuda_device).to(bf).transpose(1, 2)
    k = torch.randn(B, T, Hk, D, generator=g, device=cuda_device).to(bf).transpose(1, 2)
    gq = torch.randn(B, Hq, T, D, generator=g, device=cuda_device).to(bf)
    gk = torch.randn(B, Hk, T, D, generator=g, device=cuda_device).to(bf)
    cos, sin = O.rope_tables(D, T, 500_000.0)
    qd, kd = _leaf(q), _leaf(k)
    qr, kr = K.triton_apply_rope(qd, kd, cos.to(cuda_device, bf), sin.to(cuda_device, bf))
    torch.autograd.backward([qr, kr], [gq, gk])
    qo, ko = _leaf(q.float()), _leaf(k.float())
    rq, rk = O.apply_rope(qo, ko, cos.to(cuda_device), sin.to(cuda_device), table_dtype=bf)
    torch.autograd.backward([rq, rk], [gq.float(), gk.float()])
    _check(qr, rq, "rope q")
    _check(kr, rk, "rope k")
    _check(qd.grad, qo.grad, "rope dq")
    _check(kd.grad, ko.grad, "rope dk")


def test_swiglu_config2(cuda_device):
    from mega_trading_b200.kernels import triton_ops as K

    g = torch.Generator(device=cuda_device).manual_seed(24)
    bf = torch.bfloat16
    gate = torch.randn(N2, 2048, generator=g, device=cuda_device).to(bf)
    up = torch.randn(N2, 2048, generator=g, device=cuda_device).to(bf)
    dy = torch.randn(N2, 2048, generator=g, device=cuda_device).to(bf)
    gd, ud = _leaf(gate), _leaf(up)
    y = K.triton_swiglu_gate(gd, ud)
    y.backward(dy)
    go, uo = _leaf(gate.float()), _leaf(up.float())
    yo = O.swiglu_gate(go, uo, act_dtype=bf)
    yo.backward(dy.float())
    _check(y, yo, "swiglu y")
    _check(gd.grad, go.grad, "swiglu dgate")
    _check(ud.grad, uo.grad, "swiglu dup")
