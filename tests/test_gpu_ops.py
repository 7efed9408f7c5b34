"""GPU parity of the bandwidth operators against the CPU fp32 oracle.

Seeds and shapes follow the reference's kernel tests
(``tests/test_training.py:602-718`` of duoan/mega-trading) plus BASELINE-style
shapes and ragged / edge cases.  Tolerance: the BASELINE bar of 2e-2 normwise
max relative error for outputs and gradients, and the reference's own
allclose tolerances (6e-2 outputs, 8e-2 gradients).
"""

from __future__ import annotations

import pytest
import torch

from oracle import ops as O

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _check(actual, expected, name, atol=None):
    err = O.max_rel_error(actual, expected)
    assert err <= TOL, f"{name}: max relative error {err:.3e} > {TOL}"
    if atol is not None:
        a = actual.detach().float().cpu()
        b = expected.detach().float().cpu()
        assert torch.allclose(a, b, atol=atol, rtol=atol), f"{name}: allclose({atol}) failed"


def _leaf(t, dev, dtype):
    return t.to(dev, dtype).requires_grad_(True)


def _oracle_leaf(t, dtype):
    return t.to(dtype).float().requires_grad_(True)


@pytest.mark.parametrize("shape,dtype,seed", [((2, 512, 1024), torch.bfloat16, 19), ((4, 77, 768), torch.bfloat16, 3),
                                              ((3, 5, 200), torch.float16, 4), ((64, 768), torch.float32, 5),
                                              ((1, 1, 4096), torch.bfloat16, 6), ((2, 3, 12), torch.bfloat16, 7),
                                              ((2, 64, 1536), torch.bfloat16, 33), ((3, 2048), torch.float16, 34)])
def test_rms_norm_matches_oracle(cuda_device, shape, dtype, seed):
    from mega_trading_b200.kernels import triton_ops as K

    g = torch.Generator().manual_seed(seed)
    x = torch.randn(*shape, generator=g)
    w = torch.randn(shape[-1], generator=g)
    dy = torch.randn(*shape, generator=g)
    xd, wd = _leaf(x, cuda_device, dtype), _leaf(w, cuda_device, dtype)
    y = K.triton_rms_norm(xd, wd, eps=1e-5)
    y.backward(dy.to(cuda_device, dtype))
    xo, wo = _oracle_leaf(x, dtype), _oracle_leaf(w, dtype)
    yo = O.rms_norm(xo, wo, 1e-5)
    yo.backward(dy.to(dtype).float())
    assert y.dtype == dtype and y.shape == x.shape
    _check(y, yo, "rms_norm y", atol=6e-2)
    _check(xd.grad, xo.grad, "rms_norm dx", atol=8e-2)
    _check(wd.grad, wo.grad, "rms_norm dw")


def test_rms_norm_mixed_fp32_residual_bf16_out(cuda_device):
    from mega_trading_b200.kernels import triton_ops as K

    g = torch.Generator().manual_seed(31)
    x = torch.randn(8, 96, 768, generator=g)
    w = 1 + 0.1 * torch.randn(768, generator=g)
    dy = torch.randn(8, 96, 768, generator=g)
    xd, wd = _leaf(x, cuda_device, torch.float32), _leaf(w, cuda_device, torch.float32)
    y = K.rms_norm(xd, wd, eps=1e-5, out_dtype=torch.bfloat16)
    y.backward(dy.to(cuda_device, torch.bfloat16))
    xo, wo = _oracle_leaf(x, torch.float32), _oracle_leaf(w, torch.float32)
    yo = O.rms_norm(xo, wo, 1e-5)
    yo.backward(dy.to(torch.bfloat16).float())
    assert y.dtype == torch.bfloat16 and xd.grad.dtype == torch.float32
    _check(y, yo, "rms_norm mixed y")
    _check(xd.grad, xo.grad, "rms_norm mixed dx")
    _check(wd.grad, wo.grad, "rms_norm mixed dw")


@pytest.mark.parametrize("rows,dim", [(4096, 768), (37, 768), (5, 200)])
def test_add_rms_norm_mixed_dual_gradient(cuda_device, rows, dim):
    """bf16 branch + fp32 residual stream: the fp32 gradient and its bf16 copy come from one kernel."""
    from mega_trading_b200.kernels import triton_ops as K

    g = torch.Generator().manual_seed(rows + dim)
    x = torch.randn(rows, dim, generator=g)
    r = torch.randn(rows, dim, generator=g)
    w = 1 + 0.1 * torch.randn(dim, generator=g)
    gres = torch.randn(rows, dim, generator=g)
    gnorm = torch.randn(rows, dim, generator=g)
    xd = _leaf(x, cuda_device, torch.bfloat16)
    rd, wd = _leaf(r, cuda_device, torch.float32), _leaf(w, cuda_device, torch.float32)
    new_res, normed = K.add_rms_norm(xd, rd, wd, eps=1e-5, out_dtype=torch.bfloat16)
    assert new_res.dtype == torch.float32 and normed.dtype == torch.bfloat16
    torch.autograd.backward([new_res, normed], [gres.to(cuda_device), gnorm.to(cuda_device, torch.bfloat16)])
    assert xd.grad.dtype == torch.bfloat16 and rd.grad.dtype == torch.float32
    assert torch.equal(xd.grad, rd.grad.to(torch.bfloat16))  # same values, rounded once
    xo = x.to(torch.bfloat16).float().requires_grad_(True)
    ro, wo = r.clone().requires_grad_(True), w.clone().requires_grad_(True)
    nro, no = O.add_rms_norm(xo, ro, wo, 1e-5)
    torch.autograd.backward([nro, no], [gres, gnorm.to(torch.bfloat16).float()])
    _check(normed, no, "dual normed")
    _check(rd.grad, ro.grad, "dual d_residual")
    _check(wd.grad, wo.grad, "dual dw")


@pytest.mark.parametrize("shape,dtype,seed", [((2, 512, 1024), torch.bfloat16, 37), ((5, 33, 768), torch.float16, 8),
                                              ((16, 768), torch.float32, 9), ((40, 1536), torch.bfloat16, 35),
                                              ((7, 2048), torch.bfloat16, 36)])
def test_add_rms_norm_matches_oracle(cuda_device, shape, dtype, seed):
    from mega_trading_b200.kernels import triton_ops as K

    g = torch.Generator().manual_seed(seed)
    x = torch.randn(*shape, generator=g)
    r = torch.randn(*shape, generator=g)
    w = torch.randn(shape[-1], generator=g)
    gres = torch.randn(*shape, generator=g)
    gnorm = torch.randn(*shape, generator=g)
    xd, rd, wd = (_leaf(t, cuda_device, dtype) for t in (x, r, w))
    new_res, normed = K.triton_add_rms_norm(xd, rd, wd, eps=1e-5)
    torch.autograd.backward([new_res, normed], [gres.to(cuda_device, dtype), gnorm.to(cuda_device, dtype)])
    xo, ro, wo = (_oracle_leaf(t, dtype) for t in (x, r, w))
    nro, no = O.add_rms_norm(xo, ro, wo, 1e-5, act_dtype=dtype)
    torch.autograd.backward([nro, no], [gres.to(dtype).float(), gnorm.to(dtype).float()])
    _check(new_res, nro, "add_rms_norm new_residual", atol=6e-2)
    _check(normed, no, "add_rms_norm normed", atol=6e-2)
    _check(xd.grad, xo.grad, "add_rms_norm d_hidden", atol=8e-2)
    _check(rd.grad, ro.grad, "add_rms_norm d_residual", atol=8e-2)
    _check(wd.grad, wo.grad, "add_rms_norm dw")


def _rope_case(cuda_device, B, Hq, Hk, T, D, theta, dtype, seed, layout):
    from mega_trading_b200.kernels import triton_ops as K

    g = torch.Generator().manual_seed(seed)
    if layout == "model":  # physical [B, T, H, D] viewed as [B, H, T, D] (model.py:220-222)
        q = torch.randn(B, T, Hq, D, generator=g).transpose(1, 2)
        k = torch.randn(B, T, Hk, D, generator=g).transpose(1, 2)
    else:
        q = torch.randn(B, Hq, T, D, generator=g)
        k = torch.randn(B, Hk, T, D, generator=g)
    gq = torch.randn(B, Hq, T, D, generator=g)
    gk = torch.randn(B, Hk, T, D, generator=g)
    cos, sin = O.rope_tables(D, T, theta)
    qd = q.to(cuda_device, dtype).requires_grad_(True)
    kd = k.to(cuda_device, dtype).requires_grad_(True)
    if layout == "model":
        qd = q.transpose(1, 2).contiguous().to(cuda_device, dtype).transpose(1, 2).detach().requires_grad_(True)
        kd = k.transpose(1, 2).contiguous().to(cuda_device, dtype).transpose(1, 2).detach().requires_grad_(True)
    qo_, ko_ = K.triton_apply_rope(qd, kd, cos.to(cuda_device, dtype), sin.to(cuda_device, dtype))
    assert qo_.stride() == qd.stride()
    torch.autograd.backward([qo_, ko_], [gq.to(cuda_device, dtype), gk.to(cuda_device, dtype)])
    qo = q.to(dtype).float().requires_grad_(True)
    ko = k.to(dtype).float().requires_grad_(True)
    rq, rk = O.apply_rope(qo, ko, cos, sin, table_dtype=dtype)
    torch.autograd.backward([rq, rk], [gq.to(dtype).float(), gk.to(dtype).float()])
    _check(qo_, rq, "rope q", atol=6e-2)
    _check(ko_, rk, "rope k", atol=6e-2)
    _check(qd.grad, qo.grad, "rope dq", atol=8e-2)
    _check(kd.grad, ko.grad, "rope dk", atol=8e-2)


@pytest.mark.parametrize("B,Hq,Hk,T,D,theta,dtype,seed,layout", [
    (1, 16, 4, 512, 64, 500_000.0, torch.bfloat16, 23, "contiguous"),
    (2, 12, 4, 256, 64, 500_000.0, torch.bfloat16, 24, "model"),
    (1, 4, 2, 17, 32, 10_000.0, torch.float16, 25, "contiguous"),
    (1, 3, 1, 9, 6, 10_000.0, torch.bfloat16, 26, "contiguous"),
    (1, 2, 2, 5, 8, 10_000.0, torch.float32, 27, "model"),
])
def test_rope_matches_oracle(cuda_device, B, Hq, Hk, T, D, theta, dtype, seed, layout):
    _rope_case(cuda_device, B, Hq, Hk, T, D, theta, dtype, seed, layout)


@pytest.mark.parametrize("shape,dtype,seed", [((2, 512, 2816), torch.bfloat16, 29), ((3, 7, 2048), torch.float16, 30),
                                              ((1001,), torch.bfloat16, 31), ((64, 130), torch.float32, 32)])
def test_swiglu_matches_oracle(cuda_device, shape, dtype, seed):
    from mega_trading_b200.kernels import triton_ops as K

    g = torch.Generator().manual_seed(seed)
    gate = torch.randn(*shape, generator=g)
    up = torch.randn(*shape, generator=g)
    dy = torch.randn(*shape, generator=g)
    gd, ud = _leaf(gate, cuda_device, dtype), _leaf(up, cuda_device, dtype)
    y = K.triton_swiglu_gate(gd, ud)
    y.backward(dy.to(cuda_device, dtype))
    go, uo = _oracle_leaf(gate, dtype), _oracle_leaf(up, dtype)
    yo = O.swiglu_gate(go, uo, act_dtype=dtype)
    yo.backward(dy.to(dtype).float())
    _check(y, yo, "swiglu y", atol=6e-2)
    _check(gd.grad, go.grad, "swiglu dgate", atol=8e-2)
    _check(ud.grad, uo.grad, "swiglu dup", atol=8e-2)


def test_ops_reject_cpu_tensors():
    from mega_trading_b200.kernels import triton_ops as K

    x = torch.randn(2, 8)
    with pytest.raises(RuntimeError):
        K.triton_rms_norm(x, torch.ones(8), eps=1e-5)
    with pytest.raises(RuntimeError):
        K.triton_swiglu_gate(x, x)
