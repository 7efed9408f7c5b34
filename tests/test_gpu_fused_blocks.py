"""GPU parity of the fused model nodes against the CPU fp32 oracle.

``swiglu_packed`` reads [gate | up] from one [N, 2I] projection and writes the
packed gradient; ``qkv_rope_attention`` splits one packed [B, T, (Hq+2Hkv)D]
projection, rotates q/k, runs causal GQA attention and writes one packed
gradient.  Both are compared with the oracle's operator-by-operator math
(reference ``src/mega_trading/model.py:218-256, 286-294``).  Tolerance: 2e-2
normwise max relative error.
"""

from __future__ import annotations

import pytest
import torch

from oracle import ops as O

pytestmark = pytest.mark.gpu

TOL = 2e-2


@pytest.mark.parametrize("rows,inter,dtype,seed", [(4096, 2048, torch.bfloat16, 41), (77, 688, torch.bfloat16, 42),
                                                   (5, 64, torch.float16, 43), (1, 16, torch.bfloat16, 44)])
def test_swiglu_packed_matches_oracle(cuda_device, rows, inter, dtype, seed):
    from mega_trading_b200.kernels.fused_blocks import swiglu_packed

    g = torch.Generator().manual_seed(seed)
    gu = torch.randn(rows, 2 * inter, generator=g)
    dy = torch.randn(rows, inter, generator=g)
    gd = gu.to(cuda_device, dtype).requires_grad_(True)
    y = swiglu_packed(gd)
    y.backward(dy.to(cuda_device, dtype))
    go = gu.to(dtype).float().requires_grad_(True)
    yo = O.swiglu_gate(go[:, :inter], go[:, inter:], act_dtype=dtype)
    yo.backward(dy.to(dtype).float())
    assert y.shape == (rows, inter) and y.dtype == dtype
    assert O.max_rel_error(y, yo) <= TOL
    assert O.max_rel_error(gd.grad, go.grad) <= TOL


@pytest.mark.parametrize("B,T,Hq,Hkv,D,theta,seed", [(2, 256, 12, 4, 64, 500_000.0, 51),
                                                     (1, 300, 8, 2, 32, 10_000.0, 52),
                                                     (1, 129, 4, 4, 64, 10_000.0, 53)])
def test_qkv_rope_attention_matches_oracle(cuda_device, B, T, Hq, Hkv, D, theta, seed):
    from mega_trading_b200.kernels.fused_blocks import qkv_rope_attention

    g = torch.Generator().manual_seed(seed)
    width = (Hq + 2 * Hkv) * D
    qkv = torch.randn(B, T, width, generator=g) * 0.7
    do = torch.randn(B, T, Hq, D, generator=g)
    cos, sin = O.rope_tables(D, T, theta)
    qd = qkv.to(cuda_device, torch.bfloat16).requires_grad_(True)
    o = qkv_rope_attention(qd, cos.to(cuda_device), sin.to(cuda_device), Hq, Hkv, D)
    assert o.shape == (B, Hq, T, D)
    assert o.transpose(1, 2).is_contiguous()  # stored [B, T, H, D]
    o.backward(do.to(cuda_device, torch.bfloat16).transpose(1, 2))

    qo = qkv.to(torch.bfloat16).float().requires_grad_(True)
    q = qo[..., : Hq * D].reshape(B, T, Hq, D).transpose(1, 2)
    k = qo[..., Hq * D:(Hq + Hkv) * D].reshape(B, T, Hkv, D).transpose(1, 2)
    v = qo[..., (Hq + Hkv) * D:].reshape(B, T, Hkv, D).transpose(1, 2)
    rq, rk = O.apply_rope(q, k, cos, sin, table_dtype=torch.bfloat16)
    oo = O.causal_gqa_attention(rq, rk, v, Hq // Hkv)
    oo.backward(do.to(torch.bfloat16).float().transpose(1, 2))
    err_o = O.max_rel_error(o, oo)
    err_g = O.max_rel_error(qd.grad, qo.grad)
    assert err_o <= TOL, f"output error {err_o:.3e}"
    assert err_g <= TOL, f"packed gradient error {err_g:.3e}"
    for lo, hi in ((0, Hq * D), (Hq * D, (Hq + Hkv) * D), ((Hq + Hkv) * D, width)):
        assert O.max_rel_error(qd.grad[..., lo:hi], qo.grad[..., lo:hi]) <= TOL


def test_fused_blocks_reject_bad_input(cuda_device):
    from mega_trading_b200.kernels.fused_blocks import qkv_rope_attention, swiglu_packed

    with pytest.raises(ValueError):
        swiglu_packed(torch.zeros(4, 30, device=cuda_device, dtype=torch.bfloat16))
    cos, sin = O.rope_tables(64, 8, 10_000.0)
    with pytest.raises(ValueError):
        qkv_rope_attention(torch.zeros(1, 8, 100, device=cuda_device, dtype=torch.bfloat16), cos.to(cuda_device),
                           sin.to(cuda_device), 2, 1, 64)


@pytest.mark.parametrize("M,H,I,seed", [(4096, 768, 2048, 61), (300, 256, 512, 62), (1, 768, 256, 63),
                                        (1000, 64, 768, 64), (513, 200, 256, 66), (129, 256, 256, 67),
                                        (256, 128, 512, 68)])
def test_swiglu_mlp_matches_oracle(cuda_device, M, H, I, seed):
    """Fused SwiGLU MLP (gate inside the tcgen05 GEMM epilogues) vs the fp32 oracle.  M > 128 runs
    the gate/up GEMM on CTA pairs (M = 129: the odd CTA's rows lie past M; 256: one pair tile)."""
    from mega_trading_b200.kernels.fused_blocks import interleave_gate_up, swiglu_mlp

    g = torch.Generator().manual_seed(seed)
    bf = torch.bfloat16
    x = torch.randn(M, H, generator=g)
    w1 = torch.randn(I, H, generator=g) * 0.05
    w3 = torch.randn(I, H, generator=g) * 0.05
    w2 = torch.randn(H, I, generator=g) * 0.05
    dout = torch.randn(M, H, generator=g)
    xd, w1d, w3d, w2d = (t.to(cuda_device, bf).requires_grad_(True) for t in (x, w1, w3, w2))
    out = swiglu_mlp(xd, interleave_gate_up(w1d, w3d), w2d)
    out.backward(dout.to(cuda_device, bf))
    xo, w1o, w3o, w2o = (t.to(bf).float().requires_grad_(True) for t in (x, w1, w3, w2))
    yo = O.swiglu_gate(xo @ w1o.t(), xo @ w3o.t(), act_dtype=bf)
    oo = yo @ w2o.t()
    oo.backward(dout.to(bf).float())
    assert out.shape == (M, H) and out.dtype == bf
    for name, a, b in (("out", out, oo), ("dx", xd.grad, xo.grad), ("dw1", w1d.grad, w1o.grad),
                       ("dw3", w3d.grad, w3o.grad), ("dw2", w2d.grad, w2o.grad)):
        err = O.max_rel_error(a, b)
        assert err <= TOL, f"{name}: max relative error {err:.3e}"


def test_swiglu_gemm_gate_is_bit_exact_with_the_standalone_gate(cuda_device):
    """The forward epilogue's y equals the standalone packed gate applied to the same saved gate/up."""
    from mega_trading_b200 import _lib
    from mega_trading_b200.kernels.fused_blocks import interleave_gate_up

    lib = _lib.load()
    g = torch.Generator(device=cuda_device).manual_seed(65)
    M, H, I = 777, 768, 2048
    x = torch.randn(M, H, device=cuda_device, generator=g).bfloat16()
    w13 = interleave_gate_up(torch.randn(I, H, device=cuda_device, generator=g) * 0.05,
                             torch.randn(I, H, device=cuda_device, generator=g) * 0.05).bfloat16().contiguous()
    gu = torch.empty(M, 2 * I, device=cuda_device, dtype=torch.bfloat16)
    y = torch.empty(M, I, device=cuda_device, dtype=torch.bfloat16)
    status = _lib.status_word(cuda_device)
    _lib.check(lib.mt_swiglu_gemm_fwd(x.data_ptr(), w13.data_ptr(), gu.data_ptr(), y.data_ptr(), 2, M, H, I,
                                      status.data_ptr(), _lib.stream_ptr(cuda_device)), "swiglu_gemm forward")
    # the saved activation is the projection rounded to bf16
    ref = torch.nn.functional.linear(x.float(), w13.float())
    assert O.max_rel_error(gu, ref) <= 1e-2
    # [gate | up] from the interleaved layout, then the standalone gate
    blocks = gu.view(M, I // 128, 2, 128)
    packed = torch.cat([blocks[:, :, 0].reshape(M, I), blocks[:, :, 1].reshape(M, I)], dim=1).contiguous()
    y2 = torch.empty_like(y)
    _lib.check(lib.mt_swiglu_packed_fwd(packed.data_ptr(), y2.data_ptr(), 2, M, I, _lib.stream_ptr(cuda_device)),
               "swiglu_packed forward")
    torch.cuda.synchronize()
    assert _lib.read_status(cuda_device) == 0
    assert torch.equal(y, y2)


@pytest.mark.parametrize("B,T,H,Hq,Hkv,D,theta,seed", [(2, 256, 768, 12, 4, 64, 500_000.0, 71),
                                                       (1, 300, 256, 8, 4, 32, 10_000.0, 72),
                                                       (3, 128, 512, 4, 2, 64, 10_000.0, 73),
                                                       (1, 77, 200, 4, 2, 64, 10_000.0, 75)])
def test_qkv_proj_rope_attention_matches_oracle(cuda_device, B, T, H, Hq, Hkv, D, theta, seed):
    """Projection GEMM with RoPE in its epilogue + attention, vs the fp32 oracle chain."""
    from mega_trading_b200.kernels.fused_blocks import qkv_proj_rope_attention

    g = torch.Generator().manual_seed(seed)
    bf = torch.bfloat16
    n = (Hq + 2 * Hkv) * D
    x = torch.randn(B, T, H, generator=g)
    w = torch.randn(n, H, generator=g) * (1.0 / H ** 0.5)
    do = torch.randn(B, T, Hq, D, generator=g)
    cos, sin = O.rope_tables(D, T, theta)
    xd, wd = x.to(cuda_device, bf).requires_grad_(True), w.to(cuda_device, bf).requires_grad_(True)
    o = qkv_proj_rope_attention(xd, wd, cos.to(cuda_device), sin.to(cuda_device), Hq, Hkv, D)
    assert o.shape == (B, Hq, T, D) and o.transpose(1, 2).is_contiguous()
    o.backward(do.to(cuda_device, bf).transpose(1, 2))
    xo, wo = x.to(bf).float().requires_grad_(True), w.to(bf).float().requires_grad_(True)
    qkv = xo @ wo.t()
    q = qkv[..., : Hq * D].reshape(B, T, Hq, D).transpose(1, 2)
    k = qkv[..., Hq * D:(Hq + Hkv) * D].reshape(B, T, Hkv, D).transpose(1, 2)
    v = qkv[..., (Hq + Hkv) * D:].reshape(B, T, Hkv, D).transpose(1, 2)
    rq, rk = O.apply_rope(q, k, cos, sin, table_dtype=bf)
    oo = O.causal_gqa_attention(rq, rk, v, Hq // Hkv)
    oo.backward(do.to(bf).float().transpose(1, 2))
    for name, a, b in (("o", o, oo), ("dx", xd.grad, xo.grad), ("dw", wd.grad, wo.grad)):
        err = O.max_rel_error(a, b)
        assert err <= TOL, f"{name}: max relative error {err:.3e}"


def test_qkv_rope_gemm_rotation_is_bit_exact_with_the_rope_kernel(cuda_device):
    """Epilogue RoPE == the standalone RoPE kernel applied to the same rounded projection."""
    from mega_trading_b200 import _lib
    from mega_trading_b200.kernels import triton_ops as K

    lib = _lib.load()
    g = torch.Generator(device=cuda_device).manual_seed(74)
    B, T, H, Hq, Hkv, D = 2, 384, 768, 12, 4, 64
    n = (Hq + 2 * Hkv) * D
    x = torch.randn(B * T, H, device=cuda_device, generator=g).bfloat16()
    w = (torch.randn(n, H, device=cuda_device, generator=g) * 0.04).bfloat16()
    cos, sin = O.rope_tables(D, T, 500_000.0)
    cos2 = cos.reshape(T, D // 2).to(cuda_device, torch.bfloat16).contiguous()
    sin2 = sin.reshape(T, D // 2).to(cuda_device, torch.bfloat16).contiguous()
    status = _lib.status_word(cuda_device)
    outs = []
    for rot in ((Hq + Hkv) * D, 0):
        qkv = torch.empty(B * T, n, device=cuda_device, dtype=torch.bfloat16)
        _lib.check(lib.mt_qkv_rope_gemm(x.data_ptr(), w.data_ptr(), qkv.data_ptr(), cos2.data_ptr(), sin2.data_ptr(),
                                        D // 2, 2, B * T, H, n, rot, T, D, status.data_ptr(),
                                        _lib.stream_ptr(cuda_device)), "qkv_rope_gemm")
        outs.append(qkv.view(B, T, n))
    fused, plain = outs
    q = plain[..., : Hq * D].view(B, T, Hq, D).transpose(1, 2)
    k = plain[..., Hq * D:(Hq + Hkv) * D].view(B, T, Hkv, D).transpose(1, 2)
    qo, ko = torch.empty_like(q), torch.empty_like(k)
    K._launch_rope(q, k, cos2, sin2, qo, ko, negate=False)
    torch.cuda.synchronize()
    assert _lib.read_status(cuda_device) == 0
    assert torch.equal(fused[..., : Hq * D].view(B, T, Hq, D), qo.transpose(1, 2))
    assert torch.equal(fused[..., Hq * D:(Hq + Hkv) * D].view(B, T, Hkv, D), ko.transpose(1, 2))
    assert torch.equal(fused[..., (Hq + Hkv) * D:], plain[..., (Hq + Hkv) * D:])
    ref = torch.nn.functional.linear(x.float(), w.float()).view(B, T, n)
    assert O.max_rel_error(plain, ref) <= 1e-2
