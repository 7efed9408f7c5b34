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
