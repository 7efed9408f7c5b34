"""GPU parity of the tcgen05 causal GQA attention against the CPU fp32 oracle.

Cases: the reference's own kernel-test shapes (``tests/test_training.py:519-600``
of duoan/mega-trading: B1 Hq4 Hkv2 T17 D32 fp16 seed 11; B1 Hq16 Hkv4 T512 D64
bf16 seeds 13/17), BASELINE config-1 shapes at reduced batch, the model's
strided [B,T,H,D] layout, odd repeats (config 3: 12/4) and ragged T.
Tolerance: 2e-2 normwise max relative error (BASELINE), plus the reference's
allclose tolerances (6e-2 forward, 8e-2 gradients).
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
        bad = (a - b).abs() > atol + atol * b.abs()
        assert not bool(bad.any()), f"{name}: allclose({atol}) failed at {int(bad.sum())} elements"


def _inputs(B, Hq, Hkv, T, D, seed, scale=1.0, layout="contiguous"):
    g = torch.Generator().manual_seed(seed)
    if layout == "model":
        q = (torch.randn(B, T, Hq, D, generator=g) * scale).transpose(1, 2)
        k = (torch.randn(B, T, Hkv, D, generator=g) * scale).transpose(1, 2)
        v = (torch.randn(B, T, Hkv, D, generator=g) * scale).transpose(1, 2)
    else:
        q = torch.randn(B, Hq, T, D, generator=g) * scale
        k = torch.randn(B, Hkv, T, D, generator=g) * scale
        v = torch.randn(B, Hkv, T, D, generator=g) * scale
    do = torch.randn(B, Hq, T, D, generator=g)
    return q, k, v, do


def _to_dev(t, dev, dtype, layout):
    if layout == "model":
        return t.transpose(1, 2).contiguous().to(dev, dtype).transpose(1, 2).detach().requires_grad_(True)
    return t.to(dev, dtype).requires_grad_(True)


FWD_CASES = [
    # B, Hq, Hkv, T, D, dtype, seed, scale, layout
    (1, 4, 2, 17, 32, torch.float16, 11, 1.0, "contiguous"),
    (1, 16, 4, 512, 64, torch.bfloat16, 13, 1.0, "contiguous"),
    (2, 16, 4, 1024, 64, torch.bfloat16, 7, 0.5, "contiguous"),
    (2, 12, 4, 384, 64, torch.bfloat16, 41, 1.0, "model"),
    (1, 6, 2, 300, 64, torch.bfloat16, 42, 1.0, "contiguous"),
    (1, 8, 8, 129, 32, torch.bfloat16, 43, 1.0, "contiguous"),
    (3, 2, 1, 1, 64, torch.float16, 44, 1.0, "contiguous"),
    (1, 4, 1, 640, 64, torch.float16, 45, 2.0, "model"),
    (1, 9, 3, 2047, 64, torch.bfloat16, 46, 1.0, "contiguous"),  # odd repeats, one short of 16 tiles
    (1, 8, 1, 200, 32, torch.float16, 47, 1.0, "model"),         # repeats 8, D 32, model layout
]


@pytest.mark.parametrize("B,Hq,Hkv,T,D,dtype,seed,scale,layout", FWD_CASES)
def test_attention_forward_matches_oracle(cuda_device, B, Hq, Hkv, T, D, dtype, seed, scale, layout):
    from mega_trading_b200 import _lib
    from mega_trading_b200.kernels import triton_attention as A

    q, k, v, _ = _inputs(B, Hq, Hkv, T, D, seed, scale, layout)
    qd, kd, vd = (_to_dev(t, cuda_device, dtype, layout) for t in (q, k, v))
    with torch.no_grad():
        o = A.triton_attention(qd, kd, vd, repeats=Hq // Hkv)
        o2, lse = A._launch_fwd(qd, kd, vd, Hq // Hkv, 1.0 / D ** 0.5)
    torch.cuda.synchronize()
    assert _lib.read_status(cuda_device) == 0
    assert o.shape == q.shape and o.stride() == qd.stride()
    qo, ko, vo = (t.to(dtype).float() for t in (q, k, v))
    ref = O.causal_gqa_attention(qo, ko, vo, Hq // Hkv)
    _check(o, ref, "attention O", atol=6e-2)
    assert torch.equal(o, o2)
    ref_lse = O.attention_lse(qo, ko, Hq // Hkv)
    err = float((lse.cpu() - ref_lse).abs().max())
    assert err < 2e-2, f"lse max abs error {err}"


BWD_CASES = [
    (1, 4, 2, 17, 32, torch.float16, 11, 1.0, "contiguous"),
    (1, 16, 4, 512, 64, torch.bfloat16, 17, 1.0, "contiguous"),
    (2, 16, 4, 1024, 64, torch.bfloat16, 7, 0.5, "contiguous"),
    (2, 12, 4, 384, 64, torch.bfloat16, 51, 1.0, "model"),
    (1, 6, 2, 300, 64, torch.bfloat16, 52, 1.0, "contiguous"),
    (1, 8, 8, 129, 32, torch.bfloat16, 53, 1.0, "contiguous"),
    (3, 2, 1, 1, 64, torch.float16, 54, 1.0, "contiguous"),
    (1, 4, 1, 640, 64, torch.float16, 55, 2.0, "model"),       # fp16, repeats 4, scaled inputs
    (1, 9, 3, 257, 64, torch.bfloat16, 56, 1.0, "contiguous"),  # odd repeats, one past a tile
    (1, 4, 2, 1000, 32, torch.bfloat16, 57, 1.0, "model"),      # D 32 at a longer ragged T
    (1, 8, 1, 200, 64, torch.bfloat16, 58, 1.0, "contiguous"),  # repeats 8 (one kv head)
]


@pytest.mark.parametrize("B,Hq,Hkv,T,D,dtype,seed,scale,layout", BWD_CASES)
def test_attention_backward_matches_oracle(cuda_device, B, Hq, Hkv, T, D, dtype, seed, scale, layout):
    from mega_trading_b200 import _lib
    from mega_trading_b200.kernels import triton_attention as A

    if not hasattr(_lib.load(), "mt_attention_bwd"):
        pytest.skip("attention backward not built")
    q, k, v, do = _inputs(B, Hq, Hkv, T, D, seed, scale, layout)
    qd, kd, vd = (_to_dev(t, cuda_device, dtype, layout) for t in (q, k, v))
    o = A.triton_attention(qd, kd, vd, repeats=Hq // Hkv)
    o.backward(do.to(cuda_device, dtype))
    torch.cuda.synchronize()
    assert _lib.read_status(cuda_device) == 0
    qo, ko, vo = (t.to(dtype).float().requires_grad_(True) for t in (q, k, v))
    ref = O.causal_gqa_attention(qo, ko, vo, Hq // Hkv)
    ref.backward(do.to(dtype).float())
    _check(o, ref, "attention O", atol=6e-2)
    _check(qd.grad, qo.grad, "attention dq", atol=8e-2)
    _check(kd.grad, ko.grad, "attention dk", atol=8e-2)
    _check(vd.grad, vo.grad, "attention dv", atol=8e-2)


def test_timing_hook_times_the_main_kernel(cuda_device):
    """mt_set_timing_events: the library records caller events around its main
    attention kernels; that time is positive and within the whole call's."""
    from mega_trading_b200 import _lib
    from mega_trading_b200.kernels import triton_attention as A

    g = torch.Generator(device=cuda_device).manual_seed(81)
    q = torch.randn(4, 8, 1024, 64, device=cuda_device, generator=g).bfloat16()
    k = torch.randn(4, 2, 1024, 64, device=cuda_device, generator=g).bfloat16()
    v = torch.randn(4, 2, 1024, 64, device=cuda_device, generator=g).bfloat16()
    _lib.timer.reset()
    _lib.timer.enabled = True
    try:
        o, lse = A._launch_fwd(q, k, v, 4, 0.125)
        A._launch_bwd(q, k, v, o, lse, torch.ones_like(o), 0.125)
    finally:
        _lib.timer.enabled = False
    s = _lib.timer.summary()
    for name in ("attention_fwd", "attention_bwd"):
        n_all, ms_all = s[name]
        n_k, ms_k = s[name + "_kernel"]
        assert n_all == n_k == 1
        assert 0.0 < ms_k <= ms_all
    # the hook is cleared after each call: a plain call records nothing
    assert _lib.load().mt_set_timing_events(None, None) == 0
