"""GPU parity of the fused linear + cross-entropy against the CPU fp32 oracle.

Cases: the reference's kernel test (``tests/test_training.py:767-811`` of
duoan/mega-trading: rows 256, hidden 256, vocab 4096, ``labels[::31] = -100``,
seed 43, hidden*0.5, weight*0.02), the all-ignored case (:750-765), ragged
rows / vocab, int32 labels, and a BASELINE config-2 slice (hidden 768,
vocab 21,504).  Tolerances: loss 1e-3 relative (BASELINE), gradients 2e-2
normwise max relative error; plus the reference's own 5e-3 / 5e-2 allclose.
"""

from __future__ import annotations

import pytest
import torch

from oracle import ops as O

pytestmark = pytest.mark.gpu


def _case(cuda_device, rows, hdim, vocab, seed, ignore_every=0, int32=False, hscale=0.5, dtype=torch.bfloat16,
          grad_scale=1.0):
    from mega_trading_b200 import _lib
    from mega_trading_b200.kernels import triton_ops as K

    g = torch.Generator().manual_seed(seed)
    hidden = (torch.randn(rows, hdim, generator=g) * hscale).to(dtype)
    weight = (torch.randn(vocab, hdim, generator=g) * 0.02).to(dtype)
    labels = torch.randint(0, vocab, (rows,), generator=g, dtype=torch.long)
    if ignore_every:
        labels[::ignore_every] = -100
    if int32:
        labels = labels.to(torch.int32)
    hd = hidden.to(cuda_device).requires_grad_(True)
    wd = weight.to(cuda_device).requires_grad_(True)
    loss = K.triton_fused_linear_cross_entropy(hd, wd, labels.to(cuda_device), ignore_index=-100)
    (loss * grad_scale).backward()
    torch.cuda.synchronize()
    assert _lib.read_status(cuda_device) == 0
    ho = hidden.float().requires_grad_(True)
    wo = weight.float().requires_grad_(True)
    lo = O.linear_cross_entropy(ho, wo, labels.long(), -100)
    (lo * grad_scale).backward()
    return loss, lo, hd.grad, ho.grad, wd.grad, wo.grad


def _check_grads(dh, dho, dw, dwo):
    for name, a, b in (("dhidden", dh, dho), ("dweight", dw, dwo)):
        err = O.max_rel_error(a, b)
        assert err <= 2e-2, f"{name}: max relative error {err:.3e}"


def test_fused_ce_reference_case(cuda_device):
    loss, lo, dh, dho, dw, dwo = _case(cuda_device, 256, 256, 4096, 43, ignore_every=31)
    assert loss.dtype == torch.float32 and loss.shape == ()
    rel = abs(float(loss.detach()) - float(lo.detach())) / abs(float(lo.detach()))
    assert rel <= 1e-3, f"loss rel err {rel:.3e}"
    assert torch.allclose(loss.cpu(), lo.detach(), atol=5e-3, rtol=5e-3)
    assert torch.allclose(dh.float().cpu(), dho, atol=5e-2, rtol=5e-2)
    assert torch.allclose(dw.float().cpu(), dwo, atol=5e-2, rtol=5e-2)
    _check_grads(dh, dho, dw, dwo)


@pytest.mark.parametrize("rows,hdim,vocab,seed,ignore_every,int32,dtype", [
    (77, 64, 1000, 1, 0, False, torch.bfloat16),
    (300, 128, 17, 2, 5, True, torch.bfloat16),
    (129, 768, 2000, 3, 7, False, torch.float16),
    (2048, 768, 21504, 4, 0, False, torch.bfloat16),
])
def test_fused_ce_shapes(cuda_device, rows, hdim, vocab, seed, ignore_every, int32, dtype):
    loss, lo, dh, dho, dw, dwo = _case(cuda_device, rows, hdim, vocab, seed, ignore_every, int32, dtype=dtype,
                                       grad_scale=0.7)
    rel = abs(float(loss.detach()) - float(lo.detach())) / abs(float(lo.detach()))
    assert rel <= 1e-3, f"loss rel err {rel:.3e}"
    _check_grads(dh, dho, dw, dwo)


@pytest.mark.parametrize("rows,hdim,vocab,seed", [
    (1000, 1024, 3000, 11),   # hidden split over a cluster of 3 CTAs (384 + 384 + 256)
    (200, 1280, 500, 12),     # two hidden-column groups (1152 + 128)
    (64, 104, 300, 13),       # one partial 128-column slice
    (4096, 256, 21504, 14),   # BASELINE config-0 widths: one CTA per cluster, vocab split
    (130, 768, 129, 15),      # ragged rows and vocab tiles
])
def test_fused_ce_backward_shapes(cuda_device, rows, hdim, vocab, seed):
    loss, lo, dh, dho, dw, dwo = _case(cuda_device, rows, hdim, vocab, seed, ignore_every=9, grad_scale=1.3)
    rel = abs(float(loss.detach()) - float(lo.detach())) / abs(float(lo.detach()))
    assert rel <= 1e-3, f"loss rel err {rel:.3e}"
    _check_grads(dh, dho, dw, dwo)


def test_fused_ce_fp32_master_weight(cuda_device):
    """fp32 weight (the reference's autocast case): the kernels read its bf16 rounding and dW
    comes back in fp32, accumulated without a 16-bit rounding (triton_ops.py:352-357)."""
    from mega_trading_b200.kernels import fused_ce as F
    from mega_trading_b200.kernels import triton_ops as K

    g = torch.Generator().manual_seed(21)
    hidden = (torch.randn(512, 768, generator=g) * 0.5).to(torch.bfloat16)
    weight = torch.randn(5000, 768, generator=g) * 0.02
    labels = torch.randint(0, 5000, (512,), generator=g)
    hd = hidden.to(cuda_device).requires_grad_(True)
    wd = weight.to(cuda_device).requires_grad_(True)
    loss = K.triton_fused_linear_cross_entropy(hd, wd, labels.to(cuda_device))
    loss.backward()
    assert wd.grad.dtype == torch.float32 and hd.grad.dtype == torch.bfloat16
    ho = hidden.float().requires_grad_(True)
    wo = weight.to(torch.bfloat16).float().requires_grad_(True)
    O.linear_cross_entropy(ho, wo, labels, -100).backward()
    _check_grads(hd.grad, ho.grad, wd.grad, wo.grad)
    # the fp32 gradient is not a 16-bit value: it carries bits below bf16's mantissa
    assert bool((wd.grad != wd.grad.to(torch.bfloat16).float()).any())
    # a 16-bit compute copy with the gradient sent to the fp32 weight (the model's path)
    wd2 = weight.to(cuda_device).requires_grad_(True)
    hd2 = hidden.to(cuda_device).requires_grad_(True)
    loss2 = F.fused_linear_cross_entropy(hd2, wd2, labels.to(cuda_device), compute_weight=wd2.detach().bfloat16())
    loss2.backward()
    assert torch.equal(loss2, loss.detach())
    assert torch.equal(wd2.grad, wd.grad) and torch.equal(hd2.grad, hd.grad)


def test_fused_ce_backward_is_deterministic(cuda_device):
    from mega_trading_b200.kernels import triton_ops as K

    g = torch.Generator(device=cuda_device).manual_seed(3)
    h = torch.randn(3000, 768, device=cuda_device, generator=g).bfloat16()
    w = (torch.randn(21504, 768, device=cuda_device, generator=g) * 0.02).bfloat16()
    lab = torch.randint(0, 21504, (3000,), device=cuda_device, generator=g)
    grads = []
    for _ in range(2):
        hd, wd = h.clone().requires_grad_(True), w.float().requires_grad_(True)
        K.triton_fused_linear_cross_entropy(hd, wd, lab).backward()
        grads.append((hd.grad, wd.grad))
    assert torch.equal(grads[0][0], grads[1][0]) and torch.equal(grads[0][1], grads[1][1])


def test_fused_ce_all_ignored(cuda_device):
    from mega_trading_b200.kernels import triton_ops as K

    hidden = torch.randn(4, 64, device=cuda_device, dtype=torch.bfloat16, requires_grad=True)
    weight = torch.randn(11, 64, device=cuda_device, dtype=torch.bfloat16, requires_grad=True)
    labels = torch.full((4,), -100, dtype=torch.long, device=cuda_device)
    loss = K.triton_fused_linear_cross_entropy(hidden, weight, labels, ignore_index=-100)
    loss.backward()
    assert float(loss.detach()) == 0.0
    assert bool((hidden.grad == 0).all()) and bool((weight.grad == 0).all())


def test_fused_ce_validation_messages(cuda_device):
    from mega_trading_b200.kernels import triton_ops as K

    h = torch.randn(4, 64, device=cuda_device, dtype=torch.bfloat16)
    w = torch.randn(11, 64, device=cuda_device, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="hidden must have shape"):
        K.triton_fused_linear_cross_entropy(h[None], w, torch.zeros(4, dtype=torch.long, device=cuda_device))
    with pytest.raises(ValueError, match="labels must be an integer tensor"):
        K.triton_fused_linear_cross_entropy(h, w, torch.zeros(4, device=cuda_device))


def test_fused_ce_out_of_range_labels_set_the_status_word(cuda_device):
    """A target outside [0, V) that is not ignore_index (torch's cross_entropy, the reference's
    CPU path, rejects it) is turned by the kernels' own bounds check into a status code
    ((3 << 16) | 0xEEEE) instead of an out-of-bounds read; the row contributes no loss and no
    gradient, exactly like an ignored row."""
    from mega_trading_b200 import _lib
    from mega_trading_b200.kernels import triton_ops as K

    g = torch.Generator().manual_seed(21)
    hidden = (torch.randn(40, 64, generator=g) * 0.5).bfloat16()
    weight = (torch.randn(50, 64, generator=g) * 0.02).bfloat16()
    labels = torch.randint(0, 50, (40,), generator=g, dtype=torch.long)
    labels[3], labels[7], labels[11] = 50, -5, -100
    assert _lib.read_status(cuda_device) == 0
    hd = hidden.to(cuda_device).requires_grad_(True)
    wd = weight.to(cuda_device).requires_grad_(True)
    loss = K.triton_fused_linear_cross_entropy(hd, wd, labels.to(cuda_device), ignore_index=-100)
    loss.backward()
    code = _lib.read_status(cuda_device)  # reads and clears
    assert code == (3 << 16) | 0xEEEE, hex(code)
    assert "out of range" in _lib.describe_status(code)
    masked = labels.clone()
    masked[3] = masked[7] = -100
    ho = hidden.float().requires_grad_(True)
    wo = weight.float().requires_grad_(True)
    lo = O.linear_cross_entropy(ho, wo, masked, -100)
    lo.backward()
    rel = abs(float(loss.detach()) - float(lo.detach())) / abs(float(lo.detach()))
    assert rel <= 1e-3, f"loss rel err {rel:.3e}"
    assert bool((hd.grad[3] == 0).all()) and bool((hd.grad[7] == 0).all())
    _check_grads(hd.grad, ho.grad, wd.grad, wo.grad)
    assert _lib.read_status(cuda_device) == 0
