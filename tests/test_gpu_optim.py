"""GPU parity of the fused AdamW (``mt_adamw_step`` via ``optim.AdamWShadow``)
against the reference's optimizer, ``torch.optim.AdamW(fused=True)``
(duoan/mega-trading ``src/mega_trading/trainer.py:535-545``), on the same
parameters and gradients, and of the bf16 weight copies it writes.

Tolerance: fp32 update rounding (the two kernels order their fp32 operations
differently): rtol 1e-5 / atol 1e-7 on weights and moments after several
steps; the bf16 copies must equal the rounded weights exactly.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _params(dev, shapes, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return [torch.nn.Parameter((torch.randn(s, generator=g) * 0.02).to(dev)) for s in shapes]


@pytest.mark.parametrize("wd,lr", [(0.01, 2e-4), (0.0, 1e-3), (0.1, 3e-2)])
def test_fused_adamw_matches_torch_adamw(wd, lr):
    from mega_trading_b200.kernels.fused_blocks import GATE_BLOCK
    from mega_trading_b200.optim import AdamWShadow, PackedWeights

    dev = torch.device("cuda", 0)
    # sizes that end inside a 2048-element chunk, span several, and are tiny
    shapes = [(2 * GATE_BLOCK, 40), (2 * GATE_BLOCK, 40), (96, 64), (32, 64), (32, 64), (768,), (3, 5), (1000, 33)]
    ours = _params(dev, shapes, 1)
    ref = [torch.nn.Parameter(p.detach().clone()) for p in ours]
    packed = [PackedWeights(ours[0:2], "interleave", GATE_BLOCK), PackedWeights(ours[2:5], "rows"),
              PackedWeights([ours[7]])]
    opt = AdamWShadow(ours, lr=lr, betas=(0.9, 0.95), eps=1e-8, weight_decay=wd, packed=packed)
    ropt = torch.optim.AdamW(ref, lr=lr, betas=(0.9, 0.95), eps=1e-8, weight_decay=wd, fused=True)
    gen = torch.Generator(device="cpu").manual_seed(7)
    for step in range(4):
        for a, b in zip(ours, ref):
            grad = torch.randn(a.shape, generator=gen).to(dev) * (0.1 if step % 2 else 3.0)
            a.grad = grad.clone()
            b.grad = grad.clone()
        if step == 2:
            ours[5].grad = None  # a parameter without a gradient is left alone, as torch does
            ref[5].grad = None
        opt.step()
        ropt.step()
    torch.cuda.synchronize()
    for a, b in zip(ours, ref):
        torch.testing.assert_close(a.detach(), b.detach(), rtol=1e-5, atol=1e-7)
        sa, sb = opt.state[a], ropt.state[b]
        torch.testing.assert_close(sa["exp_avg"], sb["exp_avg"], rtol=1e-5, atol=1e-9)
        torch.testing.assert_close(sa["exp_avg_sq"], sb["exp_avg_sq"], rtol=1e-5, atol=1e-12)
        assert float(sa["step"]) == float(sb["step"])
    for pw in packed:
        assert torch.equal(pw.tensor, pw.pack()), "bf16 copy differs from the rounded weights"
        assert not pw._stale()


def test_trainer_step_with_fused_adamw_matches_torch_adamw():
    """Three training steps of a small model: the fused optimizer (with the model reading
    its bf16 copies) against torch AdamW (with the model re-packing every forward)."""
    from mega_trading_b200.data import next_token_batch
    from mega_trading_b200.model import ModelConfig
    from mega_trading_b200.train import Trainer

    dev = torch.device("cuda", 0)
    cfg = ModelConfig(vocab_size=1024, block_size=256, hidden_dim=256, layers=2, attention_heads=4, kv_heads=2,
                      intermediate_dim=512, rope_theta=10_000.0)
    a = Trainer(cfg, micro_batch=2, device=dev, lr=1e-3, seed=3)
    b = Trainer(cfg, micro_batch=2, device=dev, lr=1e-3, seed=3)
    assert type(a.opt).__name__ == "AdamWShadow"
    b.opt = torch.optim.AdamW(b.model.parameters(), lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01,
                              fused=True)
    ids, labels = next_token_batch(4, 256, seed=11, device=dev)
    ids, labels = ids % cfg.vocab_size, labels % cfg.vocab_size  # composite ids span 21,504
    for step in range(3):
        la = a.step(ids, labels)
        lb = b.step(ids, labels)
        assert abs(float(la) - float(lb)) <= 1e-4 * abs(float(lb))
        if step == 0:
            # identical gradients in the first step: the updates agree to fp32 rounding
            # (later steps start from weights 1 ulp apart, which Adam's normalised
            # update amplifies for near-zero gradients: compared through the loss)
            for (na, pa), (nb, pb) in zip(a.model.named_parameters(), b.model.named_parameters()):
                assert na == nb
                torch.testing.assert_close(pa.detach(), pb.detach(), rtol=1e-5, atol=1e-7, msg=na)
    for pw in a.model.packed_weights():
        assert pw.owned and torch.equal(pw.tensor, pw.pack())
