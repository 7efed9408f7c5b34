"""Whole-model parity: the B200 model (bf16 GEMMs, sm_100a operators) against
the CPU fp32 restatement of the reference ``TradingModel`` with identical
weights, plus a few optimizer steps of the data-parallel trainer."""

from __future__ import annotations

import pytest
import torch

from oracle import model as ref
from oracle import ops as O

pytestmark = pytest.mark.gpu


def _pair(cfg_kwargs, device, seed=0):
    from mega_trading_b200.model import ModelConfig, TradingModelB200

    torch.manual_seed(seed)
    cfg = ModelConfig(**cfg_kwargs)
    m = TradingModelB200(cfg).to(device)
    o = ref.TradingModelRef(ref.ModelConfig(**cfg_kwargs))
    o.load_state_dict({k: v.detach().cpu().float() for k, v in m.state_dict().items()})
    return m, o


DEMO = dict(vocab_size=21504, block_size=512, hidden_dim=256, layers=4, attention_heads=8, kv_heads=2,
            intermediate_dim=688, rope_theta=10_000.0)
GQA12_SMALL = dict(vocab_size=21504, block_size=1024, hidden_dim=768, layers=2, attention_heads=12, kv_heads=4,
                   intermediate_dim=2048)
# BASELINE config 4's layer shapes (d_model 1024, 16/4 heads, SwiGLU 2816) at its
# sequence length 4096, two layers
LARGE24_SLICE = dict(vocab_size=21504, block_size=4096, hidden_dim=1024, layers=2, attention_heads=16, kv_heads=4,
                     intermediate_dim=2816)


@pytest.mark.parametrize("cfg_kwargs,batch,seq", [(DEMO, 2, 512), (GQA12_SMALL, 1, 1024), (LARGE24_SLICE, 1, 4096)])
def test_model_loss_and_grads_match_oracle(cuda_device, cfg_kwargs, batch, seq):
    from mega_trading_b200 import _lib
    from mega_trading_b200.data import next_token_batch

    m, o = _pair(cfg_kwargs, cuda_device)
    ids, labels = next_token_batch(batch, seq, seed=11)
    loss, _ = m.forward_with_loss(ids.to(cuda_device), labels.to(cuda_device))
    loss.backward()
    torch.cuda.synchronize()
    assert _lib.read_status(cuda_device) == 0
    lo, _ = o.forward_with_loss(ids, labels)
    lo.backward()
    rel = abs(float(loss.detach()) - float(lo.detach())) / float(lo.detach())
    assert rel < 2e-3, f"loss {float(loss.detach()):.6f} vs oracle {float(lo.detach()):.6f}"
    ours = dict(m.named_parameters())
    worst = 0.0
    for name, p in o.named_parameters():
        err = O.max_rel_error(ours[name].grad, p.grad)
        worst = max(worst, err)
        assert err < 5e-2, f"{name}: grad max rel err {err:.3e}"
    print(f"loss rel {rel:.2e}, worst grad err {worst:.2e}")


def test_return_logits_path(cuda_device):
    from mega_trading_b200.data import next_token_batch

    m, o = _pair(DEMO, cuda_device)
    ids, labels = next_token_batch(1, 128, seed=12)
    with torch.no_grad():
        loss, logits = m.forward_with_loss(ids.to(cuda_device), labels.to(cuda_device), return_logits=True)
        fused, none = m.forward_with_loss(ids.to(cuda_device), labels.to(cuda_device))
        lo, _ = o.forward_with_loss(ids, labels)
    assert none is None and logits.shape == (1, 128, 21504)
    assert abs(float(loss.detach()) - float(lo.detach())) / float(lo.detach()) < 2e-3
    assert abs(float(fused.detach()) - float(loss.detach())) / float(loss.detach()) < 2e-3


def test_trainer_steps_reduce_loss(cuda_device):
    from mega_trading_b200.data import next_token_batch
    from mega_trading_b200.model import ModelConfig
    from mega_trading_b200.train import Trainer

    cfg = ModelConfig(**DEMO)
    tr = Trainer(cfg, micro_batch=2, device=cuda_device, lr=1e-3)
    ids, labels = next_token_batch(4, 512, seed=13, device=cuda_device)
    losses = [float(tr.step(ids, labels)) for _ in range(8)]
    assert losses[-1] < losses[0] - 0.5, losses
