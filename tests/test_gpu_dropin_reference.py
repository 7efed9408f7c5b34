"""The drop-in claim, tested on the reference's own model code.

duoan/mega-trading installed under ``baseline/_ref`` (``pip install --target``;
its package ``__init__`` needs ``accelerate``, so the modules are imported
through a stub package) builds ``TradingModel(attention_backend="triton",
dropout=0)``.  ``install()`` rebinds the model module's operator aliases
(``src/mega_trading/model.py:11-17``) to the sm_100a kernels; the model then
runs its forward_with_loss + backward under the bf16 autocast its trainer uses
(``src/mega_trading/trainer.py:336``).  It is compared with

* the same reference model and weights on its own torch operators
  (``attention_backend="auto"``), same autocast: loss within 1e-3 relative,
  every parameter gradient within 2e-2 normwise max relative error;
* the CPU fp32 oracle with the same weights: loss within 2e-3 (bf16
  activations over the layers against fp32), gradients within 5e-2.

Skipped when no installed reference is present.
"""

from __future__ import annotations

import pytest
import torch

from oracle import model as ref_oracle
from oracle import ops as O

pytestmark = pytest.mark.gpu


def _reference():
    from mega_trading_b200.microbench import load_reference

    r = load_reference()
    if r is None:
        pytest.skip("no installed reference under baseline/_ref")
    return r


def _build(model_mod, backend, cfg, state=None):
    torch.manual_seed(0)
    m = model_mod.TradingModel(attention_backend=backend, dropout=0.0, **cfg).cuda()
    if state is not None:
        m.load_state_dict(state)
    return m


def _loss_and_grads(m, ids, labels):
    with torch.autocast("cuda", dtype=torch.bfloat16):
        loss, _ = m.forward_with_loss(ids, labels, return_logits=False)
    loss.float().backward()
    return loss.detach().float(), {k: p.grad.detach().float().clone() for k, p in m.named_parameters()}


def test_reference_model_with_installed_kernels(cuda_device):
    _, _, model_mod = _reference()
    from mega_trading_b200 import _lib, install
    from mega_trading_b200.data import next_token_batch

    cfg = dict(vocab_size=1024, block_size=256, hidden_dim=256, layers=2, attention_heads=4, kv_heads=2,
               intermediate_dim=512, rope_theta=10_000.0)
    ids, labels = next_token_batch(4, 256, seed=31)
    ids, labels = (ids % 1024).cuda(), (labels % 1024).cuda()
    base = _build(model_mod, "auto", cfg)
    state = {k: v.detach().clone() for k, v in base.state_dict().items()}
    loss_t, grads_t = _loss_and_grads(base, ids, labels)

    saved = {name: getattr(model_mod, name) for name in install.ALIASES}
    try:
        install.install(model_mod, kernel_modules=False)
        for name, fn in install.ALIASES.items():
            assert getattr(model_mod, name) is fn
        launches0 = _lib.launch_count()
        fast = _build(model_mod, "triton", cfg, state)
        loss_k, grads_k = _loss_and_grads(fast, ids, labels)
        torch.cuda.synchronize()
        assert _lib.read_status(cuda_device) == 0
        assert _lib.launch_count() > launches0, "the reference model did not reach the sm_100a kernels"
    finally:
        for name, fn in saved.items():
            setattr(model_mod, name, fn)

    rel = abs(float(loss_k) - float(loss_t)) / abs(float(loss_t))
    assert rel <= 1e-3, f"loss {float(loss_k):.6f} vs reference torch path {float(loss_t):.6f} (rel {rel:.2e})"
    assert grads_k.keys() == grads_t.keys()
    for k in grads_t:
        err = O.max_rel_error(grads_k[k], grads_t[k])
        assert err <= 2e-2, f"{k}: max relative error {err:.3e} vs the reference's torch path"

    # against the fp32 CPU oracle of the same weights
    oracle = ref_oracle.TradingModelRef(ref_oracle.ModelConfig(**cfg))
    oracle.load_state_dict({k: v.detach().cpu().float() for k, v in state.items()})
    lo, _ = oracle.forward_with_loss(ids.cpu(), labels.cpu())
    lo.backward()
    rel = abs(float(loss_k) - float(lo.detach())) / abs(float(lo.detach()))
    assert rel <= 2e-3, f"loss {float(loss_k):.6f} vs oracle {float(lo.detach()):.6f}"
    for k, p in oracle.named_parameters():
        err = O.max_rel_error(grads_k[k], p.grad)
        assert err <= 5e-2, f"{k}: max relative error {err:.3e} vs the fp32 oracle"
