"""Generate the golden fixtures from duoan/mega-trading's own PyTorch code.

Run here (where the reference sources are mounted), never on the GPU box:

    python tests/golden/make_golden.py /path/to/mega-trading

It imports the reference's ``mega_trading.model`` and ``mega_trading.kernels.*``
through a stub package (the real ``mega_trading/__init__.py`` imports the
trainer, which needs ``accelerate``), runs their CPU/torch paths on small
seeded inputs and saves inputs, outputs and gradients to ``golden.pt``.
``tests/test_oracle_golden.py`` pins the oracle against these fixtures.
"""

from __future__ import annotations

import sys
import types
from pathlib import Path

import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent


def import_reference(root: Path):
    src = root / "src" / "mega_trading"
    pkg = types.ModuleType("mega_trading")
    pkg.__path__ = [str(src)]
    sys.modules["mega_trading"] = pkg
    import mega_trading.kernels.triton_attention as attn  # noqa: F401
    import mega_trading.kernels.triton_ops as ops
    import mega_trading.model as model

    return model, ops


def _grads(*ts):
    return [t.grad.clone() for t in ts]


def main(root: str) -> None:
    model_mod, ops = import_reference(Path(root))
    out: dict[str, object] = {}

    # RMSNorm (model.RMSNorm -> F.rms_norm; triton_rms_norm falls back to the same on CPU)
    g = torch.Generator().manual_seed(19)
    x = torch.randn(3, 5, 64, generator=g, requires_grad=True)
    w = torch.randn(64, generator=g, requires_grad=True)
    dy = torch.randn(3, 5, 64, generator=g)
    y = ops.triton_rms_norm(x, w, eps=1e-5)
    y.backward(dy)
    out["rms_norm"] = dict(x=x.detach(), w=w.detach(), dy=dy, y=y.detach(), dx=x.grad, dw=w.grad)

    # add + RMSNorm CPU fallback (triton_ops.py:31-41)
    g = torch.Generator().manual_seed(37)
    h = torch.randn(2, 4, 16, generator=g, requires_grad=True)
    r = torch.randn(2, 4, 16, generator=g, requires_grad=True)
    w = torch.randn(16, generator=g, requires_grad=True)
    gr = torch.randn(2, 4, 16, generator=g)
    gn = torch.randn(2, 4, 16, generator=g)
    nr, nn_ = ops.triton_add_rms_norm(h, r, w, eps=1e-5)
    torch.autograd.backward([nr, nn_], [gr, gn])
    out["add_rms_norm"] = dict(h=h.detach(), r=r.detach(), w=w.detach(), g_res=gr, g_norm=gn, new_res=nr.detach(),
                               normed=nn_.detach(), dh=h.grad, dr=r.grad, dw=w.grad)

    # RoPE through the model's RotaryEmbedding (tables cast to the input dtype, model.py:286-294)
    g = torch.Generator().manual_seed(23)
    rope = model_mod.RotaryEmbedding(head_dim=16, max_sequence_length=12, theta=500_000.0)
    q = torch.randn(2, 4, 12, 16, generator=g, requires_grad=True)
    k = torch.randn(2, 2, 12, 16, generator=g, requires_grad=True)
    gq = torch.randn(2, 4, 12, 16, generator=g)
    gk = torch.randn(2, 2, 12, 16, generator=g)
    qo, ko = rope(q, k)
    torch.autograd.backward([qo, ko], [gq, gk])
    out["rope"] = dict(q=q.detach(), k=k.detach(), gq=gq, gk=gk, theta=500_000.0, q_out=qo.detach(),
                       k_out=ko.detach(), dq=q.grad, dk=k.grad)
    # the bf16 variant: tables rounded to bf16 before the rotation
    qb = q.detach().bfloat16()
    kb = k.detach().bfloat16()
    qbo, kbo = rope(qb, kb)
    out["rope_bf16"] = dict(q=qb, k=kb, q_out=qbo, k_out=kbo)

    # SwiGLU gate (model.py:255 / triton_ops CPU fallback)
    g = torch.Generator().manual_seed(29)
    gate = torch.randn(4, 48, generator=g, requires_grad=True)
    up = torch.randn(4, 48, generator=g, requires_grad=True)
    dy = torch.randn(4, 48, generator=g)
    y = ops.triton_swiglu_gate(gate, up)
    y.backward(dy)
    out["swiglu"] = dict(gate=gate.detach(), up=up.detach(), dy=dy, y=y.detach(), dgate=gate.grad, dup=up.grad)
    gb, ub = gate.detach().bfloat16(), up.detach().bfloat16()
    out["swiglu_bf16"] = dict(gate=gb, up=ub, y=ops.triton_swiglu_gate(gb, ub))

    # causal GQA attention: the reference's torch path is SDPA (model.py:228-235)
    g = torch.Generator().manual_seed(11)
    q = torch.randn(1, 4, 17, 32, generator=g, requires_grad=True)
    k = torch.randn(1, 2, 17, 32, generator=g, requires_grad=True)
    v = torch.randn(1, 2, 17, 32, generator=g, requires_grad=True)
    do = torch.randn(1, 4, 17, 32, generator=g)
    o = F.scaled_dot_product_attention(q, k, v, dropout_p=0.0, is_causal=True, enable_gqa=True)
    o.backward(do)
    out["attention"] = dict(q=q.detach(), k=k.detach(), v=v.detach(), do=do, o=o.detach(), dq=q.grad, dk=k.grad,
                            dv=v.grad, repeats=2)

    # fused linear CE CPU fallback incl. ignored rows (triton_ops.py:99-112) and the all-ignored case
    g = torch.Generator().manual_seed(37)
    hid = torch.randn(6, 8, generator=g, requires_grad=True)
    wt = torch.randn(17, 8, generator=g, requires_grad=True)
    lab = torch.randint(0, 17, (6,), generator=g)
    lab[1] = -100
    lab[4] = -100
    loss = ops.triton_fused_linear_cross_entropy(hid, wt, lab, ignore_index=-100)
    loss.backward()
    out["fused_ce"] = dict(hidden=hid.detach(), weight=wt.detach(), labels=lab, loss=loss.detach(), dh=hid.grad,
                           dw=wt.grad)
    hid2 = torch.randn(4, 8, generator=g, requires_grad=True)
    wt2 = torch.randn(11, 8, generator=g, requires_grad=True)
    lab2 = torch.full((4,), -100, dtype=torch.long)
    loss2 = ops.triton_fused_linear_cross_entropy(hid2, wt2, lab2, ignore_index=-100)
    loss2.backward()
    out["fused_ce_all_ignored"] = dict(hidden=hid2.detach(), weight=wt2.detach(), labels=lab2, loss=loss2.detach(),
                                       dh=hid2.grad, dw=wt2.grad)

    # whole model: forward_with_loss + backward of a small TradingModel (torch path, dropout 0)
    torch.manual_seed(53)
    cfg = dict(vocab_size=64, block_size=16, hidden_dim=32, layers=2, attention_heads=4, kv_heads=2,
               intermediate_dim=48, dropout=0.0, rope_theta=10_000.0, norm_eps=1e-5)
    m = model_mod.TradingModel(**cfg)
    ids = torch.randint(0, 64, (2, 16), generator=torch.Generator().manual_seed(54))
    labels = torch.randint(0, 64, (2, 16), generator=torch.Generator().manual_seed(55))
    loss, _ = m.forward_with_loss(ids, labels, return_logits=False)
    loss.backward()
    out["model"] = dict(config=cfg, state_dict={k: v.detach().clone() for k, v in m.state_dict().items()},
                        input_ids=ids, labels=labels, loss=loss.detach(),
                        grads={n: p.grad.clone() for n, p in m.named_parameters()})

    torch.save(out, HERE / "golden.pt")
    print("wrote", HERE / "golden.pt", "keys:", sorted(out))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_golden.py <mega-trading source checkout>")
    main(sys.argv[1])
