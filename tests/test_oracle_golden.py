"""Pin the CPU oracle against golden vectors produced by the reference's own
PyTorch code (``tests/golden/make_golden.py`` ran duoan/mega-trading's
``model.py`` / ``kernels/triton_ops.py`` torch paths)."""

from __future__ import annotations

from pathlib import Path

import pytest
import torch

from oracle import model as M
from oracle import ops as O

GOLDEN = torch.load(Path(__file__).parent / "golden" / "golden.pt", weights_only=False)
TOL = dict(atol=1e-5, rtol=1e-5)


def _leaf(t):
    return t.clone().requires_grad_(True)


def test_rms_norm_golden():
    g = GOLDEN["rms_norm"]
    x, w = _leaf(g["x"]), _leaf(g["w"])
    y = O.rms_norm(x, w, 1e-5)
    y.backward(g["dy"])
    assert torch.allclose(y, g["y"], **TOL)
    assert torch.allclose(x.grad, g["dx"], **TOL)
    assert torch.allclose(w.grad, g["dw"], **TOL)


def test_add_rms_norm_golden():
    g = GOLDEN["add_rms_norm"]
    h, r, w = _leaf(g["h"]), _leaf(g["r"]), _leaf(g["w"])
    nr, nn_ = O.add_rms_norm(h, r, w, 1e-5)
    torch.autograd.backward([nr, nn_], [g["g_res"], g["g_norm"]])
    assert torch.allclose(nr, g["new_res"], **TOL)
    assert torch.allclose(nn_, g["normed"], **TOL)
    assert torch.allclose(h.grad, g["dh"], **TOL)
    assert torch.allclose(r.grad, g["dr"], **TOL)
    assert torch.allclose(w.grad, g["dw"], **TOL)


def test_rope_golden():
    g = GOLDEN["rope"]
    q, k = _leaf(g["q"]), _leaf(g["k"])
    cos, sin = O.rope_tables(q.shape[-1], q.shape[-2], g["theta"])
    qo, ko = O.apply_rope(q, k, cos, sin, table_dtype=torch.float32)
    torch.autograd.backward([qo, ko], [g["gq"], g["gk"]])
    assert torch.allclose(qo, g["q_out"], **TOL)
    assert torch.allclose(ko, g["k_out"], **TOL)
    assert torch.allclose(q.grad, g["dq"], **TOL)
    assert torch.allclose(k.grad, g["dk"], **TOL)


def test_rope_bf16_golden():
    # the oracle computes in fp32 from bf16 tables/inputs; the reference rounds each bf16 op
    g = GOLDEN["rope_bf16"]
    cos, sin = O.rope_tables(g["q"].shape[-1], g["q"].shape[-2], 500_000.0)
    qo, ko = O.apply_rope(g["q"].float(), g["k"].float(), cos, sin, table_dtype=torch.bfloat16)
    assert O.max_rel_error(qo, g["q_out"]) < 1e-2
    assert O.max_rel_error(ko, g["k_out"]) < 1e-2


def test_swiglu_golden():
    g = GOLDEN["swiglu"]
    a, b = _leaf(g["gate"]), _leaf(g["up"])
    y = O.swiglu_gate(a, b)
    y.backward(g["dy"])
    assert torch.allclose(y, g["y"], **TOL)
    assert torch.allclose(a.grad, g["dgate"], **TOL)
    assert torch.allclose(b.grad, g["dup"], **TOL)
    gb = GOLDEN["swiglu_bf16"]
    yb = O.swiglu_gate(gb["gate"].float(), gb["up"].float(), act_dtype=torch.bfloat16)
    assert torch.equal(yb.to(torch.bfloat16), gb["y"])  # silu rounded to bf16, then one rounding of the product


def test_attention_golden():
    g = GOLDEN["attention"]
    q, k, v = _leaf(g["q"]), _leaf(g["k"]), _leaf(g["v"])
    o = O.causal_gqa_attention(q, k, v, g["repeats"])
    o.backward(g["do"])
    for a, b in ((o, g["o"]), (q.grad, g["dq"]), (k.grad, g["dk"]), (v.grad, g["dv"])):
        assert torch.allclose(a, b, atol=2e-5, rtol=2e-5)


@pytest.mark.parametrize("key", ["fused_ce", "fused_ce_all_ignored"])
def test_fused_ce_golden(key):
    g = GOLDEN[key]
    h, w = _leaf(g["hidden"]), _leaf(g["weight"])
    loss = O.linear_cross_entropy(h, w, g["labels"], -100)
    loss.backward()
    assert torch.allclose(loss, g["loss"], **TOL)
    assert torch.allclose(h.grad, g["dh"], **TOL)
    assert torch.allclose(w.grad, g["dw"], **TOL)


@pytest.mark.parametrize("key", ["fused_ce", "fused_ce_all_ignored"])
@pytest.mark.parametrize("chunk", [7, 64, 8192])
def test_chunked_ce_gradients_golden(key, chunk):
    """The analytic chunked restatement (used at config-2 sizes) against the reference's outputs."""
    g = GOLDEN[key]
    loss, dh, dw = O.linear_cross_entropy_grads(g["hidden"], g["weight"], g["labels"], -100, chunk_rows=chunk)
    assert torch.allclose(loss, g["loss"].float(), **TOL)
    assert torch.allclose(dh, g["dh"], **TOL)
    assert torch.allclose(dw, g["dw"], **TOL)


def test_model_golden():
    g = GOLDEN["model"]
    c = g["config"]
    cfg = M.ModelConfig(vocab_size=c["vocab_size"], block_size=c["block_size"], hidden_dim=c["hidden_dim"],
                        layers=c["layers"], attention_heads=c["attention_heads"], kv_heads=c["kv_heads"],
                        intermediate_dim=c["intermediate_dim"], rope_theta=c["rope_theta"], norm_eps=c["norm_eps"])
    m = M.TradingModelRef(cfg)
    missing, unexpected = m.load_state_dict(g["state_dict"], strict=False)
    assert not unexpected and all(k.endswith(("cos", "sin")) for k in missing)
    loss, _ = m.forward_with_loss(g["input_ids"], g["labels"])
    loss.backward()
    assert torch.allclose(loss, g["loss"], atol=1e-5, rtol=1e-5)
    grads = dict(m.named_parameters())
    for name, ref in g["grads"].items():
        assert torch.allclose(grads[name].grad, ref, atol=1e-5, rtol=1e-4), name


def test_parameter_names_match_reference():
    from mega_trading_b200.model import ModelConfig, TradingModelB200

    g = GOLDEN["model"]
    c = g["config"]
    cfg = ModelConfig(vocab_size=c["vocab_size"], block_size=c["block_size"], hidden_dim=c["hidden_dim"],
                      layers=c["layers"], attention_heads=c["attention_heads"], kv_heads=c["kv_heads"],
                      intermediate_dim=c["intermediate_dim"], rope_theta=c["rope_theta"])
    ours = {k for k in TradingModelB200(cfg).state_dict() if not k.endswith(("cos", "sin"))}
    ref = {k for k in g["state_dict"] if not k.endswith(("cos", "sin"))}
    assert ours == ref
