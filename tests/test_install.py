"""The drop-in installer rebinds the reference model's operator aliases."""

from __future__ import annotations

import types

import pytest


def _fake_model_module():
    mod = types.ModuleType("fake_mega_trading_model")
    for name in ("_triton_attention", "_triton_apply_rope", "_triton_fused_linear_cross_entropy",
                 "_triton_rms_norm", "_triton_swiglu_gate"):
        setattr(mod, name, object())
    return mod


def test_install_rebinds_every_alias():
    from mega_trading_b200 import install as inst
    from mega_trading_b200.kernels import triton_attention, triton_ops

    mod = inst.install(_fake_model_module())
    assert mod._triton_attention is triton_attention.triton_attention
    assert mod._triton_apply_rope is triton_ops.triton_apply_rope
    assert mod._triton_fused_linear_cross_entropy is triton_ops.triton_fused_linear_cross_entropy
    assert mod._triton_rms_norm is triton_ops.triton_rms_norm
    assert mod._triton_swiglu_gate is triton_ops.triton_swiglu_gate


def test_install_rejects_foreign_modules():
    from mega_trading_b200 import install as inst

    with pytest.raises(AttributeError, match="operator alias"):
        inst.install(types.ModuleType("not_a_model"))


def test_mirror_modules_keep_reference_names_and_signatures():
    import inspect

    from mega_trading_b200.kernels import triton_attention, triton_ops

    sig = inspect.signature(triton_attention.triton_attention)
    assert list(sig.parameters) == ["query", "key", "value", "repeats"]
    assert sig.parameters["repeats"].kind is inspect.Parameter.KEYWORD_ONLY
    assert list(inspect.signature(triton_ops.triton_rms_norm).parameters) == ["hidden", "weight", "eps"]
    assert list(inspect.signature(triton_ops.triton_add_rms_norm).parameters) == ["hidden", "residual", "weight",
                                                                                   "eps"]
    assert list(inspect.signature(triton_ops.triton_apply_rope).parameters) == ["query", "key", "cos", "sin"]
    assert list(inspect.signature(triton_ops.triton_swiglu_gate).parameters) == ["gate", "up"]
    ce = inspect.signature(triton_ops.triton_fused_linear_cross_entropy)
    assert list(ce.parameters) == ["hidden", "weight", "labels", "ignore_index"]
    assert ce.parameters["ignore_index"].default == -100
