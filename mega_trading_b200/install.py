"""Drop-in installation into the reference package.

``mega_trading.model`` binds its operators as module aliases
(duoan/mega-trading ``src/mega_trading/model.py:11-17``) and routes to them
when ``attention_backend == "triton"`` (``model.py:113-122, 225-226, 252-253,
267-268, 292-293``).  ``install()`` rebinds those aliases to the sm_100a
implementations; the reference's own routing tests patch exactly these names
(``tests/test_training.py:454-477, 863``).
"""

from __future__ import annotations

import importlib
import types

from .kernels.triton_attention import triton_attention
from .kernels.triton_ops import (
    triton_add_rms_norm,
    triton_apply_rope,
    triton_fused_linear_cross_entropy,
    triton_rms_norm,
    triton_swiglu_gate,
)

ALIASES = {
    "_triton_attention": triton_attention,
    "_triton_apply_rope": triton_apply_rope,
    "_triton_fused_linear_cross_entropy": triton_fused_linear_cross_entropy,
    "_triton_rms_norm": triton_rms_norm,
    "_triton_swiglu_gate": triton_swiglu_gate,
}

# public names of the reference kernel modules and their B200 replacements
KERNEL_MODULE_FUNCTIONS = {
    "mega_trading.kernels.triton_attention": {"triton_attention": triton_attention},
    "mega_trading.kernels.triton_ops": {
        "triton_rms_norm": triton_rms_norm,
        "triton_add_rms_norm": triton_add_rms_norm,
        "triton_apply_rope": triton_apply_rope,
        "triton_swiglu_gate": triton_swiglu_gate,
        "triton_fused_linear_cross_entropy": triton_fused_linear_cross_entropy,
    },
}


def install(model_module: types.ModuleType | None = None, *, kernel_modules: bool = True) -> types.ModuleType:
    """Point the reference model's operator aliases (and, if importable, the
    reference kernel modules' public functions) at the B200 kernels.

    Returns the patched ``mega_trading.model`` module.  Models must still be
    built with ``attention_backend="triton"`` for the reference to route to
    these aliases, exactly as with its own Triton kernels.
    """
    mod = model_module if model_module is not None else importlib.import_module("mega_trading.model")
    for name, fn in ALIASES.items():
        if not hasattr(mod, name):
            raise AttributeError(f"{mod.__name__} has no operator alias {name!r}; not a mega_trading model module")
        setattr(mod, name, fn)
    if kernel_modules and model_module is None:
        for modname, fns in KERNEL_MODULE_FUNCTIONS.items():
            kmod = importlib.import_module(modname)
            for name, fn in fns.items():
                setattr(kmod, name, fn)
    return mod
