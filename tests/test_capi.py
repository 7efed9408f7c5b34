"""The C-ABI library loads on a CPU-only host, exports every symbol the header
declares, and rejects invalid arguments before touching a GPU."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "mt_b200.h"


def _declared() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"MT_API\s+[\w\s\*]+?\b(mt_\w+)\s*\(", text))


def test_header_declares_the_hot_path():
    names = _declared()
    for n in ("mt_rms_norm_fwd", "mt_rms_norm_bwd", "mt_add_rms_norm_fwd", "mt_add_rms_norm_bwd", "mt_rope",
              "mt_swiglu_fwd", "mt_swiglu_bwd", "mt_attention_fwd", "mt_attention_bwd", "mt_fused_ce_fwd",
              "mt_fused_ce_bwd", "mt_debug_wait_timeout", "mt_launch_count"):
        assert n in names


def test_library_exports_every_declared_symbol():
    from mega_trading_b200 import _lib

    lib = _lib.load()
    missing = [n for n in sorted(_declared()) if not hasattr(lib, n)]
    assert not missing, missing
    assert set(_lib.PROTOTYPES) == _declared()
    assert lib.mt_built_arch() == 100
    assert lib.mt_status_string(0) == b"ok"
    assert lib.mt_status_string(6) == b"device-side wait timed out"
    assert lib.mt_launch_count() >= 0


def test_invalid_arguments_are_rejected_without_a_gpu():
    from mega_trading_b200 import _lib

    lib = _lib.load()
    s = _lib.i64_array([0, 0, 0, 1])
    # unsupported dtype (fp32 attention) and head_dim
    assert lib.mt_attention_fwd(None, None, None, None, None, 0, 1, 1, 1, 8, 64, s, s, s, s, 1.0, None, 0, None, None) == 2
    assert lib.mt_attention_fwd(None, None, None, None, None, 2, 1, 1, 1, 8, 48, s, s, s, s, 1.0, None, 0, None, None) == 1
    # GQA head counts that do not divide
    assert lib.mt_attention_fwd(None, None, None, None, None, 2, 1, 3, 2, 8, 64, s, s, s, s, 1.0, None, 0, None, None) == 1
    # empty batch is a no-op
    assert lib.mt_attention_fwd(None, None, None, None, None, 2, 0, 2, 2, 8, 64, s, s, s, s, 1.0, None, 0, None, None) == 0
    # rms norm: bad dim, unsupported dtype combination
    assert lib.mt_rms_norm_fwd(None, 2, None, 2, None, 2, None, 4, 0, 1e-5, None) == 1
    assert lib.mt_rms_norm_fwd(ctypes.c_void_p(16), 2, None, 1, ctypes.c_void_p(16), 0, None, 4, 8, 1e-5, None) == 2
    # rope: odd head dim; swiglu: negative size / zero size
    assert lib.mt_rope(None, None, None, None, None, None, 2, 1, 1, 1, 4, 5, s, s, s, s, s, s, 0, None) == 1
    assert lib.mt_swiglu_fwd(None, None, None, 2, -1, None) == 1
    assert lib.mt_swiglu_fwd(None, None, None, 2, 0, None) == 0
    # fused CE: K not a multiple of 8, and workspace size query
    assert lib.mt_fused_ce_fwd(ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16), 1, -100, 2, 4, 10,
                               12, None, None, None, 0, None, None) == 3
    assert lib.mt_fused_ce_workspace_bytes(1024, 21504) > 1024 * 4
    assert lib.mt_attention_bwd_workspace_bytes(2, 4, 130, 64) >= 2 * 4 * 256 * 64 * 4
    assert lib.mt_attention_fwd_workspace_bytes(2, 4, 130, 64) >= 4
    # the forward's work-counter workspace: missing, misaligned or too small
    fake = ctypes.c_void_p(4096)
    st16 = _lib.i64_array([4 * 8 * 64, 8 * 64, 64, 1])
    args = (fake, fake, fake, fake, fake, 2, 1, 4, 4, 8, 64, st16, st16, st16, st16, 0.125)
    assert lib.mt_attention_fwd(*args, None, 256, fake, None) == 7
    assert lib.mt_attention_fwd(*args, ctypes.c_void_p(4100), 256, fake, None) == 7
    assert lib.mt_attention_fwd(*args, fake, 8, fake, None) == 7
    # fused AdamW: nothing to do, unsupported copy dtype, missing table
    assert lib.mt_adamw_step(None, 0, 0, 2, 1e-3, 0.9, 0.999, 1e-8, 0.0, 1e-3, 1.0, None, None) == 0
    assert lib.mt_adamw_step(ctypes.c_void_p(16), 1, 8, 0, 1e-3, 0.9, 0.999, 1e-8, 0.0, 1e-3, 1.0, None, None) == 2
    assert lib.mt_adamw_step(None, 1, 8, 2, 1e-3, 0.9, 0.999, 1e-8, 0.0, 1e-3, 1.0, None, None) == 1


@pytest.mark.parametrize("name", ["mt_rms_norm_fwd", "mt_attention_fwd", "mt_fused_ce_fwd"])
def test_prototypes_are_attached(name):
    from mega_trading_b200 import _lib

    fn = getattr(_lib.load(), name)
    assert fn.restype is ctypes.c_int and len(fn.argtypes) == len(_lib.PROTOTYPES[name][1])
