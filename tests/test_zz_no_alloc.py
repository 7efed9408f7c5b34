"""The no-allocation RMSNorm backward entry point against the allocating one.

``mt_rms_norm_bwd_noalloc`` serves callers that cannot allocate device memory
where they call the library (an FFI host without its own device allocator, or
a step that must not call cudaMalloc because it synchronises the device): its
dW scratch is a static device array inside the library instead of a
caller-provided workspace.  This file runs last so that a failure here leaves
every other test already run; it must also pass alone in a fresh process.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from oracle import ops as O

pytestmark = pytest.mark.gpu

TOL = 2e-2  # the normwise tolerance the parity tests use


def _fwd(lib, _lib, x, w):
    rows, dim = x.shape
    y = torch.empty_like(x)
    rstd = torch.empty(rows, device=x.device, dtype=torch.float32)
    st = lib.mt_rms_norm_fwd(x.data_ptr(), _lib.dtype_code(x.dtype), w.data_ptr(), _lib.dtype_code(w.dtype),
                             y.data_ptr(), _lib.dtype_code(x.dtype), rstd.data_ptr(), rows, dim, 1e-5,
                             _lib.stream_ptr(x.device))
    _lib.check(st, "mt_rms_norm_fwd")
    return rstd


def _bwd_alloc(lib, _lib, x, w, rstd, dy):
    rows, dim = x.shape
    dx = torch.empty_like(x)
    dw = torch.empty_like(w)
    ws = torch.empty(int(lib.mt_rms_norm_bwd_workspace_bytes(rows, dim)), device=x.device, dtype=torch.uint8)
    st = lib.mt_rms_norm_bwd(x.data_ptr(), _lib.dtype_code(x.dtype), w.data_ptr(), _lib.dtype_code(w.dtype),
                             rstd.data_ptr(), dy.data_ptr(), _lib.dtype_code(dy.dtype), dx.data_ptr(),
                             _lib.dtype_code(dx.dtype), dw.data_ptr(), _lib.dtype_code(dw.dtype), ws.data_ptr(),
                             ws.numel(), rows, dim, _lib.stream_ptr(x.device))
    _lib.check(st, "mt_rms_norm_bwd")
    return dx, dw


def _bwd_noalloc(lib, _lib, x, w, rstd, dy):
    rows, dim = x.shape
    dx = torch.empty_like(x)
    dw = torch.empty_like(w)
    st = lib.mt_rms_norm_bwd_noalloc(x.data_ptr(), _lib.dtype_code(x.dtype), w.data_ptr(), _lib.dtype_code(w.dtype),
                                     rstd.data_ptr(), dy.data_ptr(), _lib.dtype_code(dy.dtype), dx.data_ptr(),
                                     _lib.dtype_code(dx.dtype), dw.data_ptr(), _lib.dtype_code(dw.dtype), rows, dim,
                                     _lib.stream_ptr(x.device))
    _lib.check(st, "mt_rms_norm_bwd_noalloc")
    return dx, dw


def test_noalloc_rms_norm_bwd_matches_allocating_entry_point(cuda_device):
    from mega_trading_b200 import _lib

    lib = _lib.load()
    g = torch.Generator(device=cuda_device).manual_seed(77)
    # two calls in a row with different sizes: the second must not see the first's scratch contents
    for rows, dim in ((65536, 768), (3000, 1024)):
        x = torch.randn(rows, dim, device=cuda_device, generator=g).bfloat16()
        w = (1 + 0.1 * torch.randn(dim, device=cuda_device, generator=g)).bfloat16()
        dy = torch.randn(rows, dim, device=cuda_device, generator=g).bfloat16()
        rstd = _fwd(lib, _lib, x, w)
        dx_ref, dw_ref = _bwd_alloc(lib, _lib, x, w, rstd, dy)
        dx, dw = _bwd_noalloc(lib, _lib, x, w, rstd, dy)
        torch.cuda.synchronize()
        assert O.max_rel_error(dx, dx_ref) <= TOL
        assert O.max_rel_error(dw, dw_ref) <= TOL
        assert torch.equal(dx, dx_ref)  # same per-row kernel: identical dx


def test_noalloc_rejects_rows_wider_than_its_scratch(cuda_device):
    from mega_trading_b200 import _lib

    lib = _lib.load()
    x = torch.zeros(4, 4104, device=cuda_device, dtype=torch.bfloat16)
    w = torch.ones(4104, device=cuda_device, dtype=torch.bfloat16)
    rstd = torch.ones(4, device=cuda_device)
    dx = torch.empty_like(x)
    dw = torch.empty_like(w)
    st = lib.mt_rms_norm_bwd_noalloc(x.data_ptr(), 2, w.data_ptr(), 2, rstd.data_ptr(), x.data_ptr(), 2,
                                     dx.data_ptr(), 2, dw.data_ptr(), 2, 4, 4104, _lib.stream_ptr(x.device))
    assert st == 7  # MT_ERR_WORKSPACE
    assert b"4096" in lib.mt_last_error()
    assert ctypes.sizeof(ctypes.c_int) == 4
