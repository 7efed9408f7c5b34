"""Per-operator microbenchmarks at the BASELINE operator shapes.

``python -m mega_trading_b200.microbench [--ops attention,ce,rmsnorm,addrmsnorm,rope,swiglu] [--iters N]``

* attention: config 1 -- B=16, Hq=16, Hkv=4, D=64, T in {1024, 2048, 4096}
  (``--batch 32 --heads 12 --kv-heads 4 --seqs 2048`` is one config-3 layer),
  q/k/v ~ N(0,1)*0.5, dO ~ N(0,1), forward and backward, TFLOP/s with the
  reference's causal FLOP count (``scripts/benchmark_triton_attention.py:179-190``:
  4*B*Hq*D*T(T+1)/2 forward; backward 2.5x forward).
* ce: config 2 -- N=65,536 rows, hidden 768, vocab 21,504; forward
  (2NHV FLOP) and the logit-gradient kernel (2NHV FLOP).
* torch: the BASELINE torch comparators on the same box (SDPA flash/cuDNN,
  F.rms_norm, eager RoPE, F.silu * up, F.linear + F.cross_entropy).
* mlp: the SwiGLU GEMMs with the gate in the epilogue (2NH*2I forward,
  2NHI backward) against cuBLAS + the standalone packed gate.
* rmsnorm / addrmsnorm / rope / swiglu: config 2 token count, HBM GB/s of the
  algorithmic bytes (each input read once, each output written once).
  addrmsnorm runs the fused residual add + RMSNorm twice: all-bf16 (config 2)
  and the training step's mix (bf16 branch, fp32 residual stream, bf16 normed
  output; the backward also writes the bf16 branch gradient).

Times are CUDA-event means on the launching stream after warm-up; inputs are
regenerated per case and exceed L2 except where noted.  ``--profile`` runs
each selected case ``--iters`` times without timing (for an ncu capture).
"""

from __future__ import annotations

import argparse
import json
import math
from pathlib import Path

import torch

from . import _lib
from .kernels import triton_attention as A
from .kernels import triton_ops as K

ROOT = Path(__file__).resolve().parent.parent


def _peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def _time(fn, iters: int, warm: int = 3) -> float:
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def attention_cases(dev, iters, profile, seqs=(1024, 2048, 4096), batch=16, heads=16, kv_heads=4):
    out = []
    for T in seqs:
        B, Hq, Hkv, D = batch, heads, kv_heads, 64
        g = torch.Generator(device=dev).manual_seed(T)
        q = (torch.randn(B, Hq, T, D, device=dev, generator=g) * 0.5).bfloat16()
        k = (torch.randn(B, Hkv, T, D, device=dev, generator=g) * 0.5).bfloat16()
        v = (torch.randn(B, Hkv, T, D, device=dev, generator=g) * 0.5).bfloat16()
        do = torch.randn(B, Hq, T, D, device=dev, generator=g).bfloat16()
        scale = 1.0 / math.sqrt(D)
        o, lse = A._launch_fwd(q, k, v, Hq // Hkv, scale)
        fwd = lambda: A._launch_fwd(q, k, v, Hq // Hkv, scale)  # noqa: E731
        bwd = lambda: A._launch_bwd(q, k, v, o, lse, do, scale)  # noqa: E731
        if profile:
            for _ in range(iters):
                fwd()
                bwd()
            continue
        flops = 4.0 * B * Hq * D * T * (T + 1) / 2
        ms_f = _time(fwd, iters)
        ms_b = _time(bwd, iters)
        out.append({"op": "attention", "T": T, "B": B, "Hq": Hq, "Hkv": Hkv, "fwd_ms": ms_f, "fwd_tflops": flops / ms_f / 1e9,
                    "bwd_ms": ms_b, "bwd_tflops": 2.5 * flops / ms_b / 1e9,
                    "fwd_bwd_tflops": 3.5 * flops / (ms_f + ms_b) / 1e9})
    return out


def ce_cases(dev, iters, profile, n=65536, h=768, v=21504):
    lib = _lib.load()
    g = torch.Generator(device=dev).manual_seed(5)
    hid = (torch.randn(n, h, device=dev, generator=g) * 0.5).bfloat16()
    w = (torch.randn(v, h, device=dev, generator=g) * 0.02).bfloat16()
    lab = torch.randint(0, v, (n,), device=dev, generator=g)
    loss = torch.empty((), device=dev)
    lse2 = torch.empty(n + 3, device=dev)
    ws = torch.empty(int(lib.mt_fused_ce_workspace_bytes(n, v)), device=dev, dtype=torch.uint8)
    wsb = torch.empty(max(int(lib.mt_fused_ce_bwd_workspace_bytes(n, v, h)), 256), device=dev, dtype=torch.uint8)
    dh = torch.empty(n, h, device=dev, dtype=torch.bfloat16)
    dw = torch.empty(v, h, device=dev, dtype=torch.float32)
    one = torch.ones(1, device=dev)
    status = _lib.status_word(dev)
    stream = _lib.stream_ptr(dev)

    def fwd():
        _lib.check(lib.mt_fused_ce_fwd(hid.data_ptr(), w.data_ptr(), lab.data_ptr(), 1, -100, 2, n, v, h,
                                       loss.data_ptr(), lse2.data_ptr(), ws.data_ptr(), ws.numel(),
                                       status.data_ptr(), stream), "ce fwd")

    def bwd(want_h=True, want_w=True):
        _lib.check(lib.mt_fused_ce_bwd(hid.data_ptr(), w.data_ptr(), lab.data_ptr(), 1, -100, 2, n, v, h,
                                       lse2.data_ptr(), one.data_ptr(), dh.data_ptr() if want_h else None, 2,
                                       dw.data_ptr() if want_w else None, 0, wsb.data_ptr(), wsb.numel(),
                                       status.data_ptr(), stream), "ce bwd")

    fwd()
    if profile:
        for _ in range(iters):
            fwd()
            bwd()
        return []
    flops = 2.0 * n * h * v
    ms_f = _time(fwd, iters)
    ms_b = _time(bwd, iters)
    ms_h = _time(lambda: bwd(True, False), iters)
    ms_w = _time(lambda: bwd(False, True), iters)
    return [{"op": "fused_ce", "N": n, "H": h, "V": v, "fwd_ms": ms_f, "fwd_tflops": flops / ms_f / 1e9,
             "bwd_ms": ms_b, "bwd_tflops": 2 * flops / ms_b / 1e9, "bwd_executed_tflops": 4 * flops / ms_b / 1e9,
             "dh_pass_ms": ms_h, "dh_pass_executed_tflops": 2 * flops / ms_h / 1e9,
             "dw_pass_ms": ms_w, "dw_pass_executed_tflops": 2 * flops / ms_w / 1e9,
             "bwd_global_bytes_min": (n * h * 2) * 2 + v * h * 2 + v * h * 4 + n * 16}]


def _add_rms_case(dev, g, n, H, res_dtype, iters, profile) -> dict | None:
    """Fused residual add + RMSNorm forward and backward at one dtype mix."""
    lib = _lib.load()
    bf = torch.bfloat16
    x = torch.randn(n, H, device=dev, generator=g).to(bf)
    r = torch.randn(n, H, device=dev, generator=g).to(res_dtype)
    # the weight follows the residual stream (fp32 master weight in the training step)
    w = (1 + 0.1 * torch.randn(H, device=dev, generator=g)).to(res_dtype)
    new_res, normed = torch.empty_like(r), torch.empty(n, H, device=dev, dtype=bf)
    rstd = torch.empty(n, device=dev, dtype=torch.float32)
    gres = torch.randn(n, H, device=dev, generator=g).to(res_dtype)
    gn = torch.randn(n, H, device=dev, generator=g).to(bf)
    st = _lib.stream_ptr(dev)

    def f():
        _lib.check(lib.mt_add_rms_norm_fwd(x.data_ptr(), r.data_ptr(), _lib.dtype_code(bf), w.data_ptr(),
                                           _lib.dtype_code(res_dtype), new_res.data_ptr(), _lib.dtype_code(res_dtype),
                                           normed.data_ptr(), _lib.dtype_code(bf), rstd.data_ptr(), n, H, 1e-5, st),
                   "add_rms_norm forward")

    f()
    b = lambda: K._rms_bwd(new_res, w, rstd, gn, res_dtype, residual_grad=gres, branch_dtype=bf)  # noqa: E731
    if profile:
        for _ in range(iters):
            f()
            b()
        return None
    rb, hb = r.element_size(), 2
    # forward: hidden + residual in, new residual + normed out, rstd out
    # backward: new residual, its gradient and the normed gradient in; the residual
    # gradient (and the narrower branch copy when the dtypes differ) out
    byts_f = n * H * (hb + 2 * rb + hb) + 4 * n
    byts_b = n * H * (2 * rb + hb + rb + (hb if rb != hb else 0)) + 4 * n
    mf, mb = _time(f, iters), _time(b, iters)
    return {"op": "add_rms_norm", "N": n, "H": H, "residual": str(res_dtype).replace("torch.", ""), "fwd_ms": mf,
            "fwd_gbs": byts_f / mf / 1e6, "bwd_ms": mb, "bwd_gbs": byts_b / mb / 1e6}


def bandwidth_cases(dev, iters, profile, ops=("rmsnorm", "addrmsnorm", "rope", "swiglu"), n=65536):
    out = []
    g = torch.Generator(device=dev).manual_seed(9)
    if "rmsnorm" in ops:
        H = 768
        x = torch.randn(n, H, device=dev, generator=g).bfloat16()
        w = (1 + 0.1 * torch.randn(H, device=dev, generator=g)).bfloat16()
        dy = torch.randn(n, H, device=dev, generator=g).bfloat16()
        y, rstd = K._rms_fwd(x, w, 1e-5, torch.bfloat16)
        f = lambda: K._rms_fwd(x, w, 1e-5, torch.bfloat16)  # noqa: E731
        b = lambda: K._rms_bwd(x, w, rstd, dy, torch.bfloat16)  # noqa: E731
        if profile:
            for _ in range(iters):
                f()
                b()
        else:
            bf, bb = 2 * n * H * 2 + 4 * n, 3 * n * H * 2 + 4 * n
            mf, mb = _time(f, iters), _time(b, iters)
            out.append({"op": "rms_norm", "N": n, "H": H, "fwd_ms": mf, "fwd_gbs": bf / mf / 1e6, "bwd_ms": mb,
                        "bwd_gbs": bb / mb / 1e6})
    if "addrmsnorm" in ops:
        for res_dtype in (torch.bfloat16, torch.float32):
            r = _add_rms_case(dev, g, n, 768, res_dtype, iters, profile)
            if r is not None:
                out.append(r)
    if "rope" in ops:
        B, T, D = n // 2048, 2048, 64
        q = torch.randn(B, T, 12, D, device=dev, generator=g).bfloat16().transpose(1, 2)
        k = torch.randn(B, T, 4, D, device=dev, generator=g).bfloat16().transpose(1, 2)
        pos = torch.arange(T, device=dev, dtype=torch.float32)
        inv = 1.0 / (500000.0 ** (torch.arange(0, D, 2, device=dev, dtype=torch.float32) / D))
        fr = torch.outer(pos, inv)
        cos, sin = fr.cos().bfloat16(), fr.sin().bfloat16()
        qo, ko = torch.empty_like(q), torch.empty_like(k)
        f = lambda: K._launch_rope(q, k, cos, sin, qo, ko, negate=False)  # noqa: E731
        if profile:
            for _ in range(iters):
                f()
        else:
            byts = 2 * n * 16 * D * 2
            m = _time(f, iters)
            out.append({"op": "rope", "N": n, "heads": "12+4", "D": D, "ms": m, "gbs": byts / m / 1e6})
    if "swiglu" in ops:
        I = 2048
        gt = torch.randn(n, I, device=dev, generator=g).bfloat16()
        up = torch.randn(n, I, device=dev, generator=g).bfloat16()
        dy = torch.randn(n, I, device=dev, generator=g).bfloat16()
        lib = _lib.load()
        y, dg, du = torch.empty_like(gt), torch.empty_like(gt), torch.empty_like(gt)
        st = _lib.stream_ptr(dev)
        f = lambda: lib.mt_swiglu_fwd(gt.data_ptr(), up.data_ptr(), y.data_ptr(), 2, gt.numel(), st)  # noqa: E731
        b = lambda: lib.mt_swiglu_bwd(gt.data_ptr(), up.data_ptr(), dy.data_ptr(), dg.data_ptr(),  # noqa: E731
                                      du.data_ptr(), 2, gt.numel(), st)
        if profile:
            for _ in range(iters):
                f()
                b()
        else:
            mf, mb = _time(f, iters), _time(b, iters)
            out.append({"op": "swiglu", "N": n, "I": I, "fwd_ms": mf, "fwd_gbs": 3 * n * I * 2 / mf / 1e6,
                        "bwd_ms": mb, "bwd_gbs": 5 * n * I * 2 / mb / 1e6})
        gu = torch.cat([gt, up], dim=1)
        dgu = torch.empty_like(gu)
        f = lambda: lib.mt_swiglu_packed_fwd(gu.data_ptr(), y.data_ptr(), 2, n, I, st)  # noqa: E731
        b = lambda: lib.mt_swiglu_packed_bwd(gu.data_ptr(), dy.data_ptr(), dgu.data_ptr(), 2, n, I, st)  # noqa: E731
        if profile:
            for _ in range(iters):
                f()
                b()
        else:
            mf, mb = _time(f, iters), _time(b, iters)
            out.append({"op": "swiglu_packed", "N": n, "I": I, "fwd_ms": mf, "fwd_gbs": 3 * n * I * 2 / mf / 1e6,
                        "bwd_ms": mb, "bwd_gbs": 5 * n * I * 2 / mb / 1e6})
    return out


def adamw_cases(dev, iters, profile, model: str = "gqa12"):
    """The fused AdamW over every parameter of a BASELINE model (config 3: 92 M fp32 parameters),
    writing the bf16 GEMM-operand copies; 30 bytes per parameter (p, g, m, v read; p, m, v
    written; 2-byte copy)."""
    from .model import CONFIGS, TradingModelB200
    from .optim import AdamWShadow

    torch.manual_seed(0)
    m = TradingModelB200(CONFIGS[model]).to(dev)
    opt = AdamWShadow(m.parameters(), lr=1e-4, weight_decay=0.01, packed=m.packed_weights())
    for p in m.parameters():
        p.grad = torch.randn_like(p) * 1e-3
    numel = sum(p.numel() for p in m.parameters())
    step = lambda: opt.step()  # noqa: E731
    if profile:
        for _ in range(iters):
            step()
        return []
    ms = _time(step, iters)
    return [{"op": "adamw", "model": model, "params": numel, "ms": ms, "gbs": 30.0 * numel / ms / 1e6}]


def mlp_cases(dev, iters, profile, n=65536, h=768, inter=2048):
    """SwiGLU MLP: the fused tcgen05 GEMMs against cuBLAS + the standalone packed gate."""
    import torch.nn.functional as F

    from .kernels.fused_blocks import interleave_gate_up

    lib = _lib.load()
    g = torch.Generator(device=dev).manual_seed(11)
    x = torch.randn(n, h, device=dev, generator=g).bfloat16()
    w1 = torch.randn(inter, h, device=dev, generator=g) * 0.05
    w3 = torch.randn(inter, h, device=dev, generator=g) * 0.05
    w13 = interleave_gate_up(w1, w3).bfloat16().contiguous()
    w13c = torch.cat([w1, w3]).bfloat16()
    w2t = (torch.randn(inter, h, device=dev, generator=g) * 0.05).bfloat16()
    dout = torch.randn(n, h, device=dev, generator=g).bfloat16()
    gu = torch.empty(n, 2 * inter, device=dev, dtype=torch.bfloat16)
    y = torch.empty(n, inter, device=dev, dtype=torch.bfloat16)
    dgu = torch.empty_like(gu)
    status = _lib.status_word(dev)
    st = _lib.stream_ptr(dev)
    fwd = lambda: lib.mt_swiglu_gemm_fwd(x.data_ptr(), w13.data_ptr(), gu.data_ptr(), y.data_ptr(), 2, n, h,  # noqa: E731
                                         inter, status.data_ptr(), st)
    bwd = lambda: lib.mt_swiglu_gemm_bwd(dout.data_ptr(), w2t.data_ptr(), gu.data_ptr(), dgu.data_ptr(), 2, n,  # noqa: E731
                                         h, inter, status.data_ptr(), st)

    def unfused_fwd():
        guc = F.linear(x, w13c)
        lib.mt_swiglu_packed_fwd(guc.data_ptr(), y.data_ptr(), 2, n, inter, st)

    def unfused_bwd():
        dy = dout.mm(w2t.t())
        lib.mt_swiglu_packed_bwd(gu.data_ptr(), dy.data_ptr(), dgu.data_ptr(), 2, n, inter, st)

    if profile:
        for _ in range(iters):
            fwd()
            bwd()
        return []
    ff, fb = 2.0 * n * h * 2 * inter, 2.0 * n * h * inter
    mf, mb, uf, ub = _time(fwd, iters), _time(bwd, iters), _time(unfused_fwd, iters), _time(unfused_bwd, iters)
    return [{"op": "swiglu_gemm", "N": n, "H": h, "I": inter, "fwd_ms": mf, "fwd_tflops": ff / mf / 1e9,
             "bwd_ms": mb, "bwd_tflops": fb / mb / 1e9, "unfused_fwd_ms": uf, "unfused_bwd_ms": ub}]


def qkv_cases(dev, iters, profile, n=65536, h=768, hq=12, hkv=4, d=64, seq=2048):
    """QKV projection with RoPE in the tcgen05 epilogue against cuBLAS + the RoPE kernel."""
    import torch.nn.functional as F

    from .kernels import triton_ops as K

    lib = _lib.load()
    g = torch.Generator(device=dev).manual_seed(13)
    cols = (hq + 2 * hkv) * d
    x = torch.randn(n, h, device=dev, generator=g).bfloat16()
    w = (torch.randn(cols, h, device=dev, generator=g) * 0.04).bfloat16()
    pos = torch.arange(seq, device=dev, dtype=torch.float32)
    inv = 1.0 / (500000.0 ** (torch.arange(0, d, 2, device=dev, dtype=torch.float32) / d))
    fr = torch.outer(pos, inv)
    cos2, sin2 = fr.cos().bfloat16().contiguous(), fr.sin().bfloat16().contiguous()
    qkv = torch.empty(n, cols, device=dev, dtype=torch.bfloat16)
    status = _lib.status_word(dev)
    st = _lib.stream_ptr(dev)
    fused = lambda: lib.mt_qkv_rope_gemm(x.data_ptr(), w.data_ptr(), qkv.data_ptr(), cos2.data_ptr(),  # noqa: E731
                                         sin2.data_ptr(), d // 2, 2, n, h, cols, (hq + hkv) * d, seq, d,
                                         status.data_ptr(), st)
    B = n // seq

    def unfused():
        y = F.linear(x, w).view(B, seq, cols)
        q = y[..., : hq * d].view(B, seq, hq, d).transpose(1, 2)
        k = y[..., hq * d:(hq + hkv) * d].view(B, seq, hkv, d).transpose(1, 2)
        K._launch_rope(q, k, cos2, sin2, torch.empty_like(q), torch.empty_like(k), negate=False)

    if profile:
        for _ in range(iters):
            fused()
        return []
    fl = 2.0 * n * h * cols
    mf, mu = _time(fused, iters), _time(unfused, iters)
    return [{"op": "qkv_rope_gemm", "N": n, "H": h, "cols": cols, "ms": mf, "tflops": fl / mf / 1e9,
             "unfused_ms": mu}]


REF_DIR = Path(__file__).resolve().parent.parent / "baseline" / "_ref"


def load_reference(ref_dir: Path = REF_DIR):
    """Import duoan/mega-trading's own operator modules from an installed copy
    (``pip install --target baseline/_ref``) through a stub package: the real
    ``mega_trading/__init__.py`` imports the trainer, which needs ``accelerate``.
    Returns ``(triton_attention module, triton_ops module, model module)`` or None."""
    import sys
    import types

    src = ref_dir / "mega_trading"
    if not (src / "kernels" / "triton_ops.py").exists():
        return None
    if "mega_trading" not in sys.modules:
        pkg = types.ModuleType("mega_trading")
        pkg.__path__ = [str(src)]
        sys.modules["mega_trading"] = pkg
    import importlib

    return (importlib.import_module("mega_trading.kernels.triton_attention"),
            importlib.import_module("mega_trading.kernels.triton_ops"),
            importlib.import_module("mega_trading.model"))


def reference_cases(dev, iters, seqs=(1024, 2048, 4096), n=65536):
    """The reference's own GPU kernels (Triton, JIT-compiled for this GPU) on the same inputs and
    harness as ours: config-1 attention forward / backward, config-2 RMSNorm, add+RMSNorm, RoPE,
    SwiGLU gate and fused linear + CE.  Where the reference falls back to torch (its backward
    outside T=512 materialises fp32 T x T tensors) that is what gets timed; an out-of-memory is
    recorded as such."""
    ref = load_reference()
    if ref is None:
        return [{"op": "reference", "unavailable": f"no installed reference under {REF_DIR}"}]
    RA, RO, _ = ref
    out = []

    def timed(name, fn, **meta):
        try:
            ms = _time(fn, iters)
            out.append({"op": name, "ms": ms, **meta})
            return ms
        except torch.OutOfMemoryError as exc:
            out.append({"op": name, "oom": str(exc).splitlines()[0][:160], **meta})
            torch.cuda.empty_cache()
            return None

    for T in seqs:
        B, Hq, Hkv, D = 16, 16, 4, 64
        g = torch.Generator(device=dev).manual_seed(T)
        q = (torch.randn(B, Hq, T, D, device=dev, generator=g) * 0.5).bfloat16().requires_grad_(True)
        k = (torch.randn(B, Hkv, T, D, device=dev, generator=g) * 0.5).bfloat16().requires_grad_(True)
        v = (torch.randn(B, Hkv, T, D, device=dev, generator=g) * 0.5).bfloat16().requires_grad_(True)
        do = torch.randn(B, Hq, T, D, device=dev, generator=g).bfloat16()
        flops = 4.0 * B * Hq * D * T * (T + 1) / 2
        mf = timed("ref_attention_fwd", lambda: RA.triton_attention(q, k, v, repeats=Hq // Hkv), T=T)
        if mf:
            out[-1]["tflops"] = flops / mf / 1e9
        try:
            o = RA.triton_attention(q, k, v, repeats=Hq // Hkv)
            mb = timed("ref_attention_bwd", lambda: torch.autograd.grad(o, (q, k, v), do, retain_graph=True), T=T)
            if mb:
                out[-1]["tflops"] = 2.5 * flops / mb / 1e9
            del o
        except torch.OutOfMemoryError as exc:
            out.append({"op": "ref_attention_bwd", "T": T, "oom": str(exc).splitlines()[0][:160]})
        del q, k, v, do
        torch.cuda.empty_cache()
    # the one shape the reference runs a Triton attention backward on
    # (kernels/triton_attention.py:114-131: T=512, Hq 16 / Hkv 4, D 64, bf16), ours beside it
    B, Hq, Hkv, D, T = 64, 16, 4, 64, 512
    g = torch.Generator(device=dev).manual_seed(512)
    q = (torch.randn(B, Hq, T, D, device=dev, generator=g) * 0.5).bfloat16().requires_grad_(True)
    k = (torch.randn(B, Hkv, T, D, device=dev, generator=g) * 0.5).bfloat16().requires_grad_(True)
    v = (torch.randn(B, Hkv, T, D, device=dev, generator=g) * 0.5).bfloat16().requires_grad_(True)
    do = torch.randn(B, Hq, T, D, device=dev, generator=g).bfloat16()
    flops = 4.0 * B * Hq * D * T * (T + 1) / 2
    mf = timed("ref_attention_fwd", lambda: RA.triton_attention(q, k, v, repeats=Hq // Hkv), T=T, B=B)
    if mf:
        out[-1]["tflops"] = flops / mf / 1e9
    o = RA.triton_attention(q, k, v, repeats=Hq // Hkv)
    mb = timed("ref_attention_bwd", lambda: torch.autograd.grad(o, (q, k, v), do, retain_graph=True), T=T, B=B)
    if mb:
        out[-1]["tflops"] = 2.5 * flops / mb / 1e9
    del o
    qd, kd, vd = q.detach(), k.detach(), v.detach()
    scale = 1.0 / math.sqrt(D)
    o, lse = A._launch_fwd(qd, kd, vd, Hq // Hkv, scale)
    mf = timed("attention_fwd", lambda: A._launch_fwd(qd, kd, vd, Hq // Hkv, scale), T=T, B=B)
    if mf:
        out[-1]["tflops"] = flops / mf / 1e9
    mb = timed("attention_bwd", lambda: A._launch_bwd(qd, kd, vd, o, lse, do, scale), T=T, B=B)
    if mb:
        out[-1]["tflops"] = 2.5 * flops / mb / 1e9
    del q, k, v, do, o, lse, qd, kd, vd
    torch.cuda.empty_cache()
    g = torch.Generator(device=dev).manual_seed(9)
    H, I, V = 768, 2048, 21504
    bf = torch.bfloat16
    x = torch.randn(n, H, device=dev, generator=g).to(bf)
    r = torch.randn(n, H, device=dev, generator=g).to(bf)
    w = (1 + 0.1 * torch.randn(H, device=dev, generator=g)).to(bf)
    ms = timed("ref_rms_norm_fwd", lambda: RO.triton_rms_norm(x, w, eps=1e-5), N=n)
    if ms:
        out[-1]["gbs"] = (2 * n * H * 2 + 4 * n) / ms / 1e6
    ms = timed("ref_add_rms_norm_fwd", lambda: RO.triton_add_rms_norm(x, r, w, eps=1e-5), N=n)
    if ms:
        out[-1]["gbs"] = 4 * n * H * 2 / ms / 1e6
    del x, r
    gt = torch.randn(n, I, device=dev, generator=g).to(bf)
    up = torch.randn(n, I, device=dev, generator=g).to(bf)
    ms = timed("ref_swiglu_fwd", lambda: RO.triton_swiglu_gate(gt, up), N=n)
    if ms:
        out[-1]["gbs"] = 3 * n * I * 2 / ms / 1e6
    del gt, up
    Bt, T, D = n // 2048, 2048, 64
    qr = torch.randn(Bt, 12, T, D, device=dev, generator=g).to(bf)
    kr = torch.randn(Bt, 4, T, D, device=dev, generator=g).to(bf)
    fr = torch.outer(torch.arange(T, device=dev, dtype=torch.float32),
                     1.0 / (500000.0 ** (torch.arange(0, D, 2, device=dev, dtype=torch.float32) / D)))
    c, sn = fr.cos().to(bf)[None, None], fr.sin().to(bf)[None, None]
    ms = timed("ref_rope", lambda: RO.triton_apply_rope(qr, kr, c, sn), N=n)
    if ms:
        out[-1]["gbs"] = 2 * n * 16 * D * 2 / ms / 1e6
    del qr, kr
    hid = (torch.randn(n, H, device=dev, generator=g) * 0.5).to(bf).requires_grad_(True)
    wv = (torch.randn(V, H, device=dev, generator=g) * 0.02).to(bf).requires_grad_(True)
    lab = torch.randint(0, V, (n,), device=dev, generator=g)
    ms = timed("ref_fused_ce_fwd_bwd", lambda: RO.triton_fused_linear_cross_entropy(hid, wv, lab).backward(), N=n)
    if ms:
        out[-1]["tflops"] = 6.0 * n * H * V / ms / 1e9
    return out


def torch_comparators(dev, iters, seqs=(1024, 2048, 4096), n=65536):
    """The BASELINE torch comparators on the same box: SDPA (flash / cuDNN backends) for causal
    GQA attention at config 1, F.rms_norm, eager RoPE, F.silu * up and F.linear + F.cross_entropy
    at config 2 (library kernels, timed like ours)."""
    import torch.nn.functional as F

    out = []
    for T in seqs:
        B, Hq, Hkv, D = 16, 16, 4, 64
        g = torch.Generator(device=dev).manual_seed(T)
        q = (torch.randn(B, Hq, T, D, device=dev, generator=g) * 0.5).bfloat16().requires_grad_(True)
        k = (torch.randn(B, Hkv, T, D, device=dev, generator=g) * 0.5).bfloat16().requires_grad_(True)
        v = (torch.randn(B, Hkv, T, D, device=dev, generator=g) * 0.5).bfloat16().requires_grad_(True)
        do = torch.randn(B, Hq, T, D, device=dev, generator=g).bfloat16()
        fwd = lambda: F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)  # noqa: E731
        o = fwd()
        bwd = lambda: torch.autograd.grad(o, (q, k, v), do, retain_graph=True)  # noqa: E731
        flops = 4.0 * B * Hq * D * T * (T + 1) / 2
        mf, mb = _time(fwd, iters), _time(bwd, iters)
        out.append({"op": "torch_sdpa", "T": T, "B": B, "fwd_ms": mf, "fwd_tflops": flops / mf / 1e9, "bwd_ms": mb,
                    "bwd_tflops": 2.5 * flops / mb / 1e9, "fwd_bwd_tflops": 3.5 * flops / (mf + mb) / 1e9})
        del q, k, v, do, o
    g = torch.Generator(device=dev).manual_seed(9)
    H, I, V = 768, 2048, 21504
    x = torch.randn(n, H, device=dev, generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(H, device=dev, generator=g)).bfloat16()
    mf = _time(lambda: F.rms_norm(x, (H,), w, eps=1e-5), iters)
    out.append({"op": "torch_rms_norm", "N": n, "H": H, "fwd_ms": mf, "fwd_gbs": (2 * n * H * 2 + 4 * n) / mf / 1e6})
    gt = torch.randn(n, I, device=dev, generator=g).bfloat16()
    up = torch.randn(n, I, device=dev, generator=g).bfloat16()
    mf = _time(lambda: F.silu(gt) * up, iters)
    out.append({"op": "torch_swiglu", "N": n, "I": I, "fwd_ms": mf, "fwd_gbs": 3 * n * I * 2 / mf / 1e6})
    del gt, up
    Bt, T, D = n // 2048, 2048, 64
    qr = torch.randn(Bt, 12, T, D, device=dev, generator=g).bfloat16()
    kr = torch.randn(Bt, 4, T, D, device=dev, generator=g).bfloat16()
    fr = torch.outer(torch.arange(T, device=dev, dtype=torch.float32),
                     1.0 / (500000.0 ** (torch.arange(0, D, 2, device=dev, dtype=torch.float32) / D)))
    c, sn = fr.cos().bfloat16(), fr.sin().bfloat16()

    def rot(t):
        e, o2 = t[..., 0::2], t[..., 1::2]
        return torch.stack((e * c - o2 * sn, e * sn + o2 * c), dim=-1).flatten(-2)

    mf = _time(lambda: (rot(qr), rot(kr)), iters)
    out.append({"op": "torch_rope", "N": n, "ms": mf, "gbs": 2 * n * 16 * D * 2 / mf / 1e6})
    del qr, kr
    hid = (torch.randn(n, H, device=dev, generator=g) * 0.5).bfloat16()
    wv = (torch.randn(V, H, device=dev, generator=g) * 0.02).bfloat16()
    lab = torch.randint(0, V, (n,), device=dev, generator=g)
    ce = lambda: F.cross_entropy(F.linear(hid, wv).float(), lab)  # noqa: E731
    mf = _time(ce, max(2, iters // 2))
    out.append({"op": "torch_linear_ce", "N": n, "H": H, "V": V, "fwd_ms": mf,
                "fwd_tflops": 2.0 * n * H * V / mf / 1e9})
    return out


def run(ops: list[str], iters: int = 10, profile: bool = False, device: int = 0, attn_seqs=(1024, 2048, 4096),
        attn_batch: int = 16, ce_rows: int = 65536, heads: int = 16, kv_heads: int = 4) -> list[dict]:
    dev = torch.device("cuda", device)
    torch.cuda.set_device(dev)
    res: list[dict] = []
    if "attention" in ops:
        res += attention_cases(dev, iters, profile, attn_seqs, attn_batch, heads, kv_heads)
    if "ce" in ops:
        res += ce_cases(dev, iters, profile, n=ce_rows)
    if "mlp" in ops:
        res += mlp_cases(dev, iters, profile, n=ce_rows)
    if "qkv" in ops:
        res += qkv_cases(dev, iters, profile, n=ce_rows)
    if "torch" in ops and not profile:
        res += torch_comparators(dev, iters, attn_seqs)
    if "ref" in ops and not profile:
        res += reference_cases(dev, iters, attn_seqs)
    if "adamw" in ops:
        res += adamw_cases(dev, iters, profile)
    bw = [o for o in ops if o in ("rmsnorm", "addrmsnorm", "rope", "swiglu")]
    if bw:
        res += bandwidth_cases(dev, iters, profile, tuple(bw))
    torch.cuda.synchronize()
    status = _lib.read_status(dev)
    if status:
        raise RuntimeError(f"device status word {status:#x}")
    peaks = _peaks()
    for r in res:
        for key in list(r):
            if key.endswith("tflops"):
                r[key.replace("tflops", "frac")] = r[key] / peaks["bf16_tflops"]
            if key.endswith("gbs"):
                r[key.replace("gbs", "frac")] = r[key] / peaks["hbm_gbs"]
    return res


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--ops", default="attention,ce,rmsnorm,addrmsnorm,rope,swiglu")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--profile", action="store_true")
    ap.add_argument("--seqs", default="1024,2048,4096")
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--ce-rows", type=int, default=65536)
    ap.add_argument("--heads", type=int, default=16)
    ap.add_argument("--kv-heads", type=int, default=4)
    args = ap.parse_args(argv)
    res = run(args.ops.split(","), args.iters, args.profile, attn_seqs=tuple(int(s) for s in args.seqs.split(",")),
              attn_batch=args.batch, ce_rows=args.ce_rows, heads=args.heads, kv_heads=args.kv_heads)
    for r in res:
        print(json.dumps(r))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
