"""Host-side logic that needs no GPU: operator validation and error behaviour,
the synthetic token stream, FLOP accounting, the bench contract helpers."""

from __future__ import annotations

import math

import pytest
import torch


def test_ops_refuse_cpu_tensors_instead_of_falling_back():
    from mega_trading_b200.kernels import triton_attention as A
    from mega_trading_b200.kernels import triton_ops as K

    x = torch.randn(2, 8)
    with pytest.raises(RuntimeError, match="CUDA"):
        K.triton_rms_norm(x, torch.ones(8), eps=1e-5)
    with pytest.raises(RuntimeError, match="CUDA"):
        K.triton_swiglu_gate(x, x)
    with pytest.raises(RuntimeError, match="CUDA"):
        K.triton_add_rms_norm(x, x, torch.ones(8), eps=1e-5)
    q = torch.randn(1, 4, 8, 32)
    with pytest.raises(RuntimeError, match="requires CUDA tensors"):
        A.triton_attention(q, q[:, :2], q[:, :2], repeats=2)
    with pytest.raises(RuntimeError, match="CUDA"):
        K.triton_apply_rope(q, q, torch.ones(8, 16), torch.ones(8, 16))


def test_validation_messages_match_reference():
    from mega_trading_b200.kernels import triton_ops as K

    h = torch.randn(4, 8)
    w = torch.randn(11, 8)
    lab = torch.zeros(4, dtype=torch.long)
    with pytest.raises(ValueError, match="hidden must have shape"):
        K.triton_fused_linear_cross_entropy(h[None], w, lab)
    with pytest.raises(ValueError, match="weight must have shape"):
        K.triton_fused_linear_cross_entropy(h, w[:, :4], lab)
    with pytest.raises(ValueError, match="labels must be a 1D tensor"):
        K.triton_fused_linear_cross_entropy(h, w, lab[None])
    with pytest.raises(ValueError, match="labels must be an integer tensor"):
        K.triton_fused_linear_cross_entropy(h, w, lab.float())


def test_composite_tokens_distribution():
    from mega_trading_b200.data import VOCAB_SIZE, _ZIPF, composite_tokens, next_token_batch

    t = composite_tokens(64, 512, seed=1)
    assert t.dtype == torch.int64 and t.min() >= 0 and t.max() < VOCAB_SIZE == 21504
    dt = t % 16
    vol = (t // 16) % 16
    depth = (t // 256) % 21
    side = (t // (256 * 21)) % 2
    action = t // (256 * 21 * 2)
    assert action.max() <= 1
    for field in (dt, vol):
        freq = torch.bincount(field.flatten(), minlength=16).double() / field.numel()
        assert torch.allclose(freq, _ZIPF, atol=6e-3)
    # geometric(p=0.3) - 1: P(0) = 0.3
    assert abs(float((depth == 0).double().mean()) - 0.3) < 6e-3
    assert abs(float(side.double().mean()) - 0.5) < 6e-3
    ids, labels = next_token_batch(2, 16, seed=9)
    full = composite_tokens(2, 17, seed=9)
    assert torch.equal(ids, full[:, :-1]) and torch.equal(labels, full[:, 1:])
    assert torch.equal(composite_tokens(3, 5, seed=4), composite_tokens(3, 5, seed=4))


def test_flop_accounting_per_token_and_step():
    from mega_trading_b200.model import CONFIGS

    cfg = CONFIGS["gqa12"]
    assert cfg.matmul_params() == 92_012_544
    per_tok = cfg.train_flops_per_token(2048)
    assert math.isclose(per_tok, 684.3e6, rel_tol=2e-3)
    assert math.isclose(per_tok * 256 * 2048, 358.8e12, rel_tol=2e-3)
    big = CONFIGS["large24"]
    assert math.isclose(big.train_flops_per_token(4096), 2.460e9, rel_tol=2e-3)


def test_clock_sampler_summary_parses_nvidia_smi_rows(tmp_path):
    import bench

    s = bench.ClockSampler(0)
    s.path = tmp_path / "c.csv"
    s.path.write_text("0, 1965, 1965, 700.5, 0x0, Not Active, Not Active, Not Active, Not Active\n"
                      "0, 1800, 1965, 990.1, 0x4, Not Active, Not Active, Not Active, Active\n")
    out = s.summary()
    assert out["sm_max_mhz"] == 1965.0 and out["reasons"] == ["sw_power_cap"] and out["samples"] == 2


def test_clock_sampler_counts_only_samples_after_the_mark(tmp_path):
    import bench

    s = bench.ClockSampler(0)
    s.path = tmp_path / "c.csv"
    s.path.write_text("0, 1965, 1965, 100.0, 0x0, Not Active, Not Active, Not Active, Not Active\n")
    s.mark()  # timing starts: the idle sample above is not part of the region
    with s.path.open("a") as f:
        f.write("0, 1500, 1965, 998.0, 0x4, Not Active, Not Active, Not Active, Active\n")
    out = s.summary()
    assert out["samples"] == 1 and out["sm_mhz"] == 1500.0 and out["reasons"] == ["sw_power_cap"]


def test_gate_up_interleave_layout():
    """The fused SwiGLU weight alternates 128-row blocks of w1 and w3, and
    its gradient routes back to the right rows of each."""
    from mega_trading_b200.kernels.fused_blocks import interleave_gate_up, swiglu_mlp_supported

    w1 = torch.arange(512 * 4, dtype=torch.float32).view(512, 4).requires_grad_(True)
    w3 = (-torch.arange(512 * 4, dtype=torch.float32)).view(512, 4).requires_grad_(True)
    w13 = interleave_gate_up(w1, w3)
    assert w13.shape == (1024, 4)
    for b in range(4):
        assert torch.equal(w13[256 * b:256 * b + 128], w1[128 * b:128 * (b + 1)])
        assert torch.equal(w13[256 * b + 128:256 * (b + 1)], w3[128 * b:128 * (b + 1)])
    g = torch.randn_like(w13)
    w13.backward(g)
    for b in range(4):
        assert torch.equal(w1.grad[128 * b:128 * (b + 1)], g[256 * b:256 * b + 128])
        assert torch.equal(w3.grad[128 * b:128 * (b + 1)], g[256 * b + 128:256 * (b + 1)])
    assert swiglu_mlp_supported(2048, 768) and swiglu_mlp_supported(2816, 1024)
    assert not swiglu_mlp_supported(688, 256)


def test_fused_projection_paths_follow_the_shapes():
    from mega_trading_b200.kernels.fused_blocks import qkv_rope_gemm_supported

    assert qkv_rope_gemm_supported(12, 4, 64, 768)      # config 3: 1280 columns
    assert qkv_rope_gemm_supported(16, 4, 64, 1024)     # config 4: 1536 columns
    assert not qkv_rope_gemm_supported(8, 2, 32, 256)   # config 0: 384 columns -> cuBLAS + RoPE kernel
    assert not qkv_rope_gemm_supported(4, 2, 48, 256)   # head_dim 48


def test_packed_weight_copies_follow_the_gemm_layouts():
    """The element map the fused optimizer writes through (block / stride / start per
    parameter) reproduces the packed layouts, and the packed copy's gradient reaches
    each fp32 parameter unchanged."""
    from mega_trading_b200.kernels.fused_blocks import GATE_BLOCK, interleave_gate_up
    from mega_trading_b200.optim import PackedWeights

    torch.manual_seed(0)
    w1 = torch.nn.Parameter(torch.randn(2 * GATE_BLOCK, 48))
    w3 = torch.nn.Parameter(torch.randn(2 * GATE_BLOCK, 48))
    q = torch.nn.Parameter(torch.randn(96, 48))
    k = torch.nn.Parameter(torch.randn(32, 48))
    v = torch.nn.Parameter(torch.randn(32, 48))
    cases = [(PackedWeights([w1, w3], "interleave", GATE_BLOCK), interleave_gate_up(w1, w3)),
             (PackedWeights([q, k, v], "rows"), torch.cat([q, k, v])),
             (PackedWeights([q]), q)]
    for pw, ref in cases:
        packed = pw.pack()
        assert packed.dtype == torch.bfloat16 and torch.equal(packed, ref.detach().to(torch.bfloat16))
        flat = packed.reshape(-1)
        for part in pw.parts():
            src = part.param.detach().reshape(-1).to(torch.bfloat16)
            j = torch.arange(src.numel())
            assert torch.equal(flat[part.start + (j // part.block) * part.stride + j % part.block], src)
        g = torch.randn(packed.shape).to(torch.bfloat16)
        for p in pw.params:
            p.grad = None
        pw.get().backward(g)
        ref_params = [p.detach().clone().requires_grad_() for p in pw.params]
        if pw.kind == "interleave":
            interleave_gate_up(*ref_params).to(torch.bfloat16).backward(g)
        elif len(ref_params) > 1:
            torch.cat(ref_params).to(torch.bfloat16).backward(g)
        else:
            ref_params[0].to(torch.bfloat16).backward(g)
        for p, r in zip(pw.params, ref_params):
            assert p.grad.dtype == torch.float32 and torch.equal(p.grad, r.grad)


def test_packed_weight_copy_is_rebuilt_unless_the_fused_optimizer_owns_it():
    import gc

    from mega_trading_b200.optim import AdamWShadow, PackedWeights

    w = torch.nn.Parameter(torch.zeros(4, 8))
    pw = PackedWeights([w])
    assert torch.equal(pw.get(), torch.zeros(4, 8, dtype=torch.bfloat16))
    # torch's fused AdamW moves weights without advancing version counters: an
    # unowned copy is rebuilt in every forward
    w.grad = torch.ones(4, 8)
    torch.optim.AdamW([w], lr=0.5, fused=True).step()
    assert w._version == 0 and torch.equal(pw.get(), w.detach().to(torch.bfloat16))
    # owned: reused until a version counter moves
    opt = AdamWShadow([w], lr=1e-3, packed=[pw])
    assert pw.owned and not pw._stale()
    with torch.no_grad():
        w.fill_(1.5)  # e.g. load_state_dict
    assert pw._stale() and torch.equal(pw.get(), torch.full((4, 8), 1.5, dtype=torch.bfloat16))
    del opt
    gc.collect()
    assert not pw.owned and pw._stale()
    with pytest.raises(ValueError, match="stepped by this optimizer"):
        AdamWShadow([torch.nn.Parameter(torch.zeros(2))], packed=[pw])


def test_fused_adamw_refuses_cpu_parameters():
    from mega_trading_b200.optim import AdamWShadow

    w = torch.nn.Parameter(torch.zeros(4))
    w.grad = torch.ones(4)
    opt = AdamWShadow([w], lr=1e-3)
    with pytest.raises(RuntimeError, match="fp32 CUDA"):
        opt.step()
    with pytest.raises(ValueError):
        AdamWShadow([w], lr=-1.0)


def test_copied_packed_weights_are_not_owned():
    import copy

    from mega_trading_b200.optim import AdamWShadow, PackedWeights

    lin = torch.nn.Linear(8, 4, bias=False)
    pw = PackedWeights([lin.weight])
    lin.__dict__["_w_bf16"] = pw
    opt = AdamWShadow(lin.parameters(), packed=[pw])
    pw.get()
    clone = copy.deepcopy(lin)
    cpw = clone.__dict__["_w_bf16"]
    assert pw.owned and not cpw.owned and cpw.tensor is None
    assert cpw.params[0] is clone.weight  # the copy follows the copied parameter
    assert torch.equal(cpw.get(), clone.weight.detach().to(torch.bfloat16))
    del opt


def test_bench_workloads_match_the_model_configs():
    """Both bench workloads are BASELINE configs 3 and 4, and the CPU reference arm builds
    the oracle model with the same fields as the product's."""
    import bench

    from mega_trading_b200.model import CONFIGS

    assert set(bench.WORKLOADS) == {"gqa12", "large24"}
    w3, w4 = bench.WORKLOADS["gqa12"], bench.WORKLOADS["large24"]
    assert (w3["global_batch"], w3["seq"]) == (256, 2048) and (w4["global_batch"], w4["seq"]) == (128, 4096)
    for name in bench.WORKLOADS:
        ref = bench._ref_config(name)
        cfg = CONFIGS[name]
        for field in ("vocab_size", "hidden_dim", "layers", "attention_heads", "kv_heads", "intermediate_dim",
                      "rope_theta", "norm_eps", "block_size"):
            assert getattr(ref, field) == getattr(cfg, field), (name, field)
        assert cfg.block_size >= bench.WORKLOADS[name]["seq"]


def test_bench_reference_arm_prints_the_contract_line(capsys, monkeypatch):
    """``bench.py --impl reference`` on the host: one JSON line with the contract keys, the
    reference arm's e2e without host-device copies, and a cpu_baseline naming what ran; a
    non-zero rank prints nothing (only rank 0 runs the arm under torchrun)."""
    import json

    import bench

    monkeypatch.setenv("RANK", "1")
    assert bench.main(["--impl", "reference", "--steps", "1", "--warmup", "0"]) == 0
    assert capsys.readouterr().out == ""
    monkeypatch.setenv("RANK", "0")
    assert bench.main(["--impl", "reference", "--steps", "1", "--warmup", "0"]) == 0
    lines = [ln for ln in capsys.readouterr().out.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["unit"] == "tokens/s" and d["value"] > 0
    assert d["metric"] == bench.WORKLOADS["gqa12"]["metric"]
    assert d["cpu_baseline"]["kind"] in ("reference", "port") and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["e2e"]["value"] == d["value"]
