"""Benchmark: data-parallel training throughput of the B200 hot path.

``python bench.py --gpus N --steps K --warmup W`` (torchrun for N > 1) times K
full training steps of BASELINE config 3 -- 12 layers, d_model 768, 12/4 GQA
heads, head_dim 64, SwiGLU 2048, vocab 21,504, seq 2048, global batch 256
sequences split over the N ranks (strong scaling), bf16 GEMMs with fp32
master weights and fused AdamW -- on seeded synthetic composite-token streams
already resident in HBM.  ``--model large24`` runs BASELINE config 4 instead
(24 layers, d_model 1024, 16/4 GQA heads, SwiGLU 2816, seq 4096, global batch
128).  One JSON line on rank 0 (see the contract fields below).
``--impl reference`` times the reference's own PyTorch train step on the host
cores instead: its ``TradingModel`` from the copy installed under
``baseline/_ref`` when present, else the CPU fp32 restatement in ``oracle/``.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

# training workloads: model key in mega_trading_b200.model.CONFIGS, global batch,
# sequence length, default micro-batch per rank
WORKLOADS = {
    "gqa12": {"metric": "train tokens/s (config 3: 12L d768 GQA 12/4, seq 2048, global batch 256)",
              "workload": "config3_train_step", "global_batch": 256, "seq": 2048, "micro_batch": 128,
              "model": "12L d768 Hq12/Hkv4 D64 I2048 V21504"},
    "large24": {"metric": "train tokens/s (config 4: 24L d1024 GQA 16/4, seq 4096, global batch 128)",
                "workload": "config4_train_step", "global_batch": 128, "seq": 4096, "micro_batch": 32,
                "model": "24L d1024 Hq16/Hkv4 D64 I2816 V21504"},
}
CPU_SAMPLE_SEQS = 1
# DRAM bytes (read + write) of one attn_bwd_kernel launch measured by ncu at
# B=128, Hq=12, Hkv=4, T=2048, D=64 (profiles/attention_bwd_config3_layer.txt);
# traffic grows with the batch, so a launch of B sequences moves B/128 times this.
# Keyed by the workload whose shape it was captured on.
ATTN_BWD_DRAM_BYTES = {"gqa12": (1_904_345_088 + 1_028_964_352, 128)}


def _ref_config(name: str):
    """The oracle model configuration for a workload (same fields as the product's)."""
    from dataclasses import asdict

    from oracle.model import ModelConfig as RefCfg

    from mega_trading_b200.model import CONFIGS

    return RefCfg(**asdict(CONFIGS[name]))


def _peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms during the timed region:
    entering waits (up to 5 s) for the first sample, and only samples written after
    ``mark()`` (called right before timing starts) are summarised."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu = gpu_index
        self.proc = None
        self.path = Path(tempfile.mkstemp(prefix="clocks_", suffix=".csv")[1])
        self.skip = 0

    def _lines(self) -> list[str]:
        try:
            return self.path.read_text().splitlines()
        except OSError:
            return []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=self.path.open("w"), stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None
        t0 = time.time()
        while self.proc is not None and not self._lines() and time.time() - t0 < 5.0:
            time.sleep(0.02)
        return self

    def mark(self) -> None:
        """Samples from here on belong to the timed region."""
        self.skip = len(self._lines())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        try:
            for line in self._lines()[self.skip:]:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                    rows.append(parts)
        finally:
            self.path.unlink(missing_ok=True)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())}


def _cpu_trainer(model_name: str):
    """The CPU fp32 train step the CPU legs time: the reference's own ``TradingModel`` from the
    installed copy under ``baseline/_ref`` (its torch operator path, ``attention_backend="auto"``,
    dropout 0) when that copy is present (kind ``reference``), else the oracle's restatement
    (kind ``port``).  Both step forward_with_loss, backward and AdamW with the reference's
    settings (lr 2e-4, betas (0.9, 0.999), eps 1e-8, weight decay 0.01)."""
    from dataclasses import asdict

    from oracle.model import TradingModelRef, make_optimizer, train_step

    from mega_trading_b200.microbench import load_reference
    from mega_trading_b200.model import CONFIGS

    torch.manual_seed(0)
    ref = load_reference()
    if ref is not None:
        model = ref[2].TradingModel(dropout=0.0, attention_backend="auto", **asdict(CONFIGS[model_name]))
        opt = make_optimizer(model)

        def step(ids, labels):
            loss, _ = model.forward_with_loss(ids, labels, return_logits=False)
            loss.backward()
            opt.step()
            opt.zero_grad(set_to_none=True)
            return loss.detach()

        return step, "reference", "the reference's own TradingModel (baseline/_ref), torch operator path"
    model = TradingModelRef(_ref_config(model_name))
    opt = make_optimizer(model)
    return (lambda ids, labels: train_step(model, opt, ids, labels)), "port", "oracle restatement of the reference"


def cpu_train_tokens_per_s(seqs: int, seq_len: int, steps: int | None = None, budget_s: float = 12.0,
                           model_name: str = "gqa12") -> dict:
    """The reference's PyTorch train step on the host cores (see ``_cpu_trainer``)."""
    from mega_trading_b200.data import next_token_batch

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    train_step, kind, what = _cpu_trainer(model_name)
    ids, labels = next_token_batch(seqs, seq_len, seed=7, device="cpu")
    train_step(ids, labels)  # warm-up
    times = []
    t_start = time.perf_counter()
    while True:
        t0 = time.perf_counter()
        train_step(ids, labels)
        times.append(time.perf_counter() - t0)
        if steps is not None and len(times) >= steps:
            break
        if steps is None and time.perf_counter() - t_start > budget_s:
            break
    tok = seqs * seq_len
    return {"value": tok / statistics.mean(times), "unit": "tokens/s", "cores": torch.get_num_threads(),
            "kind": kind, "steps": len(times),
            "sample": f"{seqs} x {seq_len}-token sequence(s) per step of the {WORKLOADS[model_name]['model']} "
                      f"model ({what}), fp32, full step "
                      f"(forward, CE, backward, AdamW); {len(times)} timed step(s)"}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    steps, warm = args.steps, args.warmup
    wl = WORKLOADS[args.model]
    SEQ = wl["seq"]
    from mega_trading_b200.data import next_token_batch

    torch.set_num_threads(os.cpu_count() or 1)
    train_step, kind, what = _cpu_trainer(args.model)
    ids, labels = next_token_batch(CPU_SAMPLE_SEQS, SEQ, seed=7, device="cpu")
    for _ in range(warm):
        train_step(ids, labels)
    t0 = time.perf_counter()
    for _ in range(steps):
        train_step(ids, labels)
    el = time.perf_counter() - t0
    tok = CPU_SAMPLE_SEQS * SEQ
    value = tok * steps / el
    line = {
        "impl": "reference", "metric": wl["metric"], "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": steps, "warmup": warm, "ms_per_step": 1000 * el / steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic composite-token streams",
        "config": {"workload": wl["workload"], "architecture": wl["model"],
                   "global_batch": CPU_SAMPLE_SEQS, "seq_len": SEQ, "parallelism": "host cores"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": kind,
                         "sample": f"{CPU_SAMPLE_SEQS} x {SEQ}-token sequence per step (bounded sample of the "
                                   f"global batch of {wl['global_batch']}) through {what}, "
                                   "fp32 forward+CE+backward+AdamW"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--model", choices=tuple(WORKLOADS), default="gqa12",
                    help="gqa12 = BASELINE config 3 (default), large24 = config 4")
    ap.add_argument("--micro-batch", type=int, default=None, help="sequences per micro-step and rank")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--global-batch", type=int, default=None,
                    help="analysis only: override the workload's global batch (the metric then no longer matches "
                         "the BASELINE configuration)")
    ap.add_argument("--bucket-mb", type=int, default=64, help="DDP gradient bucket size (MB)")
    ap.add_argument("--comm-priority", choices=("high", "normal"), default="high",
                    help="stream priority of the gradient all-reduce")
    ap.add_argument("--comm-max-ctas", type=int, default=None, help="cap on the CTAs NCCL uses per collective")
    ap.add_argument("--host-profile", action="store_true",
                    help="analysis: cProfile the host side of the timed steps and print the top entries and "
                         "the host milliseconds per step to stderr")
    ap.add_argument("--phase-split", action="store_true",
                    help="also time the phases of each step (forward, backward, the last backward with the "
                         "gradient all-reduce, optimizer) with CUDA events on every rank")
    args = ap.parse_args(argv)
    if args.impl == "reference":
        run_reference(args)
        return 0

    from mega_trading_b200 import _lib
    from mega_trading_b200.data import next_token_batch
    from mega_trading_b200.model import CONFIGS
    from mega_trading_b200.train import Trainer, init_distributed

    wl = WORKLOADS[args.model]
    METRIC, GLOBAL_BATCH, SEQ = wl["metric"], wl["global_batch"], wl["seq"]
    if args.global_batch:
        GLOBAL_BATCH = int(args.global_batch)
        METRIC += f" [analysis run: global batch {GLOBAL_BATCH}]"
    rank, world, local = init_distributed("nccl", comm_high_priority=args.comm_priority == "high",
                                          comm_max_ctas=args.comm_max_ctas)
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if GLOBAL_BATCH % world:
        raise SystemExit(f"global batch {GLOBAL_BATCH} is not divisible by {world} ranks")
    cfg = CONFIGS[args.model]
    local_batch = GLOBAL_BATCH // world
    micro = min(args.micro_batch or wl["micro_batch"], local_batch)
    trainer = Trainer(cfg, micro_batch=micro, device=device, bucket_cap_mb=args.bucket_mb)
    ids, labels = next_token_batch(local_batch, SEQ, seed=1000 + rank, device=device)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    torch.cuda.reset_peak_memory_stats(device)
    for _ in range(max(args.warmup, 0)):
        trainer.step(ids, labels)
    torch.cuda.synchronize()

    # ---------------- timed region: K steps, inputs resident in HBM ----------------
    _lib.timer.reset()
    _lib.timer.enabled = True
    launches0 = _lib.launch_count()
    stream = torch.cuda.current_stream(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    if args.phase_split:
        trainer.phase_log = []
    with ClockSampler(local) as clocks:
        clocks.mark()
        start.record(stream)
        step_ev = []
        prof = None
        if args.host_profile:
            import cProfile

            prof = cProfile.Profile()
            blocked0 = trainer.monitor.blocked_s
            host_t0 = time.perf_counter()
            prof.enable()
        for _ in range(args.steps):
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record(stream)
            loss = trainer.step(ids, labels)
            ev[1].record(stream)
            step_ev.append(ev)
        if prof is not None:
            prof.disable()
            host_ms = 1000.0 * (time.perf_counter() - host_t0) / max(args.steps, 1)
        end.record(stream)
        torch.cuda.synchronize()
        if prof is not None:
            import io
            import pstats

            out = io.StringIO()
            pstats.Stats(prof, stream=out).sort_stats("tottime").print_stats(15)
            drain_ms = 1000.0 * (time.perf_counter() - host_t0) / max(args.steps, 1) - host_ms
            print(f"rank {rank}: host {host_ms:.1f} ms per step (the device finished {drain_ms * args.steps:.1f} ms "
                  f"after the host loop); status-monitor wait "
                  f"{1000.0 * (trainer.monitor.blocked_s - blocked0) / max(args.steps, 1):.1f} ms per step\n"
                  f"{out.getvalue()}", file=sys.stderr, flush=True)
    barrier()
    launches = _lib.launch_count() - launches0
    _lib.timer.enabled = False
    phases = None
    if trainer.phase_log is not None:
        ph = Trainer.phase_summary(trainer.phase_log)
        trainer.phase_log = None
        names = sorted(ph)
        vec = torch.tensor([ph[k] for k in names], device=device, dtype=torch.float64)
        if world > 1:
            allv = [torch.empty_like(vec) for _ in range(world)]
            dist.all_gather(allv, vec)
        else:
            allv = [vec]
        per_rank = torch.stack(allv).cpu()
        phases = {k: {"min_over_ranks": float(per_rank[:, i].min()), "max_over_ranks": float(per_rank[:, i].max())}
                  for i, k in enumerate(names)}
    kern = _lib.timer.summary()
    elapsed = torch.tensor([start.elapsed_time(end)], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(elapsed, op=dist.ReduceOp.MAX)
    ms_step = float(elapsed.item()) / max(args.steps, 1)
    tokens_step = GLOBAL_BATCH * SEQ
    value = tokens_step / (ms_step / 1000.0)
    clock_summary = clocks.summary()
    status = _lib.read_status(device)

    # ---------------- e2e: host token buffers, H2D + loss D2H inside the timed region ----------------
    host = torch.cat([ids.cpu(), labels[:, -1:].cpu()], dim=1).pin_memory()
    dev_tokens = torch.empty_like(host, device=device)
    loss_host = torch.empty((), dtype=torch.float32).pin_memory()
    e2e_steps = max(1, args.steps)
    barrier()
    torch.cuda.synchronize()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    e2e_ev = []
    for _ in range(e2e_steps):
        ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        ev[0].record(stream)
        dev_tokens.copy_(host, non_blocking=True)
        loss = trainer.step(dev_tokens[:, :-1], dev_tokens[:, 1:])
        loss_host.copy_(loss, non_blocking=True)
        ev[1].record(stream)
        e2e_ev.append(ev)
    e_end.record(stream)
    torch.cuda.synchronize()
    barrier()
    e_el = torch.tensor([e_start.elapsed_time(e_end)], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(e_el, op=dist.ReduceOp.MAX)
    e2e_value = tokens_step / (float(e_el.item()) / e2e_steps / 1000.0)
    status = status or _lib.read_status(device)

    def spread(evs):
        ms = sorted(a.elapsed_time(b) for a, b in evs)
        return {"min": ms[0], "median": statistics.median(ms), "max": ms[-1]} if ms else None

    # ---------------- roofline of the dominant kernel (attention backward) ----------------
    peaks = _peaks()
    B = micro
    fwd_flops = 4.0 * B * cfg.attention_heads * cfg.head_dim * SEQ * (SEQ + 1) / 2  # per launch (one layer)
    bwd_flops = 2.5 * fwd_flops
    # the main attention kernels alone (events the library records around them)
    n_bwd, ms_bwd = kern.get("attention_bwd_kernel", kern.get("attention_bwd", (0, float("nan"))))
    n_fwd, ms_fwd = kern.get("attention_fwd_kernel", kern.get("attention_fwd", (0, float("nan"))))
    achieved = bwd_flops / (ms_bwd / 1000.0) / 1e12
    # minimum: q, dO, k, v, lse, delta read once; dq, dk, dv written once (16-bit)
    rows_q = B * cfg.attention_heads * SEQ
    rows_kv = B * cfg.kv_heads * SEQ
    attn_bwd_bytes = (3 * rows_q + 4 * rows_kv) * cfg.head_dim * 2 + rows_q * 8
    if args.model in ATTN_BWD_DRAM_BYTES:
        cap_bytes, cap_b = ATTN_BWD_DRAM_BYTES[args.model]
        traffic = cap_bytes * B / cap_b
        traffic_source = f"ncu dram__bytes_read+write of one launch at B={cap_b}, scaled by B={B}"
    else:
        traffic, traffic_source = None, f"no ncu capture of this kernel at the {wl['workload']} shape"
    kernels = {name: {"launches": n, "mean_ms": ms} for name, (n, ms) in kern.items()}
    for name, fl in (("attention_fwd", fwd_flops), ("attention_bwd", bwd_flops)):
        for key in (name, name + "_kernel"):
            if key in kern:
                kernels[key]["tflops"] = fl / (kern[key][1] / 1000.0) / 1e12
    # algorithmic CE work: forward 2NHV (logits), backward 4NHV (dH and dW); the
    # backward also recomputes the logits twice (4NHV more), not counted here
    ce_flops = 2.0 * B * SEQ * cfg.hidden_dim * cfg.vocab_size
    for name, mult in (("fused_ce_fwd", 1.0), ("fused_ce_bwd", 2.0)):
        if name in kern:
            kernels[name]["tflops"] = mult * ce_flops / (kern[name][1] / 1000.0) / 1e12
            kernels[name]["tflops_executed"] = (1.0 if mult == 1.0 else 4.0) * ce_flops / (kern[name][1] / 1e3) / 1e12
    # north-star aggregate: algorithmic attention (fwd + 2.5x bwd) and fused-CE (2NHV fwd + 4NHV bwd)
    # FLOP of the timed steps over the device time of those kernels, against the sustained peak
    att_ms = sum(kern[k][0] * kern[k][1] for k in ("attention_fwd_kernel", "attention_bwd_kernel") if k in kern)
    ce_ms = sum(kern[k][0] * kern[k][1] for k in ("fused_ce_fwd", "fused_ce_bwd") if k in kern)
    att_flops = (kern.get("attention_fwd_kernel", (0, 0))[0] * fwd_flops
                 + kern.get("attention_bwd_kernel", (0, 0))[0] * bwd_flops)
    ce_flops_all = (kern.get("fused_ce_fwd", (0, 0))[0] * ce_flops + kern.get("fused_ce_bwd", (0, 0))[0] * 2 * ce_flops)
    north = None
    if att_ms + ce_ms > 0:
        ach = (att_flops + ce_flops_all) / ((att_ms + ce_ms) / 1000.0) / 1e12
        north = {"kernels": "attention fwd/bwd main kernels + fused CE fwd/bwd, algorithmic FLOP",
                 "achieved_tflops": ach, "frac_of_sustained": ach / peaks["bf16_tflops_sustained"],
                 "ms_in_timed_steps": att_ms + ce_ms, "target_frac": 0.60}
    step_flops = cfg.train_flops_per_token(SEQ) * tokens_step
    mfu = step_flops / (ms_step / 1000.0) / 1e12 / (world * peaks["bf16_tflops"])

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_train_tokens_per_s(CPU_SAMPLE_SEQS, SEQ, model_name=args.model)

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_step,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic composite-token streams (seeded, BASELINE distribution), generated on device",
            "config": {
                "workload": wl["workload"],
                "architecture": wl["model"] + " (dropout 0, tied embeddings)",
                "global_batch": GLOBAL_BATCH, "seq_len": SEQ, "micro_batch": micro,
                "grad_accum": math.ceil(local_batch / micro), "parallelism": f"dp{world}",
                "allreduce": f"NCCL, fp32 gradients, {args.bucket_mb} MB buckets overlapped with backward, "
                             f"{args.comm_priority}-priority stream"
                             + (f", at most {args.comm_max_ctas} CTAs" if args.comm_max_ctas else ""),
                "optimizer": "fused AdamW, fp32 master weights",
                "l2": f"no flush: per-step working set (activations of {micro} x {SEQ} tokens, tens of GB) "
                      "is far larger than L2",
            },
            "roofline": {
                "kernel": "attn_bwd_kernel (tcgen05, per launch = one layer of one micro-batch; CUDA events the "
                          "library records on the launch stream right around this kernel)",
                "bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops_sustained"], "unit": "TFLOP/s",
                "frac": achieved / peaks["bf16_tflops_sustained"],
                "peak_source": peaks["source"] + " (sustained bf16: the kernel runs inside a long step)",
                "traffic": traffic,
                "traffic_source": traffic_source,
                "algorithmic_flops_per_launch": bwd_flops,
                "algorithmic_bytes_per_launch": attn_bwd_bytes,
            },
            "mfu": mfu,
            "attention_ce_roofline": north,
            "kernels": kernels,
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": host.numel() * host.element_size(),
                    "d2h_bytes_per_step": 4, "steps": e2e_steps,
                    "note": "per rank: pinned host tokens copied to HBM and the loss read back every step",
                    "step_ms": spread(e2e_ev)},
            "step_ms": spread(step_ev),
            **({"phase_ms": phases} if phases is not None else {}),
            "gpu_launches": launches,
            "peak_memory_gb": torch.cuda.max_memory_allocated(device) / 1e9,
            "device_status": status,
            "clocks": clock_summary,
            "last_loss": float(loss_host),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    if status:
        print(f"device status word {status:#x}: {_lib.describe_status(status)}", file=sys.stderr, flush=True)
        return 1
    return 0


if __name__ == "__main__":
    sys.exit(main())
