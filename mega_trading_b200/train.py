"""Data-parallel training step for the B200 model.

Mirrors the reference's hot loop (``src/mega_trading/trainer.py:324-345``):
forward, next-token cross-entropy (here the fused kernel, closing the wiring
gap at ``trainer.py:337-338``), backward with the bucketed NCCL gradient
all-reduce overlapped with backward (torch DDP, as Accelerate's default
``trainer.py:1009-1023, :300-308``), fused AdamW (``trainer.py:537-545``; on
the GPU ``optim.AdamWShadow``, which also writes the bf16 weight copies).
One process per GPU; the batch is split across ranks and, inside a rank,
across micro-batches (gradient accumulation, all-reduce on the last one).
The all-reduce is the only collective of the step.
"""

from __future__ import annotations

import contextlib
import datetime
import os
import time

import torch
import torch.distributed as dist

from . import _lib
from .model import ModelConfig, TradingModelB200
from .optim import AdamWShadow


def init_distributed(backend: str = "nccl", timeout_s: int = 300, *, comm_high_priority: bool = True,
                     comm_max_ctas: int | None = None) -> tuple[int, int, int]:
    """Initialise the default process group from torchrun's environment; returns
    ``(rank, world_size, local_rank)`` (``(0, 1, 0)`` without torchrun).

    With NCCL the gradient all-reduce runs on a high-priority stream by default:
    the step's persistent kernels hold every SM, and when their CTAs retire the
    block scheduler then places the waiting all-reduce CTAs before the next
    compute kernel's, so the collective keeps pace with the backward instead of
    piling up behind it.  ``comm_max_ctas`` caps the SMs NCCL takes per collective."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world <= 1:
        return 0, 1, 0
    rank = int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    if backend == "nccl":
        torch.cuda.set_device(local)
    if not dist.is_initialized():
        kwargs = {"timeout": datetime.timedelta(seconds=timeout_s)}
        if backend == "nccl":
            kwargs["device_id"] = torch.device("cuda", local)
            opts = dist.ProcessGroupNCCL.Options()
            opts.is_high_priority_stream = bool(comm_high_priority)
            if comm_max_ctas:
                opts.config.max_ctas = int(comm_max_ctas)
            kwargs["pg_options"] = opts
        dist.init_process_group(backend=backend, **kwargs)
    return rank, world, local


class PeerLostError(RuntimeError):
    """A peer rank did not reach the start of this step within the peer timeout."""


class Trainer:
    """Owns the model replica, the DDP wrapper and the optimizer of one rank.

    ``peer_timeout_s`` (multi-rank only) turns on a host-side liveness check at
    the start of every step: each rank posts a heartbeat for the step in the
    process group's store and waits, at most that long, for every peer's.  A
    rank that has exited or stopped between steps makes the others raise
    :class:`PeerLostError` before they launch any kernel or collective of the
    step, so no device work ever waits on a missing peer.  Without it a lost
    peer surfaces as the process group's timeout on the next all-reduce."""

    def __init__(self, cfg: ModelConfig, *, micro_batch: int, device: torch.device, lr: float = 2e-4,
                 weight_decay: float = 0.01, seed: int = 0, bucket_cap_mb: int = 64,
                 model: torch.nn.Module | None = None, peer_timeout_s: float | None = None) -> None:
        torch.manual_seed(seed)  # identical initial replicas on every rank
        self.cfg = cfg
        self.device = device
        self.micro_batch = int(micro_batch)
        # `model` lets host-side tests drive the same DP logic with another module
        self.model = (model if model is not None else TradingModelB200(cfg)).to(device)
        self.world = dist.get_world_size() if dist.is_initialized() else 1
        if self.world > 1:
            self.engine = torch.nn.parallel.DistributedDataParallel(
                self.model,
                device_ids=[device.index] if device.type == "cuda" else None,
                gradient_as_bucket_view=True,
                bucket_cap_mb=bucket_cap_mb,
                broadcast_buffers=False,
            )
        else:
            self.engine = self.model
        if device.type == "cuda" and hasattr(self.model, "packed_weights"):
            # one kernel per step: the AdamW update plus the bf16 GEMM-operand copies
            self.opt = AdamWShadow(self.model.parameters(), lr=lr, betas=(0.9, 0.999), eps=1e-8,
                                   weight_decay=weight_decay, packed=self.model.packed_weights())
        else:
            self.opt = torch.optim.AdamW(
                self.model.parameters(), lr=lr, betas=(0.9, 0.999), eps=1e-8, weight_decay=weight_decay,
                fused=device.type == "cuda",
            )
        # device status word of the bounded waits and the label check: the fused
        # AdamW leaves the weights alone when it is set, and every step polls it
        # without stalling (an error raises at most two steps later)
        self.monitor = _lib.StatusMonitor(device) if device.type == "cuda" else None
        # analysis hook: a list here collects, per step, CUDA event pairs around the
        # forward, backward (the last one includes waiting for the gradient
        # all-reduce) and optimizer phases on the current stream
        self.phase_log: list | None = None
        self.peer_timeout_s = peer_timeout_s if self.world > 1 else None
        self._store = dist.distributed_c10d._get_default_store() if self.peer_timeout_s else None
        self._steps = 0

    def _await_peers(self) -> None:
        """Post this rank's heartbeat for the coming step and wait for every peer's."""
        n, me = self._steps, dist.get_rank()
        self._store.set(f"mt_hb/{n}/{me}", "1")
        if n >= 2:
            self._store.delete_key(f"mt_hb/{n - 2}/{me}")
        peers = [f"mt_hb/{n}/{r}" for r in range(self.world) if r != me]
        t0 = time.monotonic()
        try:
            self._store.wait(peers, datetime.timedelta(seconds=float(self.peer_timeout_s)))
        except Exception as exc:  # the store raises its own timeout / connection errors
            missing = [k.rsplit("/", 1)[1] for k in peers if not self._safe_check(k)]
            raise PeerLostError(
                f"rank {me}: rank(s) {', '.join(missing) or '?'} did not reach step {n} within "
                f"{time.monotonic() - t0:.1f} s ({type(exc).__name__}: {exc})") from exc

    def _safe_check(self, key: str) -> bool:
        try:
            return bool(self._store.check([key]))
        except Exception:
            return False

    def _mark(self, marks: list | None, name: str) -> None:
        if marks is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            marks.append((name, ev))

    def check_status(self) -> None:
        """Wait for the device and raise :class:`~mega_trading_b200._lib.B200KernelError` if a
        kernel of an earlier step reported an error."""
        if self.monitor is not None:
            self.monitor.flush()
            _lib.check_status(self.device)

    def step(self, input_ids: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        """One optimizer step over this rank's ``[B, T]`` batch; returns the mean loss (device scalar,
        no host synchronisation)."""
        if self._store is not None:
            self._await_peers()
        self._steps += 1
        n = input_ids.shape[0]
        chunks = max(1, (n + self.micro_batch - 1) // self.micro_batch)
        total = torch.zeros((), device=input_ids.device, dtype=torch.float32)
        marks = [] if (self.phase_log is not None and input_ids.is_cuda) else None
        self._mark(marks, "start")
        for i in range(chunks):
            lo = i * self.micro_batch
            hi = min(n, lo + self.micro_batch)
            frac = (hi - lo) / n
            sync_ctx = self.engine.no_sync() if (self.world > 1 and i < chunks - 1) else contextlib.nullcontext()
            with sync_ctx:
                loss = self.engine(input_ids[lo:hi], labels[lo:hi])
                self._mark(marks, "forward")
                (loss * frac).backward()
                self._mark(marks, "backward" if i < chunks - 1 else "backward+allreduce")
            total += loss.detach() * frac
        self.opt.step()
        self.opt.zero_grad(set_to_none=self.world == 1)
        self._mark(marks, "optimizer")
        if marks is not None:
            self.phase_log.append(marks)
        if self.monitor is not None:
            self.monitor.poll()
        return total

    @staticmethod
    def phase_summary(log: list) -> dict:
        """Mean milliseconds per phase over the steps in ``log`` (events must have completed)."""
        acc: dict[str, float] = {}
        for marks in log:
            for (_, a), (name, b) in zip(marks, marks[1:]):
                acc[name] = acc.get(name, 0.0) + a.elapsed_time(b)
        return {k: v / max(len(log), 1) for k, v in acc.items()}
