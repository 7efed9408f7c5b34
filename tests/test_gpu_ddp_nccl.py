"""Data parallelism of the B200 model over NCCL (needs 2 GPUs; skipped otherwise).

Two ranks, one per GPU, each run the DDP-wrapped model of ``Trainer`` forward
and backward on half of a batch with the sm_100a kernels; the all-reduced
gradients must be identical on both ranks and equal, within the bf16 tolerance
of the kernels, to one process's gradients on the whole batch (the reference's
Accelerate DDP step: gradient all-reduce-mean before AdamW).  Parameters after
AdamW are not compared: its first update is +-lr wherever a gradient is
non-zero, so rounding noise in near-zero gradients flips whole steps.
Ranks are child processes with a short process-group timeout, so a failure on
one ends the other's collective with an error instead of waiting."""

from __future__ import annotations

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

needs_two = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                               reason="needs two GPUs")


def _cfg():
    from mega_trading_b200.model import ModelConfig

    return ModelConfig(vocab_size=512, block_size=256, hidden_dim=256, layers=2, attention_heads=8, kv_heads=2,
                       intermediate_dim=688, rope_theta=10_000.0)


def _worker(rank, world, port, ids, labels, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    from mega_trading_b200.train import Trainer, init_distributed

    init_distributed("nccl", timeout_s=60)
    dev = torch.device("cuda", rank)
    tr = Trainer(_cfg(), micro_batch=2, device=dev, seed=0)
    n = ids.shape[0] // world
    loss = tr.engine(ids[rank * n:(rank + 1) * n].to(dev), labels[rank * n:(rank + 1) * n].to(dev))
    loss.backward()
    torch.cuda.synchronize(dev)
    grads = {k: p.grad.detach().float().cpu() for k, p in tr.model.named_parameters() if p.grad is not None}
    torch.save(grads, os.path.join(outdir, f"rank{rank}.pt"))
    dist.barrier(device_ids=[rank])
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@needs_two
def test_two_gpu_step_equals_single_gpu_step(tmp_path):
    import torch.multiprocessing as mp

    from mega_trading_b200.train import Trainer

    g = torch.Generator().manual_seed(7)
    ids = torch.randint(0, 512, (4, 256), generator=g)
    labels = torch.randint(0, 512, (4, 256), generator=g)
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, ids, labels, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    r0 = torch.load(tmp_path / "rank0.pt")
    r1 = torch.load(tmp_path / "rank1.pt")

    dev = torch.device("cuda", 0)
    single = Trainer(_cfg(), micro_batch=4, device=dev, seed=0)
    single.engine(ids.to(dev), labels.to(dev)).backward()
    ref = {k: p.grad.detach().float().cpu() for k, p in single.model.named_parameters() if p.grad is not None}
    assert set(ref) == set(r0) == set(r1)
    for k in ref:
        assert torch.equal(r0[k], r1[k]), f"all-reduced gradients differ between ranks in {k}"
        scale = ref[k].abs().max().item()
        err = (r0[k] - ref[k]).abs().max().item() / max(scale, 1e-30)
        assert err < 5e-2, f"{k}: data-parallel gradient differs from single-GPU gradient by {err:.3e}"
