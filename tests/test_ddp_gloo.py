"""Data-parallel step logic on CPU with the gloo backend (world size 2).

The same ``Trainer`` the benchmark uses, driving the CPU oracle model: after
one step, both ranks hold identical parameters equal to a single-process step
on the concatenated batch (gradient all-reduce-mean is the only exchange);
gradient accumulation over micro-batches gives the same update."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _cfg():
    from oracle.model import ModelConfig

    return ModelConfig(vocab_size=64, block_size=16, hidden_dim=32, layers=1, attention_heads=4, kv_heads=2,
                       intermediate_dim=48, rope_theta=10_000.0)


def _single_step(batch_ids, batch_labels, micro):
    from oracle.model import TradingModelRef

    from mega_trading_b200.train import Trainer

    torch.manual_seed(0)
    model = TradingModelRef(_cfg())
    tr = Trainer(_cfg(), micro_batch=micro, device=torch.device("cpu"), model=model, seed=0)
    # the oracle model takes (ids, labels) through forward_with_loss
    tr.engine = _LossWrapper(model)
    tr.step(batch_ids, batch_labels)
    return {k: v.detach().clone() for k, v in model.state_dict().items()}


class _LossWrapper(torch.nn.Module):
    def __init__(self, m):
        super().__init__()
        self.m = m

    def forward(self, ids, labels):
        return self.m.forward_with_loss(ids, labels)[0]


def _worker(rank, world, port, ids, labels, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from oracle.model import TradingModelRef

    from mega_trading_b200.train import Trainer, init_distributed

    init_distributed("gloo", timeout_s=60)
    torch.manual_seed(0)
    model = _LossWrapper(TradingModelRef(_cfg()))
    tr = Trainer(_cfg(), micro_batch=1, device=torch.device("cpu"), model=model, seed=0)
    n = ids.shape[0] // world
    tr.step(ids[rank * n:(rank + 1) * n], labels[rank * n:(rank + 1) * n])
    torch.save({k.removeprefix("m."): v.detach().clone() for k, v in model.state_dict().items()},
               os.path.join(outdir, f"rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_gloo_step_equals_single_process_step(tmp_path):
    g = torch.Generator().manual_seed(5)
    ids = torch.randint(0, 64, (4, 16), generator=g)
    labels = torch.randint(0, 64, (4, 16), generator=g)
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, ids, labels, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        assert p.exitcode == 0
    results = {r: torch.load(tmp_path / f"rank{r}.pt") for r in range(2)}
    ref = _single_step(ids, labels, micro=4)
    for k in ref:
        assert torch.allclose(results[0][k], results[1][k]), k
        assert torch.allclose(results[0][k], ref[k], atol=1e-6, rtol=1e-5), k


def test_gradient_accumulation_matches_full_batch():
    g = torch.Generator().manual_seed(6)
    ids = torch.randint(0, 64, (4, 16), generator=g)
    labels = torch.randint(0, 64, (4, 16), generator=g)
    a = _single_step(ids, labels, micro=4)
    b = _single_step(ids, labels, micro=1)
    for k in a:
        assert torch.allclose(a[k], b[k], atol=1e-6, rtol=1e-5), k
