"""Failure detection of the data-parallel step, with the failure made on the host.

Two gloo ranks on CPU run one training step together; then rank 1 leaves
between steps, either by exiting (a crashed process) or by never joining the
next step's collective (a hung process).  Rank 0's next step must end with an
error from its gradient all-reduce within the process group's timeout instead
of waiting for ever.  No GPU is involved: the same ``Trainer`` drives the CPU
oracle model (the path ``bench.py`` takes on the GPU differs only in backend).
"""

from __future__ import annotations

import json
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

PG_TIMEOUT_S = 5


def _cfg():
    from oracle.model import ModelConfig

    return ModelConfig(vocab_size=64, block_size=16, hidden_dim=32, layers=1, attention_heads=4, kv_heads=2,
                       intermediate_dim=48, rope_theta=10_000.0)


class _LossWrapper(torch.nn.Module):
    def __init__(self, m):
        super().__init__()
        self.m = m

    def forward(self, ids, labels):
        return self.m.forward_with_loss(ids, labels)[0]


def _worker(rank, world, port, mode, outdir, peer_timeout_s=None):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from oracle.model import TradingModelRef

    from mega_trading_b200.train import Trainer, init_distributed

    init_distributed("gloo", timeout_s=PG_TIMEOUT_S)
    torch.manual_seed(0)
    tr = Trainer(_cfg(), micro_batch=2, device=torch.device("cpu"), model=_LossWrapper(TradingModelRef(_cfg())),
                 seed=0, peer_timeout_s=peer_timeout_s)
    g = torch.Generator().manual_seed(rank)
    ids = torch.randint(0, 64, (2, 16), generator=g)
    labels = torch.randint(0, 64, (2, 16), generator=g)
    tr.step(ids, labels)  # both ranks complete step 1
    if rank == 1:
        if mode == "exit":
            os._exit(0)  # leaves between steps without tearing the group down
        time.sleep(PG_TIMEOUT_S * 4)  # alive, but never joins step 2
        os._exit(0)
    t0 = time.monotonic()
    outcome = {"raised": None, "elapsed_s": None, "message": None}
    try:
        tr.step(ids, labels)
    except Exception as exc:  # noqa: BLE001 - the error type is backend specific
        outcome["raised"] = type(exc).__name__
        outcome["message"] = str(exc)[:300]
    outcome["elapsed_s"] = time.monotonic() - t0
    with open(os.path.join(outdir, "rank0.json"), "w") as f:
        json.dump(outcome, f)
    os._exit(0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("mode", ["exit", "stall"])
def test_peer_leaving_between_steps_fails_the_next_collective(tmp_path, mode):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    assert procs[0].exitcode == 0
    outcome = json.loads((tmp_path / "rank0.json").read_text())
    assert outcome["raised"] is not None, "rank 0's step with a missing peer did not fail"
    # the collective ends within the process-group timeout (plus start-up slack), not after the peer
    assert outcome["elapsed_s"] < PG_TIMEOUT_S * 3, outcome
    if dist.is_initialized():
        dist.destroy_process_group()


HEARTBEAT_S = 2.0


@pytest.mark.parametrize("mode", ["exit", "stall"])
def test_peer_heartbeat_raises_before_the_collective(tmp_path, mode):
    """With ``peer_timeout_s`` the surviving rank learns of the missing peer on the host, at the
    start of its next step, and raises PeerLostError naming it before launching any work."""
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, str(tmp_path), HEARTBEAT_S)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    assert procs[0].exitcode == 0
    outcome = json.loads((tmp_path / "rank0.json").read_text())
    assert outcome["raised"] == "PeerLostError", outcome
    assert "rank(s) 1" in outcome["message"], outcome
    assert HEARTBEAT_S * 0.5 < outcome["elapsed_s"] < HEARTBEAT_S + PG_TIMEOUT_S, outcome
