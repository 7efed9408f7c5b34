"""A rank lost between steps, on NCCL ranks (needs 2 GPUs; skipped otherwise).

Two child processes, one per GPU, with NVLS off, run one data-parallel step of
the sm_100a model together (its gradient all-reduce included) and synchronise.
Then rank 1 leaves between steps, with no kernel or collective in flight:
either it exits, or it stays alive and never starts step 2.  Rank 0's
``Trainer`` (``peer_timeout_s``) posts its heartbeat for step 2 in the process
group's store and waits for rank 1's; it must raise ``PeerLostError`` naming
rank 1 within the timeout, before launching any kernel of step 2, and its GPU
must stay usable (a kernel runs afterwards and the device status word is 0).
The failure is made on the host only: nothing faults, traps or hangs a GPU.
"""

from __future__ import annotations

import json
import os
import socket
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

needs_two = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                               reason="needs two GPUs")
PEER_TIMEOUT_S = 3.0


def _cfg():
    from mega_trading_b200.model import ModelConfig

    return ModelConfig(vocab_size=512, block_size=256, hidden_dim=256, layers=2, attention_heads=8, kv_heads=2,
                       intermediate_dim=688, rope_theta=10_000.0)


def _worker(rank, world, port, mode, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    from mega_trading_b200 import _lib
    from mega_trading_b200.train import PeerLostError, Trainer, init_distributed

    init_distributed("nccl", timeout_s=60)
    dev = torch.device("cuda", rank)
    tr = Trainer(_cfg(), micro_batch=2, device=dev, seed=0, peer_timeout_s=PEER_TIMEOUT_S)
    g = torch.Generator().manual_seed(rank)
    ids = torch.randint(0, 512, (2, 256), generator=g).to(dev)
    labels = torch.randint(0, 512, (2, 256), generator=g).to(dev)
    tr.step(ids, labels)  # step 1 on both ranks, all-reduce included
    torch.cuda.synchronize(dev)
    tr.check_status()
    if rank == 1:
        if mode == "exit":
            os._exit(0)  # nothing of ours in flight: the step above was synchronised
        time.sleep(PEER_TIMEOUT_S * 3)
        os._exit(0)
    launches0 = _lib.launch_count()
    outcome = {"raised": None, "message": None, "elapsed_s": None}
    t0 = time.monotonic()
    try:
        tr.step(ids, labels)
    except PeerLostError as exc:
        outcome["raised"] = "PeerLostError"
        outcome["message"] = str(exc)[:300]
    outcome["elapsed_s"] = time.monotonic() - t0
    outcome["launches_in_failed_step"] = _lib.launch_count() - launches0
    # the device is still usable and no kernel reported an error
    x = torch.ones(1024, device=dev)
    outcome["after"] = float((x * 2).sum().item())
    outcome["status"] = int(_lib.read_status(dev))
    with open(os.path.join(outdir, "rank0.json"), "w") as f:
        json.dump(outcome, f)
    os._exit(0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@needs_two
@pytest.mark.parametrize("mode", ["exit", "stall"])
def test_lost_rank_is_detected_before_the_next_collective(tmp_path, mode):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        if p.is_alive():
            p.kill()
            p.join()
    assert [p.exitcode for p in procs] == [0, 0]
    out = json.loads((tmp_path / "rank0.json").read_text())
    assert out["raised"] == "PeerLostError", out
    assert "rank(s) 1" in out["message"], out
    assert PEER_TIMEOUT_S * 0.5 < out["elapsed_s"] < PEER_TIMEOUT_S + 10, out
    assert out["launches_in_failed_step"] == 0, out
    assert out["after"] == 2048.0 and out["status"] == 0, out
