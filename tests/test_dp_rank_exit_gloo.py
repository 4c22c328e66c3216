"""A data-parallel rank that leaves between steps, on CPU ranks (gloo).

Two ranks run one data-parallel step of the crater CNN (the oracle's step on
each shard, gradients summed with remora_b200.cnn.process_group_allreduce).
Rank 1 then leaves between steps, with nothing in flight: it exits, or it
stalls (stays alive without joining the next collective).  Rank 0's next
step must end with an error from its gradient allreduce -- at once when the
peer's connection closes, within the process group's short timeout when it
stalls -- instead of waiting for good; the test bounds every process and
kills any that outlives it."""

from __future__ import annotations

import json
import multiprocessing as mp
import os
import socket
import sys
import time
from datetime import timedelta
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]

GROUP_TIMEOUT_S = 10


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, port: int, out: str, mode: str) -> None:
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    import torch
    import torch.distributed as dist

    from remora_b200 import crater
    from remora_b200.cnn import process_group_allreduce, shard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=timedelta(seconds=GROUP_TIMEOUT_S))
    allreduce = process_group_allreduce()
    params = crater.init_params()
    imgs, labs = crater.make_batch(4)
    lo, hi = shard(4, 2, rank)

    def step() -> None:
        _, g = oracle.cnn_step(params, imgs[lo:hi], labs[lo:hi], batch_total=4, apply_sgd=False)
        allreduce(torch.from_numpy(g))

    step()  # both ranks: one good step
    if rank == 1:
        if mode == "stall":
            # alive, but never joins the next step (until rank 0 has its answer)
            end = time.monotonic() + 3 * GROUP_TIMEOUT_S
            while time.monotonic() < end and not Path(out).exists():
                time.sleep(0.2)
        os._exit(0)  # leaves between steps, with no collective in flight
    t0 = time.monotonic()
    try:
        step()
        result = {"raised": False}
    except Exception as exc:  # the collective's error
        result = {"raised": True, "type": type(exc).__name__, "message": str(exc)[:200]}
    result["seconds"] = time.monotonic() - t0
    Path(out).write_text(json.dumps(result))
    os._exit(0)


@pytest.mark.parametrize("mode", ["exit", "stall"])
def test_a_rank_that_leaves_ends_the_next_allreduce_with_an_error(tmp_path, mode):
    ctx = mp.get_context("spawn")
    port = _free_port()
    out = str(tmp_path / "rank0.json")
    procs = [ctx.Process(target=_rank_main, args=(r, port, out, mode)) for r in range(2)]
    for p in procs:
        p.start()
    deadline = time.monotonic() + 6 * GROUP_TIMEOUT_S + 60
    for p in procs:
        p.join(timeout=max(1.0, deadline - time.monotonic()))
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
        p.join(5)
    assert not alive, "a rank outlived the bound: the collective did not end"
    result = json.loads(Path(out).read_text())
    assert result["raised"], result
    assert result["seconds"] < (5 if mode == "exit" else 3 * GROUP_TIMEOUT_S), result
