"""Data-parallel crater-CNN step on CPU ranks (gloo, world size 2).

Each rank takes its shard of the global batch (remora_b200.cnn.shard),
computes its gradient with the oracle's CNN step scaled by 1/global batch,
and sums it over ranks with the same reduction the GPU step uses
(remora_b200.cnn.process_group_allreduce).  The summed gradient must equal
the single-process gradient of the whole batch, and the replicas' updated
parameters must be identical on every rank.  Reference: the crater CNN of
examples/crater_train.py (the data-parallel form splits its batch).
"""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "oracle"))

GLOBAL = 8
LR = 0.05


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _batches():
    from remora_b200 import crater

    # the global batch is the concatenation of the ranks' shards
    parts = [crater.make_batch(GLOBAL // 2, start=r * (GLOBAL // 2)) for r in range(2)]
    return np.concatenate([p[0] for p in parts]), np.concatenate([p[1] for p in parts])


def _rank_main(rank: int, world: int, port: int, out_dir: str) -> None:
    import oracle

    from remora_b200 import crater
    from remora_b200.cnn import process_group_allreduce, shard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        imgs, labs = _batches()
        lo, hi = shard(GLOBAL, world, rank)
        params = crater.init_params()
        loss, g = oracle.cnn_step(params, imgs[lo:hi], labs[lo:hi], batch_total=GLOBAL, apply_sgd=False)
        grad = torch.from_numpy(g)
        process_group_allreduce()(grad)
        lsum = torch.tensor([loss], dtype=torch.float64)
        dist.all_reduce(lsum)
        new = params - np.float32(LR) * grad.numpy()
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), grad=grad.numpy(), params=new, loss=lsum.numpy())
    finally:
        dist.destroy_process_group()


def test_shard_bounds():
    from remora_b200.cnn import shard

    assert [shard(4096, 8, r) for r in (0, 7)] == [(0, 512), (3584, 4096)]
    assert shard(10, 1, 0) == (0, 10)
    with pytest.raises(ValueError):
        shard(10, 4, 0)
    with pytest.raises(ValueError):
        shard(8, 2, 2)


def test_dp_gradient_matches_full_batch(tmp_path):
    import oracle

    from remora_b200 import crater

    world = 2
    mp.spawn(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    res = [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]
    # identical replicas after the update
    assert np.array_equal(res[0]["grad"], res[1]["grad"])
    assert np.array_equal(res[0]["params"], res[1]["params"])
    # the reduced gradient is the full-batch gradient (summation order of the
    # per-sample terms differs: f32 tolerance)
    imgs, labs = _batches()
    loss, g_full = oracle.cnn_step(crater.init_params(), imgs, labs, batch_total=GLOBAL, apply_sgd=False)
    scale = float(np.abs(g_full).max())
    np.testing.assert_allclose(res[0]["grad"], g_full, rtol=1e-4, atol=1e-5 * scale)
    assert abs(float(res[0]["loss"][0]) - loss) <= 1e-5 * max(1.0, abs(loss))
