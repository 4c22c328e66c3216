"""Worker for the multi-GPU data-parallel CNN test (launched by torchrun).

Each rank takes its shard of a global batch, runs CraterCNN.step with the
NCCL gradient allreduce (eagerly, then as a captured CUDA graph), and saves
its parameters.  Rank 0 also saves the single-GPU step on the whole batch.
"""

from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[2]))

from remora_b200 import crater  # noqa: E402
from remora_b200.cnn import CraterCNN, process_group_allreduce, shard  # noqa: E402


def main() -> None:
    out_dir = Path(sys.argv[1])
    global_batch = int(sys.argv[2])
    precision = sys.argv[3]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    try:
        parts = [crater.make_batch(global_batch // world, start=r * (global_batch // world)) for r in range(world)]
        imgs = np.concatenate([q[0] for q in parts])
        labs = np.concatenate([q[1] for q in parts])
        lo, hi = shard(global_batch, world, rank)
        x = torch.from_numpy(imgs[lo:hi]).to(dev)
        y = torch.from_numpy(labs[lo:hi]).to(dev)
        net = CraterCNN(dev, hi - lo, global_batch, lr=0.05, allreduce=process_group_allreduce(),
                        precision=precision)
        net.step(x, y)                 # eager step with the allreduce
        net.capture(x, y)              # records (and runs) a second step
        net.replay()                   # third step from the graph
        torch.cuda.synchronize()
        np.save(out_dir / f"params_rank{rank}.npy", net.params.cpu().numpy())
        net.release_graphs()           # graphs holding NCCL calls go before the group
        dist.barrier()
        if rank == 0:
            ref = CraterCNN(dev, global_batch, global_batch, lr=0.05, precision=precision)
            xa, ya = torch.from_numpy(imgs).to(dev), torch.from_numpy(labs).to(dev)
            for _ in range(3):
                ref.step(xa, ya)
            torch.cuda.synchronize()
            np.save(out_dir / "params_single.npy", ref.params.cpu().numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
