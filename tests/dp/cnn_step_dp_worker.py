"""Worker for the two-GPU test of remora_b200_cnn_step (launched by
torchrun): rank 0 makes an NCCL unique id through the library, the ranks
share it over a host (gloo) group, each makes its communicator with
remora_b200_nccl_comm_init and runs two SGD steps of its shard through the
one C entry point; rank 0 also runs the whole batch on one GPU."""

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
from remora_b200.cnn import cnn_step, nccl_comm_destroy, nccl_comm_init, nccl_unique_id, shard  # noqa: E402


def main() -> None:
    out_dir = Path(sys.argv[1])
    global_batch = int(sys.argv[2])
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("gloo", timeout=timedelta(seconds=60))  # host channel for the unique id only
    comm = None
    try:
        box = [nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        comm = nccl_comm_init(world, box[0], rank)
        parts = [crater.make_batch(global_batch // world, start=r * (global_batch // world)) for r in range(world)]
        imgs = np.concatenate([q[0] for q in parts])
        labs = np.concatenate([q[1] for q in parts])
        lo, hi = shard(global_batch, world, rank)
        x, y = torch.from_numpy(imgs[lo:hi]).to(dev), torch.from_numpy(labs[lo:hi]).to(dev)
        p = torch.from_numpy(crater.init_params()).to(dev)
        g = torch.zeros(crater.NPARAMS, dtype=torch.float32, device=dev)
        for _ in range(2):
            cnn_step(p, g, x, y, batch_total=global_batch, lr=0.05, comm=comm)
        torch.cuda.synchronize()
        np.save(out_dir / f"params_rank{rank}.npy", p.cpu().numpy())
        dist.barrier()
        if rank == 0:
            xa, ya = torch.from_numpy(imgs).to(dev), torch.from_numpy(labs).to(dev)
            pa = torch.from_numpy(crater.init_params()).to(dev)
            ga = torch.zeros_like(pa)
            for _ in range(2):
                cnn_step(pa, ga, xa, ya, lr=0.05)
            torch.cuda.synchronize()
            np.save(out_dir / "params_single.npy", pa.cpu().numpy())
        dist.barrier()
    finally:
        if comm is not None:
            nccl_comm_destroy(comm)
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
