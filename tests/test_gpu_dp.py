"""Data-parallel crater-CNN step on two GPUs: torchrun launches two ranks
(tests/dp/cnn_dp_worker.py) that split a global batch, sum their gradients
with the NCCL allreduce (eager and inside a captured CUDA graph) and apply
the same SGD update.  The replicas must stay bitwise identical and match
the single-GPU step on the whole batch (per-sample gradients are summed in
another order across ranks: 3xTF32 tolerance).  Skipped with fewer than two
GPUs."""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def _gpus() -> int:
    import torch

    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
def test_cnn_data_parallel_two_gpus(tmp_path):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29517", str(ROOT / "tests" / "dp" / "cnn_dp_worker.py"),
           str(tmp_path), "64", "3xtf32"]
    r = subprocess.run(["timeout", "-k", "30", "240", *cmd], env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    p0 = np.load(tmp_path / "params_rank0.npy")
    p1 = np.load(tmp_path / "params_rank1.npy")
    ps = np.load(tmp_path / "params_single.npy")
    assert np.array_equal(p0, p1)
    assert np.isfinite(p0).all()
    init = np.asarray(__import__("remora_b200.crater", fromlist=["init_params"]).init_params())
    step = np.abs(ps - init).max()
    assert step > 0
    np.testing.assert_allclose(p0, ps, rtol=1e-4, atol=1e-4 * step)


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
def test_cnn_step_entry_point_two_gpus_with_a_library_communicator(tmp_path):
    """remora_b200_cnn_step with an ncclComm_t made by
    remora_b200_nccl_comm_init (tests/dp/cnn_step_dp_worker.py): the two
    replicas stay bitwise identical and match the one-GPU step on the whole
    batch at the 3xTF32 tolerance."""
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29518", str(ROOT / "tests" / "dp" / "cnn_step_dp_worker.py"),
           str(tmp_path), "64"]
    r = subprocess.run(["timeout", "-k", "30", "240", *cmd], env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    p0 = np.load(tmp_path / "params_rank0.npy")
    p1 = np.load(tmp_path / "params_rank1.npy")
    ps = np.load(tmp_path / "params_single.npy")
    assert np.array_equal(p0, p1) and np.isfinite(p0).all()
    init = np.asarray(__import__("remora_b200.crater", fromlist=["init_params"]).init_params())
    step = np.abs(ps - init).max()
    np.testing.assert_allclose(p0, ps, rtol=1e-4, atol=1e-4 * step)
