"""Checkpoint and resume of the crater-CNN training state on the host.

The reference keeps parameter snapshots every K epochs in memory
(examples/crater_train.py:236,263-264); remora_b200.cnn.save_checkpoint /
load_checkpoint write and read them as .npz.  A run that stops after two SGD
steps, checkpoints, and resumes from the file for a third must end with the
same parameters, bit for bit, as a run of three steps (the oracle's step is
deterministic)."""

from __future__ import annotations

import numpy as np
import pytest

from remora_b200 import crater
from remora_b200.cnn import load_checkpoint, save_checkpoint


def test_round_trip_keeps_every_field(tmp_path):
    p = crater.init_params()
    save_checkpoint(tmp_path / "c.npz", p, 17, lr=0.01, batch_total=4096, precision="mixed")
    st = load_checkpoint(tmp_path / "c.npz")
    assert np.array_equal(st["params"], p) and st["params"].dtype == np.float32
    assert (st["step"], st["lr"], st["batch_total"], st["precision"]) == (17, 0.01, 4096, "mixed")
    assert (st["data_seed"], st["parameter_seed"]) == (crater.DATA_SEED, crater.PARAMETER_SEED)
    assert sorted(f.name for f in tmp_path.iterdir()) == ["c.npz"]  # no temporary left behind


def test_a_wrong_size_or_layout_is_refused(tmp_path):
    with pytest.raises(ValueError):
        save_checkpoint(tmp_path / "c.npz", np.zeros(10, np.float32), 0, lr=0.01, batch_total=8)
    p = crater.init_params()
    save_checkpoint(tmp_path / "c.npz", p, 0, lr=0.01, batch_total=8)
    with np.load(tmp_path / "c.npz") as f:
        d = {k: f[k] for k in f.files}
    d["layout"] = d["layout"][::-1]
    np.savez(tmp_path / "bad.npz", **d)
    with pytest.raises(ValueError):
        load_checkpoint(tmp_path / "bad.npz")


def test_resume_from_a_checkpoint_matches_an_unbroken_run(tmp_path, oracle_mod):
    imgs, labs = crater.make_batch(6)
    straight = crater.init_params()
    for _ in range(3):
        oracle_mod.cnn_step(straight, imgs, labs, lr=0.05)
    first = crater.init_params()
    for _ in range(2):
        oracle_mod.cnn_step(first, imgs, labs, lr=0.05)
    save_checkpoint(tmp_path / "c.npz", first, 2, lr=0.05, batch_total=6)
    st = load_checkpoint(tmp_path / "c.npz")
    resumed = st["params"]
    for _ in range(3 - st["step"]):
        oracle_mod.cnn_step(resumed, imgs, labs, lr=st["lr"])
    np.testing.assert_array_equal(resumed, straight)
