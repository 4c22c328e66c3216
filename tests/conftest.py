"""Shared test configuration.

Tests marked ``gpu`` need a B200 and the built library; everything else runs
on a CPU-only machine.  GPU tests fail (they do not skip) when no CUDA device
is present, so a run that was meant to exercise the device cannot pass
silently without it.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
for p in (str(ROOT), str(ROOT / "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def _reference() -> str | None:
    import oracle

    root = oracle.reference_root()
    return str(root) if root is not None else None


# The reference checkout for the tests that run its front end or read its
# sources (REMORA_REFERENCE, else where the oracle's build found it); None
# skips them.
REFERENCE = _reference()


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and libremora_b200.so")


def golden(name: str) -> dict[str, np.ndarray]:
    with np.load(GOLDEN / f"{name}.npz") as f:
        return {k: f[k] for k in f.files}


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        raise RuntimeError("GPU test run without a CUDA device")
    major, _ = torch.cuda.get_device_capability(0)
    if major != 10:
        raise RuntimeError(f"GPU tests need an sm_100 device, found sm_{major}x")
    return torch.device("cuda", 0)


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle as oracle_module

    oracle_module.lib()
    return oracle_module


def to_dev(a: np.ndarray, device):
    import torch

    return torch.from_numpy(np.array(a, copy=True, order="C")).to(device)


def to_host(t) -> np.ndarray:
    """Device-to-host copy after surfacing any device-side wait that ran out
    (remora_b200_synchronize raises RemoraTimeoutError)."""
    from remora_b200 import ops

    ops.synchronize(t.device.index)
    return t.detach().cpu().numpy()
