"""The allocation-free scan entry point, remora_b200_scan_noalloc.

It serves callers that cannot allocate device memory (their device memory is
owned by another allocator, or cudaMalloc's possible device synchronisation
is not acceptable on their path); its scratch is one fixed 1 MiB device
array.  Called through the C ABI, its results must match remora_b200_scan's
on the same inputs, on two calls in a row (the second call reuses the array
the first one left behind).  This file is collected last.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from remora_b200 import _lib as L
from remora_b200.abi import tensor_descriptor
from remora_b200.codegen import scan_spec
from remora_b200.errors import RemoraLimitError, RemoraUnsupportedError
from remora_b200.runtime import context

pytestmark = pytest.mark.gpu

MAX_RANK1 = 268_304_384  # elements a rank-1 scan may have with 1 MiB of scratch


def _scan(entry, spec, x, out):
    import torch

    xd, od = tensor_descriptor(x), tensor_descriptor(out)
    stream = ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)
    fn = getattr(L.lib(), entry)
    L.check(fn(context(x.device.index).ptr, ctypes.byref(spec), ctypes.addressof(xd), ctypes.addressof(od), x.dim(),
               stream), entry)
    L.check(L.lib().remora_b200_synchronize(context(x.device.index).ptr, stream), "synchronize")
    return out.cpu().numpy()


@pytest.mark.parametrize("case", ["f32_rank1", "i32_rank1_exclusive", "f32_right", "f32_rank2", "i32_rank3"])
def test_noalloc_scan_matches_scan_twice(cuda, case):
    import torch

    rng = np.random.default_rng(2024)
    shapes = {"f32_rank1": (3_000_017,), "i32_rank1_exclusive": (1_000_003,), "f32_right": (77_777,),
              "f32_rank2": (4096, 48), "i32_rank3": (513, 9, 7)}
    shape = shapes[case]
    if case.startswith("i32"):
        host = rng.integers(-1000, 1000, shape).astype(np.int32)
        spec = scan_spec(dtype="i32", init=5, exclusive=case.endswith("exclusive"))
    else:
        host = rng.uniform(-1, 1, shape).astype(np.float32)
        spec = scan_spec(init=0.25, right=case == "f32_right")
    x = torch.from_numpy(host).to(cuda)
    ref = _scan("remora_b200_scan", spec, x, torch.empty_like(x))
    for _ in range(2):
        got = _scan("remora_b200_scan_noalloc", spec, x, torch.empty_like(x))
        if host.dtype == np.int32 or len(shape) == 1:
            # integer scans are exact; rank-1 f32 scans use the same tiles
            np.testing.assert_array_equal(got, ref)
        else:
            # rank >= 2 uses fewer row segments here, so f32 sums reassociate
            mag = np.cumsum(np.abs(host.astype(np.float64)), axis=0) + 1.0
            assert np.all(np.abs(got.astype(np.float64) - ref) <= 1e-5 * np.abs(ref) + 2e-6 * mag)


def test_noalloc_scan_limits(cuda):
    import torch

    big = torch.zeros(MAX_RANK1 + 1, dtype=torch.float32, device=cuda)
    with pytest.raises(RemoraLimitError):
        _scan("remora_b200_scan_noalloc", scan_spec(), big, big)
    ok = big[:MAX_RANK1]
    out = _scan("remora_b200_scan_noalloc", scan_spec(), ok, torch.empty_like(ok))
    assert out[-1] == 0.0
    del big, ok
    x = torch.arange(40, dtype=torch.float32, device=cuda)
    with pytest.raises(RemoraUnsupportedError):
        _scan("remora_b200_scan_noalloc", scan_spec(), x[::2], torch.empty(20, device=cuda))
