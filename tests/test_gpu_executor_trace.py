"""The reference's own executor on this backend, on the device.

tests/golden/executor_traces.json holds, for each known-answer case of the
reference's GPU executor tests (tests/test_executor.py:434-770 of the
reference) and two larger cases, every runtime call that the reference's
unmodified RemoraExecutor (remora/executor.py:17-143) made when it ran this
backend's kernel specs (recorded by tests/golden/make_executor_traces.py).
Here each call sequence is replayed, call for call and argument for
argument, through B200Runtime: load_ptx of the spec module, get_function,
alloc, copy_host_to_device, memset_d32 (the is_reduction branch of
remora/executor.py:73-76), launch with descriptors carrying the recorded
sizes, strides and offsets, synchronize, copy_device_to_host, free.  The
result must equal the reference test's known answer bit for bit (maps and
small sums), or the reference interpreter's value at the f32 fold tolerance.
"""

from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import GOLDEN
from remora_b200.abi import make_memref_descriptor
from remora_b200.codegen import SpecModule, meta_from_record, spec_from_record
from remora_b200.runtime import B200Runtime

pytestmark = pytest.mark.gpu

TRACES = json.loads((GOLDEN / "executor_traces.json").read_text())


def replay(rec: dict) -> tuple[np.ndarray, list[str]]:
    """Run one recorded call sequence through B200Runtime; returns the array
    the last copy_device_to_host filled and the ops replayed."""
    metas = {m["name"]: meta_from_record(m) for m in rec["metas"]}
    module_specs = SpecModule({k: spec_from_record(v) for k, v in rec["spec"].items()})
    rt = B200Runtime()
    module = None
    kernels: dict = {}
    ptr: dict[int, int] = {}
    result = None
    ops = []
    for call in rec["trace"]:
        op = call["op"]
        ops.append(op)
        if op == "load_ptx":
            module = rt.load_ptx(module_specs)
        elif op == "get_function":
            kernels[call["name"]] = module.get_function(call["name"])
        elif op == "alloc":
            ptr[call["ret"]] = rt.alloc(call["nbytes"])
        elif op == "copy_host_to_device":
            a = np.frombuffer(bytes.fromhex(call["data"]), dtype=call["dtype"]).reshape(call["shape"])
            rt.copy_host_to_device(a, ptr[call["ptr"]])
        elif op == "memset_d32":
            rt.memset_d32(ptr[call["ptr"]], call["value"], call["count"])
        elif op == "launch":
            descs = []
            for d in call["args"]:
                base = ptr[d["aligned"]]
                assert d["allocated"] == d["aligned"]
                descs.append(make_memref_descriptor(base, d["sizes"], d["strides"], offset=d["offset"]))
            kernels[call["name"]].launch(tuple(call["grid"]), tuple(call["block"]), descs)
        elif op == "synchronize":
            rt.synchronize()
        elif op == "copy_device_to_host":
            result = np.empty(call["shape"], dtype=call["dtype"])
            rt.copy_device_to_host(ptr[call["ptr"]], result)
        elif op == "free":
            rt.free(ptr.pop(call["ptr"]))
        elif op == "module_close":
            module.close()
        elif op == "close":
            rt.close()
        else:
            raise AssertionError(f"unknown recorded call {op}")
    assert not ptr, "every allocation is freed"
    assert set(kernels) <= set(metas)
    return result, ops


@pytest.mark.parametrize("rec", TRACES, ids=lambda r: r["case"])
def test_reference_executor_call_sequence_on_device(cuda, rec):
    got, ops = replay(rec)
    ans = rec["answer"]
    want = np.frombuffer(bytes.fromhex(ans["data"]), dtype=ans["dtype"]).reshape(ans["shape"])
    assert got.dtype == want.dtype and got.shape == want.shape
    if rec["answer_kind"].startswith("known answer"):
        np.testing.assert_array_equal(got, want)
    else:
        np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6 * max(1.0, float(np.abs(want).max())))
    if rec["metas"][0]["is_reduction"]:
        assert "memset_d32" in ops
