"""Host checks of tests/golden/executor_traces.json, the call sequences the
reference's unmodified RemoraExecutor (remora/executor.py:17-143) makes on
this backend's kernel specs (replayed on the device by
tests/test_gpu_executor_trace.py).  Where the reference is at hand
(conftest.REFERENCE), the traces are recomputed and must equal the
fixture."""

from __future__ import annotations

import json
import sys

import pytest

from conftest import GOLDEN, REFERENCE

TRACES = json.loads((GOLDEN / "executor_traces.json").read_text())


def test_traces_cover_the_reference_known_answers():
    names = {r["case"] for r in TRACES}
    assert {"scale", "add", "sum", "dot", "inc_i32", "add_i32", "scale_rank2", "add_rank2", "scale_rank3",
            "add_rank3"} <= names
    for rec in TRACES:
        ops = [c["op"] for c in rec["trace"]]
        allocated: set[int] = set()
        for c in rec["trace"]:
            if c["op"] == "alloc":
                allocated.add(c["ret"])
            elif c["op"] in ("copy_host_to_device", "memset_d32", "copy_device_to_host"):
                assert c["ptr"] in allocated
            elif c["op"] == "launch":
                assert all(d["aligned"] in allocated for d in c["args"])
            elif c["op"] == "free":
                allocated.remove(c["ptr"])
        assert not allocated, rec["case"]
        assert ops.index("launch") < ops.index("copy_device_to_host")
        # the reduction branch zeroes the output before the launch
        if rec["metas"][0]["is_reduction"]:
            assert ops.index("memset_d32") < ops.index("launch")
        else:
            assert "memset_d32" not in ops


@pytest.mark.skipif(REFERENCE is None, reason="the reference checkout is not at hand")
def test_traces_are_what_the_unmodified_executor_does():
    sys.path.insert(0, str(GOLDEN))
    from make_executor_traces import build_records

    assert build_records(REFERENCE) == TRACES
