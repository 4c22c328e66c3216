"""Generate tests/golden/executor_traces.json: what the reference's own
executor asks of a runtime when it runs this backend's kernels.

For each known-answer case of the reference's GPU executor tests
(tests/test_executor.py:434-770 of the reference: scale, add, sum, dot, inc,
i32 add, rank-2 and rank-3 maps), plus a larger sum and a chained cell fold,
the kernel specs come from remora_b200.reference_codegen (the reference's
front end, then this backend's lowering), and the reference's RemoraExecutor
(remora/executor.py:17-143), imported unmodified, runs them over a
recording runtime: every call it makes (load_ptx, get_function, alloc,
copy_host_to_device, memset_d32, launch with its descriptor fields, synchronize,
copy_device_to_host, free) is written down with its arguments.  The GPU test
(tests/test_gpu_executor_trace.py) replays each call sequence through
B200Runtime, so the box needs neither the reference nor its front end, and
checks the result against the reference test's known answer.

    REMORA_REFERENCE=/path/to/remorac python tests/golden/make_executor_traces.py
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
OUT = HERE / "executor_traces.json"


def _reference() -> str:
    sys.path.insert(0, str(ROOT / "oracle"))
    from oracle import reference_root  # REMORA_REFERENCE, or where the oracle's build found it

    root = reference_root()
    if root is None:
        raise SystemExit("set REMORA_REFERENCE to the reference checkout (the directory holding remora/)")
    return str(root)


# (case, source, function, kernel name, [(elem, dims)], include_prelude,
#  inputs, known answer, call) -- inputs and answers are the reference
#  tests' literals; call is "main" (execute_main) or "name" (execute).
def cases() -> list[tuple]:
    f, i = "f", "i"
    v4 = [1, 2, 3, 4]
    w4 = [10, 20, 30, 40]
    m23 = [[1, 2, 3], [4, 5, 6]]
    t221 = [[[1], [2]], [[3], [4]]]
    big = np.random.Generator(np.random.PCG64(1729)).uniform(-1, 1, 1000).astype(np.float32)
    rng = np.random.Generator(np.random.PCG64(1730))
    x4 = rng.standard_normal((3, 4, 5, 16)).astype(np.float32)
    return [
        ("scale_by_name", "def scale xs = map (* 2.0) xs", "scale", "remora_scale", [(f, (4,))], True,
         [(v4, f)], ([2, 4, 6, 8], f), "name"),
        ("scale", "def scale xs = map (* 2.0) xs", "scale", "remora_scale", [(f, (4,))], True,
         [(v4, f)], ([2, 4, 6, 8], f), "main"),
        ("add", "def add xs ys = map (+) xs ys", "add", "remora_add", [(f, (4,)), (f, (4,))], True,
         [(v4, f), (w4, f)], ([11, 22, 33, 44], f), "main"),
        ("sum", "def sum xs = fold (+) 0.0 xs", "sum", "remora_sum", [(f, (4,))], False,
         [(v4, f)], (10, f), "main"),
        ("dot", "def dot xs ys = fold (+) 0.0 (map (*) xs ys)", "dot", "remora_dot", [(f, (4,)), (f, (4,))], False,
         [(v4, f), (w4, f)], (300, f), "main"),
        ("inc_i32", "def inc xs = map (+ 2) xs", "inc", "remora_inc", [(i, (4,))], False,
         [(v4, i)], ([3, 4, 5, 6], i), "main"),
        ("add_i32", "def add xs ys = map (+) xs ys", "add", "remora_add", [(i, (4,)), (i, (4,))], False,
         [(v4, i), (w4, i)], ([11, 22, 33, 44], i), "main"),
        ("scale_rank2", "def scale xs = map (* 2.0) xs", "scale", "remora_scale2d", [(f, (2, 3))], True,
         [(m23, f)], ([[2, 4, 6], [8, 10, 12]], f), "main"),
        ("add_rank2", "def add xs ys = map (+) xs ys", "add", "remora_add2d", [(f, (2, 3)), (f, (2, 3))], True,
         [(m23, f), ([[10, 20, 30], [40, 50, 60]], f)], ([[11, 22, 33], [44, 55, 66]], f), "main"),
        ("scale_rank3", "def scale xs = map (* 2.0) xs", "scale", "remora_scale3d", [(f, (2, 2, 1))], True,
         [(t221, f)], ([[[2], [4]], [[6], [8]]], f), "main"),
        ("add_rank3", "def add xs ys = map (+) xs ys", "add", "remora_add3d", [(f, (2, 2, 1)), (f, (2, 2, 1))], True,
         [(t221, f), ([[[10], [20]], [[30], [40]]], f)], ([[[11], [22]], [[33], [44]]], f), "main"),
        # beyond the reference's literals: answers from its interpreter
        ("sum_1000", "def sum xs = fold (+) 0.0 xs", "sum", "remora_sum", [(f, (1000,))], False,
         [(big, f)], None, "main"),
        ("chained_cell_fold",
         "def chained x = map (\\row -> fold (+) 0.0 (map (\\v -> if 0.5 < v * 2.5 + 1.0 then v * 2.5 + 1.0 "
         "else 0.0) row)) x",
         "chained", "remora_chained", [(f, (3, 4, 5, 16))], True, [(x4, f)], None, "main"),
    ]


class RecordingRuntime:
    """The runtime duck type RemoraExecutor drives (remora/runtime.py:243-412),
    writing down every call instead of touching a device."""

    def __init__(self) -> None:
        self.calls: list[dict] = []
        self.next = 1

    def load_ptx(self, module):
        self.calls.append({"op": "load_ptx"})
        return RecordingModule(self)

    def alloc(self, nbytes: int) -> int:
        ptr = self.next << 20
        self.next += 1
        self.calls.append({"op": "alloc", "nbytes": int(nbytes), "ret": ptr})
        return ptr

    def free(self, ptr: int) -> None:
        self.calls.append({"op": "free", "ptr": int(ptr)})

    def copy_host_to_device(self, host_array: np.ndarray, device_ptr: int) -> None:
        a = np.ascontiguousarray(host_array)
        self.calls.append({"op": "copy_host_to_device", "ptr": int(device_ptr), "dtype": a.dtype.name,
                           "shape": list(a.shape), "data": a.tobytes().hex()})

    def memset_d32(self, device_ptr: int, value: int, count: int) -> None:
        self.calls.append({"op": "memset_d32", "ptr": int(device_ptr), "value": int(value), "count": int(count)})

    def synchronize(self) -> None:
        self.calls.append({"op": "synchronize"})

    def copy_device_to_host(self, device_ptr: int, host_array: np.ndarray) -> None:
        self.calls.append({"op": "copy_device_to_host", "ptr": int(device_ptr), "dtype": host_array.dtype.name,
                           "shape": list(host_array.shape)})
        host_array[...] = 0

    def close(self) -> None:
        self.calls.append({"op": "close"})


class RecordingModule:
    def __init__(self, rt: RecordingRuntime) -> None:
        self.rt = rt

    def get_function(self, name: str):
        self.rt.calls.append({"op": "get_function", "name": name})
        return RecordingKernel(self.rt, name)

    def close(self) -> None:
        self.rt.calls.append({"op": "module_close"})


class RecordingKernel:
    def __init__(self, rt: RecordingRuntime, name: str) -> None:
        self.rt, self.name = rt, name

    def launch(self, grid, block, args, **kw) -> None:
        from remora_b200.abi import descriptor_rank

        descs = []
        for a in args:
            r = descriptor_rank(a)
            descs.append({"rank": r, "allocated": int(a.allocated or 0), "aligned": int(a.aligned or 0),
                          "offset": int(a.offset), "sizes": [int(getattr(a, f"size{d}")) for d in range(r)],
                          "strides": [int(getattr(a, f"stride{d}")) for d in range(r)]})
        self.rt.calls.append({"op": "launch", "name": self.name, "grid": list(grid), "block": list(block),
                              "args": descs, "kw": sorted(kw)})


def build_records(ref: str) -> list[dict]:
    """The traces, computed afresh with the reference at ``ref``."""
    sys.path.insert(0, ref)
    sys.path.insert(0, str(ROOT))
    from remora.executor import RemoraExecutor  # the reference's executor, unmodified
    from remora.parser import parse_program
    from remora.runtime import _lambda_callable
    from remora.typechecker import TypeChecker
    from remora.types import FLOAT, INT, ArrayType, FuncType, StaticDim

    from remora_b200.codegen import meta_record, spec_record
    from remora_b200.reference_codegen import compile_function_source_to_b200_artifacts

    def interpret(source: str, fn: str, ptypes, rtype, args):
        ch = TypeChecker()
        ch.check_program(parse_program(source))
        typed = ch._typed_top_level_function(ch._functions[fn], FuncType(tuple(ptypes), rtype),
                                             ch._build_prelude_env())
        return _lambda_callable(typed, {})(*args)

    elem = {"f": FLOAT, "i": INT}
    npt = {"f": np.float32, "i": np.int32}
    out = []
    for name, src, fn, kname, params, prelude, inputs, known, call in cases():
        ptypes = tuple(ArrayType(elem[e], tuple(StaticDim(d) for d in dims)) for e, dims in params)
        module, metas, hir = compile_function_source_to_b200_artifacts(src, fn, ptypes, include_prelude=prelude,
                                                                       kernel_name=kname)
        arrays = [np.asarray(v, dtype=npt[e]) for v, e in inputs]
        rt = RecordingRuntime()
        ex = RemoraExecutor(module, metas, runtime=rt)
        if call == "name":
            ex.execute(kname, arrays)
        else:
            ex.execute_main(arrays)
        ex.close()
        if known is not None:
            answer = np.asarray(known[0], dtype=npt[known[1]])
            kind = "known answer of the reference's test"
        else:
            got = interpret(src, fn, ptypes, hir.return_type, [np.array(a) for a in arrays])
            answer = np.asarray(got, dtype=np.float32).reshape(metas[0].output_shape or ())
            kind = "reference interpreter (Python-float arithmetic)"
        out.append({"case": name, "kernel": kname, "call": call,
                    "spec": {k: spec_record(s) for k, s in module.kernels.items()},
                    "metas": [meta_record(m) for m in metas], "trace": rt.calls,
                    "answer": {"dtype": answer.dtype.name, "shape": list(answer.shape),
                               "data": answer.tobytes().hex()},
                    "answer_kind": kind})
    return out


def main() -> None:
    out = build_records(_reference())
    for rec in out:
        print(rec["case"], [c["op"] for c in rec["trace"]])
    OUT.write_text(json.dumps(out, indent=1) + "\n")
    print(f"wrote {len(out)} traces to {OUT}")


if __name__ == "__main__":
    main()
