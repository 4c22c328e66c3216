"""Specs from the reference compiler's HIR (remora_b200.reference_codegen),
without a GPU.

The fixture tests/golden/reference_programs.{json,npz} holds, per program,
the spec the codegen produced from the reference's front end, seeded inputs
and the reference interpreter's output.  Here: the codegen reproduces the
recorded specs (where the reference is importable), every recorded map or
fold program compiles for sm_100a with NVRTC, and the oracle run on the
recorded specs gives the interpreter's outputs, so each spec means what the
program says.  tests/test_gpu_reference_programs.py runs the same records on
the device."""

from __future__ import annotations

import ctypes
import json
import os
import sys

import numpy as np
import pytest

from conftest import REFERENCE, GOLDEN
from remora_b200 import _lib as L
from remora_b200.codegen import (AppendSpec, FoldSpec, MapSpec, RotateSpec, ScanSpec, SortSpec, meta_from_record,
                                 spec_from_record, spec_record)
from remora_b200.errors import RemoraUnsupportedError

REF = REFERENCE or ""
have_ref = REFERENCE is not None


def records():
    return json.loads((GOLDEN / "reference_programs.json").read_text())


def arrays():
    with np.load(GOLDEN / "reference_programs.npz") as f:
        return {k: f[k] for k in f.files}


def close(got: np.ndarray, want: np.ndarray) -> None:
    assert got.shape == want.shape and got.dtype == want.dtype
    if got.dtype == np.float32:
        # the interpreter computes scalar arithmetic in Python floats and folds
        # in f64; the compiled path rounds every f32 operation
        scale = float(np.abs(want).max()) if want.size else 0.0
        np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6 * scale)
    else:
        np.testing.assert_array_equal(got, want)


def oracle_run(orc, spec, meta, ins):
    if isinstance(spec, MapSpec):
        return orc.run_map(spec.program, ins, meta.output_shape, np.dtype(meta.output_dtype))
    if isinstance(spec, FoldSpec):
        if spec.spec.mode == L.FOLD_ALL:
            return orc.fold_all(spec.spec, ins)
        return orc.cell_fold(spec.spec, ins, spec.spec.cell_rank)
    if isinstance(spec, ScanSpec):
        return orc.scan(spec.spec, ins[0])
    if isinstance(spec, AppendSpec):
        return orc.append(ins[spec.left], ins[1 - spec.left])
    if isinstance(spec, RotateSpec):
        return orc.rotate(ins[0], spec.shift)
    if isinstance(spec, SortSpec):
        return orc.grade(ins[0]) if spec.grade else orc.sort(ins[0])
    raise AssertionError(type(spec))


def test_records_round_trip_and_cover_every_spec_kind():
    kinds = set()
    for rec in records():
        spec = spec_from_record(rec["spec"])
        assert spec_record(spec) == rec["spec"]
        meta = meta_from_record(rec["meta"])
        assert meta.name == rec["kernel"] and meta.num_inputs == rec["n_inputs"]
        kinds.add(rec["spec"]["kind"])
    assert kinds == {"map", "fold", "scan", "append", "rotate", "sort"}


def test_oracle_on_recorded_specs_gives_interpreter_outputs(oracle_mod):
    a = arrays()
    for rec in records():
        spec, meta = spec_from_record(rec["spec"]), meta_from_record(rec["meta"])
        ins = [a[f"{rec['name']}__in{k}"] for k in range(rec["n_inputs"])]
        got = np.asarray(oracle_run(oracle_mod, spec, meta, ins))
        want = a[f"{rec['name']}__out"]
        close(got.astype(want.dtype) if got.dtype != want.dtype and want.dtype == np.bool_ else got, want)


def test_recorded_programs_compile_for_sm100a():
    lib = L.lib()
    for rec in records():
        spec = spec_from_record(rec["spec"])
        if isinstance(spec, MapSpec):
            assert lib.remora_b200_jit_check(ctypes.byref(spec.program), -1, None, 0) == 0, L.last_error()
        elif isinstance(spec, FoldSpec) and spec.spec.has_premap:
            assert lib.remora_b200_jit_check(ctypes.byref(spec.spec.premap), spec.spec.op, None, 0) == 0, \
                L.last_error()


@pytest.mark.skipif(not have_ref, reason="the reference front end is not importable here")
def test_codegen_reproduces_recorded_specs():
    sys.path.insert(0, REF)
    sys.path.insert(0, str(GOLDEN))
    import make_reference_programs as mk

    from remora_b200.reference_codegen import compile_function_source_to_b200_artifacts

    by_name = {r["name"]: r for r in records()}
    for name, syntax, source, fn, params, _kind in mk.PROGRAMS:
        ptypes = tuple(mk.A(e, *d) for e, d in params)
        module, metas, _ = compile_function_source_to_b200_artifacts(
            source, fn, ptypes, include_prelude=False, kernel_name=f"remora_{name}", syntax=syntax)
        (kname, spec), = module.kernels.items()
        assert spec_record(spec) == by_name[name]["spec"], name
        assert metas[0] == meta_from_record(by_name[name]["meta"]), name


@pytest.mark.skipif(not have_ref, reason="the reference front end is not importable here")
@pytest.mark.parametrize("source,fn,params", [
    # fold with a non-literal initial value
    ("(define/pi () (f [x (Array Float 4) y (Array Float 4)] Float) (fold + (reduce + 0.0 y) x))", "f",
     [("f", (4,)), ("f", (4,))]),
    # a map over something other than the parameters
    ("(define/pi () (f [x (Array Float 4)] (Array Float 4)) (map (* 2.0) (reverse x)))", "f", [("f", (4,))]),
    # a fold of a rank-2 array (an array-valued accumulator)
    ("(define/pi () (f [x (Array Float 3 4)] (Array Float 4)) (fold + [0.0 0.0 0.0 0.0] x))", "f",
     [("f", (3, 4))]),
])
def test_unsupported_shapes_raise(source, fn, params):
    sys.path.insert(0, REF)
    sys.path.insert(0, str(GOLDEN))
    import make_reference_programs as mk

    from remora_b200.reference_codegen import compile_function_source_to_b200_artifacts

    ptypes = tuple(mk.A(e, *d) for e, d in params)
    try:
        compile_function_source_to_b200_artifacts(source, fn, ptypes, include_prelude=False, syntax="lisp")
    except RemoraUnsupportedError:
        return
    except Exception as exc:  # the reference's own front end rejected the program first
        pytest.skip(f"front end: {type(exc).__name__}")
    raise AssertionError("expected RemoraUnsupportedError")
