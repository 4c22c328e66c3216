"""Whole-program plans (remora_b200.program_plan) without a GPU.

tests/golden/program_plans.{json,npz} holds the reference's acceptance
programs (tests/acceptance/pass/*.remora) and a few more, planned from
the reference front end's HIR, with the reference's result for each.  Here a
CPU interpreter of plans, built on the oracle, runs every recorded plan and
must give those results: the plan means what the program says.  Where the
reference is importable, the planner must reproduce the recorded plans.
tests/test_gpu_program_plan.py runs the same plans on the device."""

from __future__ import annotations

import json
import os
import sys

import numpy as np
import pytest

from conftest import REFERENCE, GOLDEN
from remora_b200 import _lib as L
from remora_b200.program_plan import Plan

REF = REFERENCE or ""
have_ref = REFERENCE is not None
_NP = {0: np.float32, 1: np.int32, 2: np.bool_}


def programs() -> list[dict]:
    return json.loads((GOLDEN / "program_plans.json").read_text())["programs"]


def expected(name: str) -> np.ndarray:
    with np.load(GOLDEN / "program_plans.npz") as f:
        return f[f"{name}__out"]


def close(got: np.ndarray, want: np.ndarray) -> None:
    assert got.shape == want.shape and got.dtype == want.dtype, (got.shape, want.shape, got.dtype, want.dtype)
    if got.dtype == np.float32:
        np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6 * (float(np.abs(want).max()) if want.size else 0))
    else:
        np.testing.assert_array_equal(got, want)


def run_plan_on_oracle(orc, plan: Plan, inputs: list[np.ndarray] | None = None, *, all_results: bool = False):
    """The plan's steps, each on the oracle, over numpy buffers: its result,
    or with ``all_results`` the list of ``plan.results``."""
    store: dict[int, np.ndarray] = {}
    for i, b in enumerate(plan.buffers):
        if b.input is not None:
            store[i] = np.ascontiguousarray(inputs[b.input], dtype=_NP[b.dtype]).reshape(b.shape)

    def get(i: int) -> np.ndarray:
        b = plan.buffers[i]
        if b.view is not None:
            base, off, st = b.view
            arr = get(base)
            es = arr.itemsize
            return np.ndarray(b.shape, dtype=arr.dtype, buffer=arr, offset=off * es, strides=[s * es for s in st])
        if i not in store:
            store[i] = (np.array(b.const, dtype=_NP[b.dtype]) if b.const is not None
                        else np.zeros(b.shape, dtype=_NP[b.dtype]))
        return store[i]

    for s in plan.steps:
        op = s["op"]
        if op == "map":
            out = plan.buffers[s["out"]]
            store[s["out"]] = orc.run_map(s["program"], [get(i) for i in s["ins"]], out.shape, _NP[out.dtype])
        elif op == "fold":
            sp = s["spec"]
            ins = [np.ascontiguousarray(get(i)) for i in s["ins"]]
            store[s["out"]] = (orc.fold_all(sp, ins) if sp.mode == L.FOLD_ALL
                               else orc.cell_fold(sp, ins, sp.cell_rank))
        elif op == "array_fold":
            store[s["out"]] = orc.array_fold(s["spec"], np.ascontiguousarray(get(s["in"])),
                                             np.ascontiguousarray(get(s["init"])))
        elif op == "scan":
            store[s["out"]] = orc.scan(s["spec"], np.ascontiguousarray(get(s["in"])))
        elif op == "append":
            store[s["out"]] = orc.append(get(s["a"]), get(s["b"]))
        elif op == "rotate":
            store[s["out"]] = orc.rotate(get(s["in"]), int(s["shift"]))
        elif op == "sort":
            store[s["out"]] = orc.sort(get(s["in"]))
        elif op == "grade":
            store[s["out"]] = orc.grade(get(s["in"]))
        elif op == "gemm":
            store[s["out"]] = orc.matmul(get(s["a"]), get(s["b"]))
        elif op == "im2col":
            store[s["out"]] = orc.im2col(get(s["in"]), s["kh"], s["kw"], s["stride"])
        elif op == "col2im":
            h, w = plan.buffers[s["out"]].shape
            store[s["out"]] = orc.col2im(np.ascontiguousarray(get(s["in"])), h, w, s["kh"], s["kw"], s["stride"])
        else:
            raise AssertionError(op)
    def result(r: int) -> np.ndarray:
        res = plan.buffers[r]
        return np.asarray(get(r)).astype(_NP[res.dtype]).reshape(res.shape)

    if all_results:
        return [result(r) for r in (plan.results or [plan.result])]
    return result(plan.result)


def test_fixture_covers_the_acceptance_programs():
    progs = programs()
    names = {p["name"] for p in progs}
    # 44 of the reference's 45 acceptance programs (one does not pass the
    # reference's own front end) and 11 more
    assert len(names) == 55
    ops = {op for p in progs for op in p["steps"]}
    assert ops == {"map", "fold", "array_fold", "scan", "append", "rotate", "sort", "grade"}
    for p in progs:
        plan = Plan.from_record(p["plan"])
        assert plan.to_record() == p["plan"]


@pytest.mark.parametrize("rec", programs(), ids=lambda r: r["name"])
def test_plan_on_the_oracle_gives_the_reference_value(oracle_mod, rec):
    close(run_plan_on_oracle(oracle_mod, Plan.from_record(rec["plan"])), expected(rec["name"]))


@pytest.mark.skipif(not have_ref, reason="the reference front end is not importable here")
def test_planner_reproduces_recorded_plans():
    sys.path.insert(0, REF)
    from remora_b200.program_plan import compile_source_to_plan

    for rec in programs():
        plan = compile_source_to_plan(rec["source"], syntax=rec["syntax"])
        assert plan.to_record() == rec["plan"], rec["name"]


@pytest.mark.skipif(not have_ref, reason="the reference front end is not importable here")
@pytest.mark.parametrize("source", [
    "let xs = [[1, 2], [3, 4]] in\nmap (\\row -> row[0 + 1 * 0] * row) xs",  # a whole cell in a scalar body
    "let xs = [[1, 2], [3, 4]] in\nmap (\\row -> row[0:1]) xs",             # a cell slice
    "fold (\\acc x -> acc * x + 1) 1 (iota 5)",                            # a fold step other than acc op x
])
def test_unsupported_programs_raise(source):
    sys.path.insert(0, REF)
    from remora_b200.errors import RemoraUnsupportedError
    from remora_b200.program_plan import compile_source_to_plan

    try:
        compile_source_to_plan(source)
    except RemoraUnsupportedError:
        return
    except Exception as exc:  # the reference's own front end rejected it first
        pytest.skip(f"front end: {type(exc).__name__}")
    raise AssertionError("expected RemoraUnsupportedError")


# ------------------------------------------------------- function plans
# tests/golden/function_plans.{json,npz}: functions with parameters (arrays
# and scalars) that no single kernel computes, planned by plan_from_function
# from the reference's function front end; seeded inputs and the
# interpreter's outputs.
def function_records() -> list[dict]:
    return json.loads((GOLDEN / "function_plans.json").read_text())


def function_io(rec: dict) -> tuple[list[np.ndarray], np.ndarray]:
    with np.load(GOLDEN / "function_plans.npz") as f:
        return [f[f"{rec['name']}__in{k}"] for k in range(len(rec["params"]))], f[f"{rec['name']}__out"]


def close_for(rec: dict, got: np.ndarray, want: np.ndarray) -> None:
    """A plan with a GEMM step runs it in 3xTF32 on the device, checked at the
    3xTF32 GEMM tolerance (rtol 1e-4 + atol 1e-4·max|ref|); every other plan
    at the f32 one."""
    if "gemm" in rec["steps"]:
        np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4 * float(np.abs(want).max()))
    else:
        close(got, want)


@pytest.mark.parametrize("rec", function_records(), ids=lambda r: r["name"])
def test_function_plan_on_the_oracle_gives_the_interpreter_value(oracle_mod, rec):
    ins, want = function_io(rec)
    plan = Plan.from_record(rec["plan"])
    assert plan.to_record() == rec["plan"]
    assert [b.input for b in plan.buffers if b.input is not None] == list(range(len(rec["params"])))
    close(run_plan_on_oracle(oracle_mod, plan, ins), want)


@pytest.mark.skipif(not have_ref, reason="the reference front end is not importable here")
@pytest.mark.parametrize("name, with_dot", [
    ("matvec", "def mv m v = map (\\row -> dot row v) m"),
    ("matmul_rows", "def mm a bt = map (\\r -> map (\\c -> dot r c) bt) a"),
])
def test_the_preludes_dot_plans_like_its_inlined_form(name, with_dot):
    """``dot`` reaches the planner as the front end's chain of lets over
    ``sum (map (*) a b)``; it must give the same plan as the inlined fold."""
    sys.path.insert(0, REF)
    from remora.types import FLOAT, ArrayType, StaticDim

    from remora_b200.program_plan import compile_function_source_to_plan

    rec = next(r for r in function_records() if r["name"] == name)
    ptypes = tuple(ArrayType(FLOAT, tuple(StaticDim(x) for x in d)) for _, d in rec["params"])
    plan = compile_function_source_to_plan(with_dot, rec["function"], ptypes)
    assert plan.to_record() == rec["plan"]


def test_a_fold_of_a_mapped_row_is_one_fused_fold():
    recs = {r["name"]: r for r in function_records()}
    for name in ("row_sumsq", "chained_rows"):
        plan = Plan.from_record(recs[name]["plan"])
        (step,) = plan.steps
        assert step["op"] == "fold" and step["spec"].has_premap and step["spec"].cell_rank == 1


def test_lifted_dots_become_one_fold_or_one_gemm():
    recs = {r["name"]: r for r in function_records()}
    assert recs["matvec"]["steps"] == ["fold"] and recs["matmul_rows"]["steps"] == ["gemm"]
    plan = Plan.from_record(recs["matvec"]["plan"])
    (step,) = plan.steps
    vec = plan.buffers[step["ins"][1]]
    assert vec.view is not None and vec.view[2][0] == 0  # the vector, repeated for every row
    plan = Plan.from_record(recs["matmul_transpose"]["plan"])
    (step,) = plan.steps
    assert plan.buffers[step["b"]].shape == (20, 17)


def test_a_fold_with_a_runtime_init_folds_from_the_identity():
    rec = next(r for r in function_records() if r["name"] == "fold_init_param")
    plan = Plan.from_record(rec["plan"])
    fold, combine = plan.steps
    assert fold["op"] == "fold" and fold["spec"].init_f == 0.0 and combine["op"] == "map"
    assert plan.buffers[combine["ins"][0]].input == 0  # the init parameter, then the sum


@pytest.mark.skipif(not have_ref, reason="the reference front end is not importable here")
def test_planner_reproduces_recorded_function_plans():
    sys.path.insert(0, REF)
    from remora.types import BOOL, FLOAT, INT, ArrayType, StaticDim

    from remora_b200.program_plan import compile_function_source_to_plan

    elem = {"f": FLOAT, "i": INT, "b": BOOL}
    for rec in function_records():
        ptypes = tuple(elem[e] if d is None else ArrayType(elem[e], tuple(StaticDim(x) for x in d))
                       for e, d in rec["params"])
        plan = compile_function_source_to_plan(rec["source"], rec["function"], ptypes, syntax=rec["syntax"])
        assert plan.to_record() == rec["plan"], rec["name"]


@pytest.mark.skipif(not have_ref, reason="the reference front end is not importable here")
def test_prelude_functions_inside_cell_maps_plan_like_written_out_folds(oracle_mod):
    """The front end inlines ``sum`` and ``dot`` as chains of lets; after
    let inlining they plan exactly like the folds written out."""
    sys.path.insert(0, REF)
    from remora.types import FLOAT, ArrayType, StaticDim

    from remora_b200.program_plan import compile_function_source_to_plan

    rec = next(r for r in function_records() if r["name"] == "row_sumsq")
    ptypes = (ArrayType(FLOAT, tuple(StaticDim(d) for d in rec["params"][0][1])),)
    assert compile_function_source_to_plan("def rn x = map (\\row -> dot row row) x", "rn",
                                           ptypes).to_record() == rec["plan"]
    summed = compile_function_source_to_plan("def rs x = map (\\row -> sum row) x", "rs", ptypes)
    written = compile_function_source_to_plan("def rs x = map (\\row -> fold (+) 0.0 row) x", "rs", ptypes)
    assert summed.to_record() == written.to_record()
    x = np.random.default_rng(3).standard_normal(rec["params"][0][1]).astype(np.float32)
    close(run_plan_on_oracle(oracle_mod, summed, [x]), x.astype(np.float64).sum(axis=1).astype(np.float32))


@pytest.mark.skipif(not have_ref, reason="the reference front end is not importable here")
def test_let_inlining_keeps_a_let_that_a_lambda_would_capture(oracle_mod):
    """In ``let t = s in map (\\s -> s * t) v`` substituting t := s would
    make the lambda's own s the factor; the let stays and t is the outer s."""
    sys.path.insert(0, REF)
    from remora.types import FLOAT, ArrayType, StaticDim

    from remora_b200.program_plan import compile_function_source_to_plan

    plan = compile_function_source_to_plan("def f s v = let t = s in map (\\s -> s * t) v", "f",
                                           (FLOAT, ArrayType(FLOAT, (StaticDim(3),))))
    got = run_plan_on_oracle(oracle_mod, plan, [np.float32(2.0), np.array([1.0, 2.0, 3.0], np.float32)])
    np.testing.assert_array_equal(got, np.array([2.0, 4.0, 6.0], np.float32))


@pytest.mark.skipif(not have_ref, reason="the reference front end is not importable here")
@pytest.mark.parametrize("source, fn, shapes", [
    # an integer lifted dot: not the f32 dense core, and not a fold of the cell alone
    ("def f m v = map (\\row -> fold (+) 0 (map (*) row v)) m", "f", [("i", (4, 3)), ("i", (3,))]),
    # a product of row times vector: not a dot
    ("def f m v = map (\\row -> fold (*) 1.0 (map (*) row v)) m", "f", [("f", (4, 3)), ("f", (3,))]),
    # a map over the cell that reads a scalar parameter
    ("def f s m = map (\\row -> fold (+) 0.0 (map (\\x -> x * s) row)) m", "f", [("f", None), ("f", (4, 3))]),
    # a fold step other than acc op x inside a cell map
    ("def f m = map (\\row -> fold (\\acc x -> acc * x + 1.0) 1.0 row) m", "f", [("f", (4, 3))]),
])
def test_near_miss_function_forms_raise(source, fn, shapes):
    sys.path.insert(0, REF)
    from remora.types import FLOAT, INT, ArrayType, StaticDim

    from remora_b200.errors import RemoraUnsupportedError
    from remora_b200.program_plan import compile_function_source_to_plan

    from remora.compiler import compile_function_source
    from remora_b200.program_plan import plan_from_function

    elem = {"f": FLOAT, "i": INT}
    ptypes = tuple(elem[e] if d is None else ArrayType(elem[e], tuple(StaticDim(x) for x in d)) for e, d in shapes)
    # the reference's front end alone first: only its own rejection skips
    try:
        artifact = compile_function_source(source, fn, ptypes, verify=False, include_prelude=True, syntax="ml")
    except Exception as exc:
        pytest.skip(f"front end: {type(exc).__name__}")
    # the planner on the HIR it returned must refuse with exactly this error
    with pytest.raises(RemoraUnsupportedError):
        plan_from_function(artifact.hir_function)


@pytest.mark.skipif(not have_ref, reason="the reference front end is not importable here")
def test_a_let_read_once_inside_a_lambda_stays_one_array(oracle_mod):
    """``let r = map (*) v v`` read once inside a cell map's lambda is not
    substituted into the lambda (that would make the vector product part of
    the per-row body): the plan computes r once, then one fused fold."""
    sys.path.insert(0, REF)
    from remora.types import FLOAT, ArrayType, StaticDim

    from remora_b200.program_plan import compile_function_source_to_plan

    src = "def f v m = let r = map (*) v v in map (\\row -> fold (+) 0.0 (map (*) row r)) m"
    plan = compile_function_source_to_plan(src, "f", (ArrayType(FLOAT, (StaticDim(3),)),
                                                      ArrayType(FLOAT, (StaticDim(4), StaticDim(3)))))
    assert [st["op"] for st in plan.steps] == ["map", "fold"]
    v = np.array([1.0, 2.0, 3.0], np.float32)
    m = np.arange(12, dtype=np.float32).reshape(4, 3)
    got = run_plan_on_oracle(oracle_mod, plan, [v, m])
    np.testing.assert_allclose(got, (m * (v * v)).sum(axis=1), rtol=1e-6)
