"""Value and gradient of fold-of-elementwise losses (remora_b200.autodiff)
without a GPU: the symbolic derivative against central differences in f64,
and the recorded specs (tests/golden/reference_gradients.json, made from the
reference's front end) on the oracle against the reference's tape AD and,
for its three GPU cases, its closed forms (rtol 1e-5, the reference's own
tolerance, tests/test_ad_source.py:605)."""

from __future__ import annotations

import json
import math
import os
import sys

import numpy as np
import pytest

from conftest import REFERENCE, GOLDEN
from remora_b200 import _lib as L
from remora_b200.autodiff import derivative
from remora_b200.codegen import spec_from_record
from remora_b200.errors import RemoraUnsupportedError
from remora_b200.program import BinaryExpr, CmpExpr, ConstantExpr, InputExpr, SelectExpr, UnaryExpr


REF = REFERENCE or ""
needs_ref = pytest.mark.skipif(REFERENCE is None,
                               reason="the reference front end is not importable here")


def records():
    return json.loads((GOLDEN / "reference_gradients.json").read_text())


def arrays():
    with np.load(GOLDEN / "reference_gradients.npz") as f:
        return {k: f[k] for k in f.files}


def evaluate(e, xs):
    if isinstance(e, InputExpr):
        return xs[e.index]
    if isinstance(e, ConstantExpr):
        return float(e.value)
    if isinstance(e, BinaryExpr):
        a, b = evaluate(e.left, xs), evaluate(e.right, xs)
        return {"+": a + b, "-": a - b, "*": a * b, "/": a / b}[e.op]
    if isinstance(e, UnaryExpr):
        a = evaluate(e.operand, xs)
        return {"neg": lambda: -a, "exp": lambda: math.exp(a), "log": lambda: math.log(a),
                "sqrt": lambda: math.sqrt(a)}[e.op]()
    if isinstance(e, CmpExpr):
        a, b = evaluate(e.left, xs), evaluate(e.right, xs)
        return float({">": a > b, "<": a < b, ">=": a >= b, "<=": a <= b, "==": a == b, "!=": a != b}[e.op])
    if isinstance(e, SelectExpr):
        return evaluate(e.then_expr, xs) if evaluate(e.condition, xs) else evaluate(e.else_expr, xs)
    raise AssertionError(e)


X, Y = InputExpr(0), InputExpr(1)
EXPRS = [
    BinaryExpr("*", BinaryExpr("+", X, ConstantExpr(1.0)), BinaryExpr("-", X, ConstantExpr(2.0))),
    BinaryExpr("/", X, BinaryExpr("+", X, Y)),
    BinaryExpr("*", UnaryExpr("exp", BinaryExpr("*", X, Y)), UnaryExpr("log", Y)),
    SelectExpr(CmpExpr(">", X, Y), BinaryExpr("*", X, X), UnaryExpr("neg", UnaryExpr("sqrt", Y))),
    BinaryExpr("-", ConstantExpr(3.0), BinaryExpr("/", ConstantExpr(1.0), BinaryExpr("*", X, BinaryExpr("*", Y, Y)))),
]


@pytest.mark.parametrize("e", EXPRS)
def test_derivative_matches_central_differences(e):
    rng = np.random.default_rng(3)
    for _ in range(20):
        pt = [float(rng.uniform(0.3, 2.0)), float(rng.uniform(0.3, 2.0))]
        for k in (0, 1):
            h = 1e-6
            up, dn = list(pt), list(pt)
            up[k] += h
            dn[k] -= h
            fd = (evaluate(e, up) - evaluate(e, dn)) / (2 * h)
            assert evaluate(derivative(e, k), pt) == pytest.approx(fd, rel=1e-5, abs=1e-6)


def test_derivative_simplifies_constants():
    assert derivative(ConstantExpr(2.0), 0) == ConstantExpr(0.0)
    assert derivative(BinaryExpr("*", X, ConstantExpr(3.0)), 0) == ConstantExpr(3.0)
    assert derivative(BinaryExpr("+", X, Y), 1) == ConstantExpr(1.0)
    with pytest.raises(RemoraUnsupportedError):
        derivative("not an expression", 0)


def test_recorded_specs_on_the_oracle(oracle_mod):
    a = arrays()
    for rec in records():
        ins = [a[f"{rec['name']}__in{k}"] for k in range(rec["n_inputs"])]
        for kname, kr in rec["kernels"].items():
            spec = spec_from_record(kr["spec"])
            if kname.endswith("_value"):
                got = float(oracle_mod.fold_all(spec.spec, ins))
                want = float(a[f"{rec['name']}__value"])
                if not math.isnan(want):  # NaN: the interpreter cannot evaluate this loss
                    assert got == pytest.approx(want, rel=1e-5, abs=1e-6)
            else:
                k = 0 if kname.endswith("_grad_x") else 1
                got = oracle_mod.run_map(spec.program, ins, ins[0].shape, np.float32)
                np.testing.assert_allclose(got, a[f"{rec['name']}__grad{k}"], rtol=1e-5, atol=1e-6)
                if f"{rec['name']}__closed" in a and k == 0:
                    np.testing.assert_allclose(got, a[f"{rec['name']}__closed"], rtol=1e-5, atol=1e-6)
    assert {r["name"] for r in records()} >= {"polynomial", "cubic", "division"}
    assert L.F32 == 0


# ------------------------------------------------- value-and-grad plans
# tests/golden/value_and_grad_plans.{json,npz}: wider losses (scalar
# parameters, several folds, rank-2 and rank-3 arrays summed by maps of cell
# folds, scalars outside the folds) planned from the reference's front end,
# with the reference interpreter's value and the tape's gradients.
# Tolerances: elementwise gradients rtol 1e-5 + atol 1e-6·max|ref|; sums
# (the value and the gradients of scalar parameters) rtol 1e-4, since an f32
# fold of up to 65,536 terms, added in sequence as the reference's compiled
# path adds them, is 1.5e-5 from the f64 tape.
def plan_records():
    return json.loads((GOLDEN / "value_and_grad_plans.json").read_text())


def plan_arrays():
    with np.load(GOLDEN / "value_and_grad_plans.npz") as f:
        return {k: f[k] for k in f.files}


def check_value_and_grads(rec, got: list[np.ndarray]) -> None:
    a = plan_arrays()
    n = rec["name"]
    assert float(got[0]) == pytest.approx(float(a[f"{n}__value"]), rel=1e-4)
    for k, shape in enumerate(rec["shapes"]):
        g, want = np.asarray(got[k + 1], np.float64), a[f"{n}__grad{k}"]
        assert g.shape == want.shape
        if shape is None:
            assert float(g) == pytest.approx(float(want), rel=1e-4, abs=1e-6)
        elif "gemm" in rec["steps"]:
            # a batched layer's products run as 3xTF32 GEMMs on the device:
            # the 3xTF32 GEMM tolerance
            np.testing.assert_allclose(g, want, rtol=1e-4, atol=1e-4 * float(np.abs(want).max()))
        else:
            np.testing.assert_allclose(g, want, rtol=1e-5, atol=1e-6 * float(np.abs(want).max()))


@pytest.mark.parametrize("rec", plan_records(), ids=lambda r: r["name"])
def test_value_and_grad_plan_on_the_oracle(oracle_mod, rec):
    from remora_b200.program_plan import Plan
    from test_program_plan import run_plan_on_oracle

    a = plan_arrays()
    ins = [a[f"{rec['name']}__in{k}"] for k in range(len(rec["shapes"]))]
    plan = Plan.from_record(rec["plan"])
    assert plan.to_record() == rec["plan"]
    check_value_and_grads(rec, run_plan_on_oracle(oracle_mod, plan, ins, all_results=True))


def test_the_fixture_covers_scalars_ranks_and_several_folds():
    recs = {r["name"]: r for r in plan_records()}
    assert any(None in r["shapes"] for r in recs.values())
    assert {len(s) for r in recs.values() for s in r["shapes"] if s} == {1, 2, 3}
    assert recs["two_shapes"]["steps"].count("fold") == 2


def test_a_batched_layer_is_one_gemm_forward_and_two_backward():
    """Z = X W^T forward; dW = G^T X and dX = G W backward.  The reference's
    tape cannot trace these nested maps, so the fixture's gradients are the
    derivative's closed form (marked in the fixture); the value is the
    reference interpreter's."""
    recs = {r["name"]: r for r in plan_records()}
    a = plan_arrays()
    for name in ("batched_linear", "batched_relu"):
        assert recs[name]["steps"].count("gemm") == 3 and f"{name}__closed_form" in a
    # two layers: two GEMMs forward, four backward (dW2, dH, dW1, dX)
    assert recs["batched_mlp"]["steps"].count("gemm") == 6 and "batched_mlp__closed_form" in a


def test_a_linear_layer_backward_is_an_outer_product_and_a_transposed_product():
    """For loss = sum((W x - y)^2): the forward folds rows of W times x once;
    dL/dW is one map over stride-0 views of the adjoint and of x, dL/dx one
    cell fold over W's transposed view."""
    from remora_b200.program_plan import Plan

    rec = next(r for r in plan_records() if r["name"] == "linear_mse")
    plan = Plan.from_record(rec["plan"])
    w_grad, x_grad = plan.buffers[plan.results[1]], plan.buffers[plan.results[2]]
    assert w_grad.shape == (48, 32) and x_grad.shape == (32,)
    outer = next(s for s in plan.steps if s.get("out") == plan.results[1])
    assert outer["op"] == "map" and [plan.buffers[i].view[2] for i in outer["ins"]] == [(1, 0), (0, 1)]
    wt = next(s for s in plan.steps if s.get("out") == plan.results[2])
    assert wt["op"] == "fold" and plan.buffers[wt["ins"][0]].view[2] == (1, 32)


def test_the_reference_tape_drops_a_fold_init():
    """remora/ad.py:_trace_fold records sum(arr) as a fold's value, without
    its init: for log (fold + 1.0 (exp y)) its gradient is exp y / sum exp y
    where the mathematics give exp y / (1 + sum exp y).  The plan follows the
    mathematics (the fixture's expected gradient is the closed form)."""
    a = plan_arrays()
    y = a["log_init__in0"].astype(np.float64)
    e = np.exp(y)
    np.testing.assert_allclose(a["log_init__tape_grad0"], e / e.sum(), rtol=1e-12)
    np.testing.assert_allclose(a["log_init__grad0"], e / (1.0 + e.sum()), rtol=1e-12)


@needs_ref
def test_planner_reproduces_recorded_value_and_grad_plans():
    sys.path.insert(0, REF)
    from remora.types import FLOAT, ArrayType, StaticDim

    from remora_b200.autodiff import compile_value_and_grad_plan_source

    for rec in plan_records():
        ptypes = tuple(FLOAT if s is None else ArrayType(FLOAT, tuple(StaticDim(d) for d in s))
                       for s in rec["shapes"])
        if rec["source"] is None:
            # the reference's own model source, read from its tree
            sys.path.insert(0, str(GOLDEN))
            from make_reference_gradients import crater_example

            src = crater_example()._CNN_FULL_LISP_SRC
        else:
            src = rec["source"]
        plan = compile_value_and_grad_plan_source(src, rec.get("function", "loss"), ptypes,
                                                  include_prelude=rec.get("include_prelude", True),
                                                  syntax=rec.get("syntax", "lisp"))
        assert plan.to_record() == rec["plan"], rec["name"]


def test_the_reference_crater_model_is_one_value_and_grad_plan():
    """The reference trains its crater CNN through six gradient functions,
    each compiled and run on its own (examples/crater_train.py:169-198).
    Here its loss (cnn-loss, examples/crater_train.py:29-59) is one plan:
    im2col once, the forward, then one backward that reaches every
    parameter, the kernel through the patch matrix's transpose and the image
    through col2im.  Its value and nine gradients are checked against the
    reference interpreter and tape by test_value_and_grad_plan_on_the_oracle
    and, on the device, by test_gpu_autodiff."""
    from remora_b200.program_plan import Plan

    rec = next(r for r in plan_records() if r["name"] == "crater_cnn")
    plan = Plan.from_record(rec["plan"])
    steps = rec["steps"]
    assert steps.count("im2col") == 1 and steps.count("col2im") == 1
    assert steps.index("im2col") == 0 and len(plan.results) == 1 + 9
    shapes = [plan.buffers[r].shape for r in plan.results]
    assert shapes == [(), (3, 3), (), (4, 900), (4,), (4,), (), (900,), (32, 32), ()]
    a = plan_arrays()
    assert float(a["crater_cnn__value"]) > 0.0 and "crater_cnn__closed_form" not in a


@needs_ref
@pytest.mark.parametrize("src, shapes", [
    # an array parameter outside the folds
    ("(define/pi () (loss [x (Array Float 4)] Float) (+ (fold + 0.0 x) (index x 0)))", [(4,)]),
    # a product fold
    ("(define/pi () (loss [x (Array Float 4)] Float) (fold * 1.0 x))", [(4,)]),
    # int parameters
    ("(define/pi () (loss [x (Array Int 4)] Int) (fold + 0 x))", ["int"]),
    # no fold at all
    ("(define/pi () (loss [w Float] Float) (* w w))", [None]),
])
def test_unsupported_losses_raise(src, shapes):
    sys.path.insert(0, REF)
    from remora.types import FLOAT, INT, ArrayType, StaticDim

    from remora_b200.autodiff import compile_value_and_grad_plan_source

    ptypes = tuple(FLOAT if s is None else ArrayType(INT, (StaticDim(4),)) if s == "int"
                   else ArrayType(FLOAT, tuple(StaticDim(d) for d in s)) for s in shapes)
    try:
        compile_value_and_grad_plan_source(src, "loss", ptypes)
    except RemoraUnsupportedError:
        return
    except Exception as exc:  # the reference's own front end rejected it first
        pytest.skip(f"front end: {type(exc).__name__}")
    raise AssertionError("expected RemoraUnsupportedError")


def test_plan_inputs_are_checked_against_the_plan():
    from remora_b200.errors import RemoraShapeError
    from remora_b200.program_plan import Plan, _check_inputs

    rec = next(r for r in plan_records() if r["name"] == "linreg")
    plan = Plan.from_record(rec["plan"])
    good = [np.float32(1.0), np.float32(0.0), np.zeros(256, np.float32), np.zeros(256, np.float32)]
    assert [a.shape for a in _check_inputs(plan, good)] == [(), (), (256,), (256,)]
    with pytest.raises(RemoraShapeError):
        _check_inputs(plan, good[:3])
    with pytest.raises(RemoraShapeError):
        _check_inputs(plan, [*good[:3], np.zeros(255, np.float32)])


@needs_ref
def test_losses_written_with_the_preludes_sum_and_dot(oracle_mod):
    """``sum`` and ``dot`` reach the loss as the front end's lets; the plan
    reads through them: loss = sum (x * y) + dot x x / 2, so dL/dx = y + x
    and dL/dy = x."""
    sys.path.insert(0, REF)
    from remora.types import FLOAT, ArrayType, StaticDim

    from remora_b200.autodiff import compile_value_and_grad_plan_source
    from remora_b200.program_plan import Plan
    from test_program_plan import run_plan_on_oracle

    vec = ArrayType(FLOAT, (StaticDim(50),))
    plan = compile_value_and_grad_plan_source("def loss x y = sum (map (*) x y) + dot x x / 2.0", "loss",
                                              (vec, vec), syntax="ml")
    rng = np.random.default_rng(9)
    x, y = (rng.standard_normal(50).astype(np.float32) for _ in range(2))
    value, gx, gy = run_plan_on_oracle(oracle_mod, Plan.from_record(plan.to_record()), [x, y], all_results=True)
    xd, yd = x.astype(np.float64), y.astype(np.float64)
    assert float(value) == pytest.approx(float((xd * yd).sum() + (xd * xd).sum() / 2), rel=1e-5)
    np.testing.assert_allclose(gx, yd + xd, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(gy, xd, rtol=1e-5, atol=1e-6)
