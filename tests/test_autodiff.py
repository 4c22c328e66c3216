"""Value and gradient of fold-of-elementwise losses (remora_b200.autodiff)
without a GPU: the symbolic derivative against central differences in f64,
and the recorded specs (tests/golden/reference_gradients.json, made from the
reference's front end) on the oracle against the reference's tape AD and,
for its three GPU cases, its closed forms (rtol 1e-5, the reference's own
tolerance, remora/tests/test_ad_source.py:605)."""

from __future__ import annotations

import json
import math

import numpy as np
import pytest

from conftest import GOLDEN
from remora_b200 import _lib as L
from remora_b200.autodiff import derivative
from remora_b200.codegen import spec_from_record
from remora_b200.errors import RemoraUnsupportedError
from remora_b200.program import BinaryExpr, CmpExpr, ConstantExpr, InputExpr, SelectExpr, UnaryExpr


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
