"""Generate tests/golden/reference_gradients.{json,npz}: losses
``fold + lit (elementwise expression)`` compiled by the reference's front
end and lowered by remora_b200.autodiff to a value fold and one gradient map
per parameter; expected values and gradients from the reference's tape AD
(remora/ad.py:trace_via_tape_multi).  Also tests/golden/
value_and_grad_plans.{json,npz}: wider losses (scalar parameters, several
folds, rank-2 and rank-3 arrays) as value-and-grad plans, with the
interpreter's value and the tape's gradients.  The first three losses and their
closed-form gradients are the reference's own GPU gradient tests
(tests/test_ad_source.py:569-605).  Regenerate with:

    REMORA_REFERENCE=/path/to/remorac python tests/golden/make_reference_gradients.py
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(Path(__file__).resolve().parents[2] / "oracle"))
from oracle import reference_root  # noqa: E402  (REMORA_REFERENCE, or where the oracle's build found it)

if reference_root() is None:
    raise SystemExit("set REMORA_REFERENCE to the reference checkout (the directory holding remora/)")
REF = str(reference_root())
sys.path.insert(0, REF)
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(HERE))

from make_golden import specialise  # noqa: E402
from remora.ad import trace_via_tape_multi  # noqa: E402
from remora.runtime import _lambda_callable  # noqa: E402
from remora.types import FLOAT, ArrayType, StaticDim  # noqa: E402

from remora_b200.autodiff import compile_value_and_grad_source  # noqa: E402
from remora_b200.codegen import meta_record, spec_record  # noqa: E402

N = 8
VEC = ArrayType(FLOAT, (StaticDim(N),))
LOSSES = [
    ("polynomial", "(define/pi () (loss [x (Array Float 8)] Float) (fold + 0.0 (* (+ x 1.0) (- x 2.0))))", 1),
    ("cubic", "(define/pi () (loss [x (Array Float 8)] Float) (fold + 0.0 (* (* x x) x)))", 1),
    ("division", "(define/pi () (loss [x (Array Float 8)] Float) (fold + 0.0 (/ x (+ x 1.0))))", 1),
    ("exp_two_inputs", "(define/pi () (loss [x (Array Float 8) y (Array Float 8)] Float) "
                       "(fold + 0.5 (* (exp x) (- y (* x y)))))", 2),
    ("log_select", "(define/pi () (loss [x (Array Float 8)] Float) "
                   "(fold + 0.0 (map (lambda (v) (select (> v 1.0) (log v) (* v v))) x)))", 1),
]


# Losses for the value-and-grad plans (autodiff.value_and_grad_plan_from_hir):
# scalar parameters, several folds, arrays of rank 2 and 3 summed by maps of
# cell folds, scalars outside the folds.  (name, source, parameter shapes;
# None = a Float scalar)
def A(*dims: int) -> ArrayType:
    return ArrayType(FLOAT, tuple(StaticDim(d) for d in dims))


PLAN_LOSSES = [
    ("linreg", "(define/pi () (loss [w Float b Float x (Array Float 256) y (Array Float 256)] Float) "
               "(/ (fold + 0.0 (* (- (+ (* w x) b) y) (- (+ (* w x) b) y))) 256.0))", [None, None, (256,), (256,)]),
    ("logistic", "(define/pi () (loss [w Float b Float x (Array Float 300) t (Array Float 300)] Float) "
                 "(fold + 0.0 (log (+ 1.0 (exp (- 0.0 (* t (+ (* w x) b))))))))", [None, None, (300,), (300,)]),
    ("frobenius", "(define/pi () (loss [m (Array Float 16 24)] Float) "
                  "(fold + 0.0 (map (lambda (row) (fold + 0.0 (map (lambda (v) (* v v)) row))) m)))", [(16, 24)]),
    ("rank3_cells", "(define/pi () (loss [m (Array Float 2 3 40)] Float) (fold + 0.0 (map (lambda (p) "
                    "(fold + 0.0 (map (lambda (row) (fold + 0.0 (* row (exp row)))) p))) m)))", [(2, 3, 40)]),
    ("scaled", "(define/pi () (loss [s Float x (Array Float 200)] Float) (* s (fold + 0.0 (* x x))))",
     [None, (200,)]),
    ("cell_inits", "(define/pi () (loss [m (Array Float 12 20)] Float) "
                   "(fold + 1.5 (map (lambda (row) (fold + 0.25 (exp row))) m)))", [(12, 20)]),
    ("two_shapes", "(define/pi () (loss [x (Array Float 64) y (Array Float 48)] Float) "
                   "(+ (* 0.5 (fold + 0.0 (* x x))) (log (fold + 0.0 (exp y)))))", [(64,), (48,)]),
    ("large", "(define/pi () (loss [m (Array Float 64 1024) c Float] Float) (/ (fold + 0.0 (map (lambda (row) "
              "(fold + 0.0 (map (lambda (v) (* (- v c) (- v c))) row))) m)) 65536.0))", [(64, 1024), None]),
    # log (1 + sum exp y): the fold's init enters the loss non-linearly
    ("log_init", "(define/pi () (loss [y (Array Float 40)] Float) (log (fold + 1.0 (exp y))))", [(40,)]),
    # a linear layer (examples/crater_train.py:38-44): rows of w times x
    ("linear_mse", "def loss w x y = fold (+) 0.0 (map (\\r -> r * r) (map (-) "
                   "(map (\\row -> fold (+) 0.0 (map (*) row x)) w) y))", [(48, 32), (32,), (48,)], "ml"),
    ("linear_bias_mean", "def loss w x b y = (fold (+) 0.0 (map (\\r -> r * r) (map (-) (map (+) "
                         "(map (\\row -> fold (+) 0.0 (map (*) row x)) w) b) y))) / 64.0",
     [(64, 40), (40,), (64,), (64,)], "ml"),
    ("linear_logistic", "def loss w x t = fold (+) 0.0 (map (\\z -> log (1.0 + exp (0.0 - z))) (map (*) t "
                        "(map (\\row -> fold (+) 0.0 (map (*) row x)) w)))", [(30, 20), (20,), (30,)], "ml"),
    # two layers: h = relu(W1 x + b1), loss = sum((W2 h - y)^2)
    ("mlp_relu", "def loss w1 b1 w2 x y = let h = map (\\v -> if v < 0.0 then 0.0 else v) (map (+) "
                 "(map (\\row -> fold (+) 0.0 (map (*) row x)) w1) b1) in fold (+) 0.0 (map (\\r -> r * r) "
                 "(map (-) (map (\\row -> fold (+) 0.0 (map (*) row h)) w2) y))",
     [(64, 32), (64,), (16, 64), (32,), (16,)], "ml"),
    # two layers with a smooth activation scaled by a scalar parameter
    ("mlp_scaled", "def loss w1 s w2 x = let h = map (\\v -> s * exp (0.0 - v * v)) "
                   "(map (\\row -> fold (+) 0.0 (map (*) row x)) w1) in "
                   "fold (+) 0.0 (map (\\r -> r * r) (map (\\row -> fold (+) 0.0 (map (*) row h)) w2))",
     [(24, 16), None, (8, 24), (16,)], "ml"),
    # a batch of rows through a layer: Z = X W^T, summed over both axes
    ("batched_linear", "def loss w x y = fold (+) 0.0 (map (\\r -> fold (+) 0.0 (map (\\v -> v * v) r)) "
                       "(map (-) (map (\\xi -> map (\\row -> fold (+) 0.0 (map (*) row xi)) w) x) y))",
     [(48, 32), (64, 32), (64, 48)], "ml"),
    ("batched_relu", "def loss w x y = fold (+) 0.0 (map (\\r -> fold (+) 0.0 (map (\\v -> v * v) r)) "
                     "(map (-) (map (\\v -> if v < 0.0 then 0.0 else v) "
                     "(map (\\xi -> map (\\row -> fold (+) 0.0 (map (*) row xi)) w) x)) y))",
     [(40, 24), (72, 24), (72, 40)], "ml"),
    # a batch through two layers: H = relu(X W1^T), Z = H W2^T
    ("batched_mlp", "def loss w1 w2 x y = let h = map (\\v -> if v < 0.0 then 0.0 else v) "
                    "(map (\\xi -> map (\\row -> fold (+) 0.0 (map (*) row xi)) w1) x) in "
                    "fold (+) 0.0 (map (\\r -> fold (+) 0.0 (map (\\v -> v * v) r)) "
                    "(map (-) (map (\\hi -> map (\\row -> fold (+) 0.0 (map (*) row hi)) w2) h) y))",
     [(32, 16), (8, 32), (48, 16), (48, 8)], "ml"),
]


def closed_batched(name: str, args: list[np.ndarray]) -> list[np.ndarray]:
    """Gradients of the batched-layer losses.  The reference's tape cannot
    trace a map nested in a map over another array (remora/ad.py broadcasts
    the two operands of the inner product against each other), so these
    come from the derivative: Z = X W^T, G = dL/dZ, dW = G^T X, dX = G W."""
    w, x, y = (np.asarray(a, np.float64) for a in args)
    z = x @ w.T
    if name == "batched_relu":
        r = np.maximum(z, 0.0) - y
        g = 2.0 * r * (z > 0.0)
    else:
        r = z - y
        g = 2.0 * r
    return [g.T @ x, g @ w, -2.0 * r]


def closed_batched_mlp(name: str, args: list[np.ndarray]) -> list[np.ndarray]:
    """H = relu(X W1^T), Z = H W2^T, loss = sum((Z - Y)^2)."""
    w1, w2, x, y = (np.asarray(a, np.float64) for a in args)
    a1 = x @ w1.T
    h = np.maximum(a1, 0.0)
    r = h @ w2.T - y
    g2 = 2.0 * r
    g1 = (g2 @ w2) * (a1 > 0.0)
    return [g1.T @ x, g2.T @ h, g1 @ w1, -2.0 * r]


CLOSED = {"batched_linear": closed_batched, "batched_relu": closed_batched, "batched_mlp": closed_batched_mlp}


def specialise_ml(src: str, name: str, ptypes, rtype):
    from remora.parser import parse_program
    from remora.typechecker import TypeChecker
    from remora.types import FuncType

    ch = TypeChecker()
    ch.check_program(parse_program(src))
    return ch._typed_top_level_function(ch._functions[name], FuncType(tuple(ptypes), rtype), ch._build_prelude_env())


def closed_log_init(y: np.ndarray) -> np.ndarray:
    """d/dy log(1 + sum exp y) = exp y / (1 + sum exp y)."""
    e = np.exp(y.astype(np.float64))
    return e / (1.0 + e.sum())


def plan_losses(rng) -> None:
    from remora_b200.autodiff import compile_value_and_grad_plan_source

    records, arrays = [], {}
    for name, src, shapes, *rest in PLAN_LOSSES:
        syntax = rest[0] if rest else "lisp"
        ptypes = tuple(FLOAT if s is None else A(*s) for s in shapes)
        plan = compile_value_and_grad_plan_source(src, "loss", ptypes, syntax=syntax)
        args = [np.float32(rng.uniform(0.5, 1.0)) if s is None else rng.uniform(-1.0, 1.0, s).astype(np.float32)
                for s in shapes]
        if name == "logistic":
            args[3] = np.where(rng.random(300) < 0.5, -1.0, 1.0).astype(np.float32)
        sp = (specialise_ml if syntax == "ml" else specialise)(src, "loss", list(ptypes), FLOAT)
        if name in CLOSED:
            grads = CLOSED[name](name, args)
        else:
            tape, idx = trace_via_tape_multi(sp.body, [np.asarray(a, np.float64) for a in args],
                                             [p[0] for p in sp.params])
            adj = tape.reverse()
            grads = [np.asarray(adj[i], dtype=np.float64).reshape(np.shape(a)) for i, a in zip(idx, args)]
        if name == "log_init":
            # remora/ad.py:_trace_fold records a fold's value without its
            # init, so the tape's gradient here is exp y / sum exp y; the
            # mathematics (and the interpreter's value) say 1 + sum exp y
            arrays[f"{name}__tape_grad0"] = grads[0]
            grads = [closed_log_init(args[0])]
        arrays[f"{name}__value"] = np.asarray(_lambda_callable(sp, {})(*args), dtype=np.float64)
        for k, a in enumerate(args):
            arrays[f"{name}__in{k}"] = np.asarray(a, np.float32)
            arrays[f"{name}__grad{k}"] = grads[k]
        if name in CLOSED:
            arrays[f"{name}__closed_form"] = np.asarray(1)  # gradients from the derivative, not the tape
        records.append({"name": name, "source": src, "syntax": syntax,
                        "shapes": [None if s is None else list(s) for s in shapes],
                        "plan": plan.to_record(), "steps": [s["op"] for s in plan.steps]})
        print(name, [s["op"] for s in plan.steps])
    crater_plan(records, arrays)
    (HERE / "value_and_grad_plans.json").write_text(json.dumps(records, indent=1) + "\n")
    np.savez(HERE / "value_and_grad_plans.npz", **arrays)


def crater_example():
    """The reference's crater-CNN example module (examples/crater_train.py),
    loaded from the reference tree: its model source, parameter types,
    initial parameters, data and dropout masks."""
    import importlib.util

    spec = importlib.util.spec_from_file_location("crater_train", os.path.join(REF, "examples", "crater_train.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules["crater_train"] = mod
    spec.loader.exec_module(mod)
    return mod


def crater_plan(records, arrays) -> None:
    """The reference's own crater CNN loss (cnn-loss of
    examples/crater_train.py:29-59: im2col conv, ReLU, dropout mask, a
    900 -> 4 linear layer, ReLU, a 4 -> 1 layer, stable BCE) as ONE
    value-and-grad plan, on the reference's initial parameters, its first
    training image and a dropout mask it makes; value from the reference
    interpreter, every gradient from its tape (remora/ad.py).  The model
    source is not stored: the tests read it from the reference tree."""
    from remora_b200.autodiff import compile_value_and_grad_plan_source

    ct = crater_example()
    ptypes = ct._parameter_types()
    plan = compile_value_and_grad_plan_source(ct._CNN_FULL_LISP_SRC, "cnn-loss", ptypes, include_prelude=False,
                                              syntax="lisp")
    images, labels = ct.make_tiny_dataset(2)
    args = [*ct.initialize_parameters(), ct.make_dropout_mask(seed=42), images[0], np.float32(labels[0])]
    sp = specialise(ct._CNN_FULL_LISP_SRC, "cnn-loss", list(ptypes), FLOAT)
    tape, idx = trace_via_tape_multi(sp.body, [np.asarray(a, np.float64) for a in args], [p[0] for p in sp.params])
    adj = tape.reverse()
    name = "crater_cnn"
    arrays[f"{name}__value"] = np.asarray(_lambda_callable(sp, {})(*args), dtype=np.float64)
    for k, (i, a) in enumerate(zip(idx, args)):
        arrays[f"{name}__in{k}"] = np.asarray(a, np.float32)
        arrays[f"{name}__grad{k}"] = np.asarray(adj[i], dtype=np.float64).reshape(np.shape(a))
    shapes = [None if not np.shape(a) else list(np.shape(a)) for a in args]
    records.append({"name": name, "source": None, "source_in_reference": "examples/crater_train.py:_CNN_FULL_LISP_SRC",
                    "function": "cnn-loss", "include_prelude": False, "syntax": "lisp", "shapes": shapes,
                    "plan": plan.to_record(), "steps": [s["op"] for s in plan.steps]})
    print(name, [s["op"] for s in plan.steps])


def main() -> None:
    x = np.linspace(0.25, 2.0, N, dtype=np.float32)
    y = np.linspace(-1.0, 1.5, N, dtype=np.float32)
    records, arrays = [], {}
    for name, src, n in LOSSES:
        ptypes = (VEC,) * n
        module, metas = compile_value_and_grad_source(src, "loss", ptypes, name=f"remora_{name}")
        args = [x, y][:n]
        sp = specialise(src, "loss", list(ptypes), FLOAT)
        tape, idx = trace_via_tape_multi(sp.body, [a.astype(np.float64) for a in args], [p[0] for p in sp.params])
        adj = tape.reverse()
        grads = [np.asarray(adj[i], dtype=np.float64) for i in idx]
        try:
            arrays[f"{name}__value"] = np.asarray(_lambda_callable(sp, {})(*args), dtype=np.float64)
        except TypeError:  # the interpreter divides whole arrays with float(); no value to record
            arrays[f"{name}__value"] = np.asarray(np.nan)
        for k, a in enumerate(args):
            arrays[f"{name}__in{k}"] = a
            arrays[f"{name}__grad{k}"] = grads[k]
        records.append({"name": name, "source": src, "n_inputs": n,
                        "kernels": {m.name: {"spec": spec_record(module.kernels[m.name]), "meta": meta_record(m)}
                                    for m in metas}})
        print(name, [m.name for m in metas])
    # the reference's closed forms for its three GPU cases
    closed = {"polynomial": 2.0 * x - 1.0, "cubic": 3.0 * x * x, "division": 1.0 / ((x + 1.0) ** 2)}
    for name, g in closed.items():
        np.testing.assert_allclose(arrays[f"{name}__grad0"], g, rtol=1e-5, atol=1e-6)
        arrays[f"{name}__closed"] = g.astype(np.float32)
    (HERE / "reference_gradients.json").write_text(json.dumps(records, indent=1) + "\n")
    np.savez(HERE / "reference_gradients.npz", **arrays)
    plan_losses(np.random.default_rng(2718))


if __name__ == "__main__":
    main()
