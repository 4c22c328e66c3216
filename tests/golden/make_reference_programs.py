"""Generate tests/golden/reference_programs.{json,npz}: Remora programs
compiled by the reference's own front end (remora.compiler.
compile_function_source) and lowered by remora_b200.reference_codegen to
this backend's specs, with seeded inputs and the outputs of the reference
interpreter (remora/runtime.py:_lambda_callable).  The GPU test replays the
recorded specs through B200Executor, so the GPU box needs neither the
reference nor its front end.  The reference is only needed to regenerate:

    REMORA_REFERENCE=/path/to/remorac python tests/golden/make_reference_programs.py

The first programs are the ones the reference's GPU executor tests compile
(tests/test_executor.py: scale, add, sum, dot, inc); the rest cover
the other shapes the codegen accepts.  tests/golden/function_plans.{json,npz}
hold functions no single kernel computes, planned by
remora_b200.program_plan.plan_from_function, with seeded inputs and the
interpreter's outputs.
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

from remora.lisp_reader import parse_lisp  # noqa: E402
from remora.parser import parse_program  # noqa: E402
from remora.runtime import _lambda_callable  # noqa: E402
from remora.typechecker import TypeChecker  # noqa: E402
from remora.types import BOOL, FLOAT, INT, ArrayType, FuncType, StaticDim  # noqa: E402

from remora_b200.codegen import meta_record, spec_record  # noqa: E402
from remora_b200.reference_codegen import compile_function_source_to_b200_artifacts  # noqa: E402

SEED = 1729
ELEM = {"f": FLOAT, "i": INT, "b": BOOL}
NP = {"f": np.float32, "i": np.int32, "b": np.bool_}


def A(e: str, *dims: int) -> ArrayType:
    return ArrayType(ELEM[e], tuple(StaticDim(d) for d in dims))


# (name, syntax, source, function, [(elem, dims)], input maker)
PROGRAMS = [
    ("scale", "ml", "def scale xs = map (* 2.0) xs", "scale", [("f", (4,))], "known:1,2,3,4"),
    ("add", "ml", "def add xs ys = map (+) xs ys", "add", [("f", (4,)), ("f", (4,))], "known:1,2,3,4|10,20,30,40"),
    ("sum", "ml", "def sum xs = fold (+) 0.0 xs", "sum", [("f", (4,))], "known:1,2,3,4"),
    ("dot", "ml", "def dot xs ys = fold (+) 0.0 (map (*) xs ys)", "dot", [("f", (4,)), ("f", (4,))],
     "known:1,2,3,4|10,20,30,40"),
    ("inc", "ml", "def inc xs = map (+ 2) xs", "inc", [("i", (4,))], "known:1,2,3,4"),
    ("scale_rank3", "ml", "def scale xs = map (* 2.0) xs", "scale", [("f", (3, 5, 7))], "normal"),
    ("add_rank2", "ml", "def add xs ys = map (+) xs ys", "add", [("f", (16, 33)), ("f", (16, 33))], "normal"),
    ("chain", "lisp", """
(define/pi () (chain [x (Array Float 6 7 8)] (Array Float 6 7 8))
  (map (lambda (v) (select (> (+ (* v 2.5) 1.0) 0.5) (+ (* v 2.5) 1.0) 0.0)) x))
""", "chain", [("f", (6, 7, 8))], "normal"),
    ("chained_fold", "lisp", """
(define/pi () (chained [x (Array Float 3 4 5 16)] (Array Float 3 4 5))
  (map (lambda (row) (fold + 0.0 (map (lambda (v) (select (> (+ (* v 2.5) 1.0) 0.5) (+ (* v 2.5) 1.0) 0.0)) row)))
       x))
""", "chained", [("f", (3, 4, 5, 16))], "normal"),
    ("row_sumsq", "lisp", """
(define/pi () (rows [x (Array Float 9 40)] (Array Float 9))
  (map (lambda (row) (fold + 0.0 (map (lambda (v) (* v v)) row))) x))
""", "rows", [("f", (9, 40))], "uniform"),
    ("exp_neg", "lisp", """
(define/pi () (en [x (Array Float 50)] (Array Float 50)) (map (lambda (v) (exp (- 0.0 v))) x))
""", "en", [("f", (50,))], "uniform"),
    ("int_lambda", "lisp", """
(define/pi () (il [x (Array Int 4 9) y (Array Int 4 9)] (Array Int 4 9)) (map (lambda (a b) (+ (* a 3) b)) x y))
""", "il", [("i", (4, 9)), ("i", (4, 9))], "ints"),
    ("gt_mask", "lisp", """
(define/pi () (gm [x (Array Float 30)] (Array Bool 30)) (map (lambda (v) (> v 0.25)) x))
""", "gm", [("f", (30,))], "normal"),
    ("bool_and", "lisp", """
(define/pi () (ba [x (Array Bool 17) y (Array Bool 17)] (Array Bool 17)) (map && x y))
""", "ba", [("b", (17,)), ("b", (17,))], "bools"),
    ("prod", "lisp", """
(define/pi () (pr [x (Array Float 12)] Float) (fold * 1.0 x))
""", "pr", [("f", (12,))], "near_one"),
    ("scan_add", "lisp", """
(define/pi () (sc [x (Array Float 300)] (Array Float 300)) (scan + 0.5 x))
""", "sc", [("f", (300,))], "uniform"),
    ("scan_int_exclusive", "lisp", """
(define/pi () (si [x (Array Int 40)] (Array Int 40)) (escan + 3 x))
""", "si", [("i", (40,))], "ints"),
    ("append", "lisp", """
(define/pi () (ap [x (Array Float 7 3) y (Array Float 4 3)] (Array Float 11 3)) (append x y))
""", "ap", [("f", (7, 3)), ("f", (4, 3))], "normal"),
    ("rotate", "lisp", """
(define/pi () (ro [x (Array Int 9 2)] (Array Int 9 2)) (rotate x 4))
""", "ro", [("i", (9, 2))], "ints"),
    ("sort", "lisp", """
(define/pi () (so [x (Array Float 333)] (Array Float 333)) (sort < x))
""", "so", [("f", (333,))], "normal"),
    ("sort_rows", "lisp", """
(define/pi () (sr [x (Array Int 6 50)] (Array Int 6 50)) (sort < x))
""", "sr", [("i", (6, 50))], "small_ints"),
    ("grade", "lisp", """
(define/pi () (gr [x (Array Int 500)] (Array Int 500)) (grade < x))
""", "gr", [("i", (500,))], "small_ints"),
]


# The interpreter evaluates `&&` with Python's `and`, which is undefined for
# whole arrays; the compiled path lowers it to arith.andi (elementwise), which
# is what these expected values follow.
ELEMENTWISE = {"bool_and": lambda x, y: np.logical_and(x, y)}


# Functions no single kernel computes, run as device plans
# (program_plan.plan_from_function): several steps, views, scalar parameters
# (dims None), a fold whose init is a parameter.
FUNCTION_PLANS = [
    ("scan_of_map", "ml", "def f xs = scan (+) 0.0 (map (* 0.5) xs)", "f", [("f", (100,))], "normal"),
    ("reverse_map", "ml", "def f xs = map (+ 1) (reverse xs)", "f", [("i", (9,))], "ints"),
    ("scalar_param", "ml", "def f s xs = map (\\x -> x * s + 1.0) xs", "f", [("f", None), ("f", (7,))], "normal"),
    ("fold_init_param", "ml", "def f s xs = fold (+) s xs", "f", [("f", None), ("f", (50,))], "normal"),
    ("int_fold_init", "ml", "def f k xs = fold (+) k (map (* 3) xs)", "f", [("i", None), ("i", (40,))], "ints"),
    ("rows_then_sort", "lisp", """
(define/pi () (f [x (Array Float 6 30)] (Array Float 6)) (sort < (map (lambda (row) (fold + 0.0 row)) x)))
""", "f", [("f", (6, 30))], "normal"),
    ("transpose_rows", "lisp", """
(define/pi () (f [x (Array Float 5 8)] (Array Float 8)) (map (lambda (row) (fold + 0.0 row)) (transpose x)))
""", "f", [("f", (5, 8))], "normal"),
    ("mask_count", "lisp", """
(define/pi () (f [t Float x (Array Float 64)] Int) (fold + 0 (map (lambda (v) (select (> v t) 1 0)) x)))
""", "f", [("f", None), ("f", (64,))], "normal"),
    # folds of a map over each row, the map fused into the fold: row sums of
    # squares, and the thresholded chain of the chained-map benchmark
    ("row_sumsq", "ml", "def rn x = map (\\row -> fold (+) 0.0 (map (\\v -> v * v) row)) x", "rn",
     [("f", (64, 256))], "normal"),
    ("chained_rows", "ml", "def ch x = map (\\row -> fold (+) 0.0 (map (\\v -> if 0.5 < v * 2.5 + 1.0 "
                           "then v * 2.5 + 1.0 else 0.0) row)) x", "ch", [("f", (16, 32, 64))], "normal"),
    # lifted dot products, written as the prelude's dot a b = sum (map (*) a b)
    # inlined (stdlib/prelude.rem:11,14): rows times a vector, rows times rows
    ("matvec", "ml", "def mv m v = map (\\row -> fold (+) 0.0 (map (*) row v)) m", "mv",
     [("f", (64, 48)), ("f", (48,))], "normal"),
    ("matvec_init", "lisp", """
(define/pi () (f [m (Array Float 7 9) v (Array Float 9)] (Array Float 7)) (map (lambda (row) (fold + 1.5 (map * row v))) m))
""", "f", [("f", (7, 9)), ("f", (9,))], "normal"),
    ("linear", "ml", "def lin w x b = map (+) (map (\\row -> fold (+) 0.0 (map (*) row x)) w) b", "lin",
     [("f", (32, 64)), ("f", (64,)), ("f", (32,))], "normal"),
    ("matmul_rows", "ml", "def mm a bt = map (\\r -> map (\\c -> fold (+) 0.0 (map (*) r c)) bt) a", "mm",
     [("f", (96, 40)), ("f", (80, 40))], "normal"),
    ("matmul_transpose", "ml", "def mm a b = map (\\r -> map (\\c -> fold (+) 0.0 (map (*) r c)) (transpose b)) a",
     "mm", [("f", (33, 20)), ("f", (20, 17))], "normal"),
]


def function_plans(rng) -> None:
    from remora.compiler import compile_function_source

    from remora_b200.program_plan import compile_function_source_to_plan

    records, arrays = [], {}
    for name, syntax, source, fn, params, kind in FUNCTION_PLANS:
        ptypes = tuple(ELEM[e] if d is None else A(e, *d) for e, d in params)
        plan = compile_function_source_to_plan(source, fn, ptypes, syntax=syntax)
        rtype = compile_function_source(source, fn, ptypes, verify=False, include_prelude=False,
                                        syntax=syntax).function_type.result
        inputs = [make_input(kind, k, e, d or (), rng) for k, (e, d) in enumerate(params)]
        out = np.asarray(interpret(source, syntax, fn, ptypes, rtype, [np.array(a) for a in inputs]))
        res = plan.buffers[plan.result]
        out = out.astype({0: np.float32, 1: np.int32, 2: np.bool_}[res.dtype]).reshape(res.shape)
        for k, a in enumerate(inputs):
            arrays[f"{name}__in{k}"] = a
        arrays[f"{name}__out"] = out
        records.append({"name": name, "source": source.strip(), "syntax": syntax, "function": fn,
                        "params": [[e, None if d is None else list(d)] for e, d in params],
                        "plan": plan.to_record(), "steps": [st["op"] for st in plan.steps]})
        print(name, [st["op"] for st in plan.steps], out.shape, out.dtype)
    (HERE / "function_plans.json").write_text(json.dumps(records, indent=1) + "\n")
    np.savez(HERE / "function_plans.npz", **arrays)


def make_input(kind: str, k: int, e: str, dims: tuple[int, ...], rng) -> np.ndarray:
    if kind.startswith("known:"):
        vals = kind[6:].split("|")[k]
        return np.array([float(v) for v in vals.split(",")], dtype=NP[e]).reshape(dims)
    if kind == "normal":
        return rng.standard_normal(dims).astype(NP[e])
    if kind == "uniform":
        return rng.uniform(-1, 1, dims).astype(NP[e])
    if kind == "near_one":
        return rng.uniform(0.9, 1.1, dims).astype(NP[e])
    if kind == "ints":
        return rng.integers(-1000, 1000, dims).astype(NP[e])
    if kind == "small_ints":
        return rng.integers(-5, 5, dims).astype(NP[e])
    if kind == "bools":
        return rng.random(dims) < 0.5
    raise ValueError(kind)


def interpret(source: str, syntax: str, fn: str, ptypes, rtype, args):
    ch = TypeChecker()
    ch.check_program(parse_lisp(source) if syntax == "lisp" else parse_program(source))
    f = ch._functions[fn]
    typed = ch._typed_top_level_function(f, FuncType(tuple(ptypes), rtype), ch._build_prelude_env())
    return _lambda_callable(typed, {})(*args)


def main() -> None:
    rng = np.random.default_rng(SEED)
    records = []
    arrays: dict[str, np.ndarray] = {}
    for name, syntax, source, fn, params, kind in PROGRAMS:
        ptypes = tuple(A(e, *d) for e, d in params)
        module, metas, hir = compile_function_source_to_b200_artifacts(
            source, fn, ptypes, include_prelude=False, kernel_name=f"remora_{name}", syntax=syntax)
        (kname, spec), = module.kernels.items()
        inputs = [make_input(kind, k, e, d, rng) for k, (e, d) in enumerate(params)]
        if name in ELEMENTWISE:
            out = ELEMENTWISE[name](*inputs)
        else:
            out = interpret(source, syntax, fn, ptypes, hir.return_type, [np.array(a) for a in inputs])
        meta = metas[0]
        out = np.asarray(out).astype({"float32": np.float32, "int32": np.int32, "bool": np.bool_}[meta.output_dtype])
        for k, a in enumerate(inputs):
            arrays[f"{name}__in{k}"] = a
        arrays[f"{name}__out"] = out
        records.append({"name": name, "kernel": kname, "source": source.strip(), "syntax": syntax,
                        "spec": spec_record(spec), "meta": meta_record(meta), "n_inputs": len(inputs)})
        print(name, type(spec).__name__, out.shape, out.dtype)
    (HERE / "reference_programs.json").write_text(json.dumps(records, indent=1) + "\n")
    np.savez(HERE / "reference_programs.npz", **arrays)
    function_plans(np.random.default_rng(SEED + 1))


if __name__ == "__main__":
    main()
