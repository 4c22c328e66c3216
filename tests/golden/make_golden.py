"""Generate the golden fixtures in this directory from the Remora reference.

Runs the reference's own interpreter (remora/runtime.py:_lambda_callable,
evaluate_source) and tape AD (remora/ad.py:trace_via_tape_multi) on small
seeded inputs and stores inputs and outputs as .npz files.  The reference is
only needed to regenerate them:

    REMORA_REFERENCE=/path/to/remorac python tests/golden/make_golden.py

Tests read the committed .npz files and never import the reference.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(Path(__file__).resolve().parents[2] / "oracle"))
from oracle import reference_root  # noqa: E402  (REMORA_REFERENCE, or where the oracle's build found it)

if reference_root() is None:
    raise SystemExit("set REMORA_REFERENCE to the reference checkout (the directory holding remora/)")
REF = str(reference_root())
sys.path.insert(0, REF)

from remora.ad import trace_via_tape_multi  # noqa: E402
from remora.lisp_reader import parse_lisp  # noqa: E402
from remora.runtime import _lambda_callable, evaluate_source  # noqa: E402
from remora.typechecker import TypeChecker  # noqa: E402
from remora.types import BOOL, FLOAT, INT, ArrayType, FuncType, StaticDim  # noqa: E402

DATA_SEED = 1729


def A(elem, *dims):
    return ArrayType(elem, tuple(StaticDim(d) for d in dims))


def specialise(src: str, name: str, ptypes, rtype):
    ch = TypeChecker()
    ch.check_program(parse_lisp(src))
    fn = ch._functions[name]
    return ch._typed_top_level_function(fn, FuncType(tuple(ptypes), rtype), ch._build_prelude_env())


def call(src: str, name: str, ptypes, rtype, *args):
    return np.asarray(_lambda_callable(specialise(src, name, ptypes, rtype), {})(*args))


def lisp_list(a: np.ndarray) -> str:
    if a.dtype.kind == "f":
        return "[" + " ".join(repr(float(v)) for v in a.ravel()) + "]"
    return "[" + " ".join(str(int(v)) for v in a.ravel()) + "]"


def save(name: str, **arrays) -> None:
    np.savez(HERE / f"{name}.npz", **arrays)
    print(name, {k: (v.shape, v.dtype) for k, v in arrays.items()})


def main() -> None:
    rng = np.random.default_rng(DATA_SEED)

    # Fused chained maps + threshold mask + last-axis fold (the chained-map
    # workload at a small shape).
    x = rng.standard_normal((3, 4, 5, 8)).astype(np.float32)
    src = """
(define/pi () (cellsum [row (Array Float 8)] Float)
  (fold + 0.0 (map (lambda (v) (select (> (+ (* v 2.5) 1.0) 0.5) (+ (* v 2.5) 1.0) 0.0)) row)))
(define/pi () (chained [x (Array Float 3 4 5 8)] (Array Float 3 4 5))
  (map cellsum x))
"""
    save("chained_maps", x=x, out=call(src, "chained", [A(FLOAT, 3, 4, 5, 8)], A(FLOAT, 3, 4, 5), x))

    # Chained map alone (no fold), elementwise.
    src = """
(define/pi () (chain [x (Array Float 6 7)] (Array Float 6 7))
  (map (lambda (v) (select (> (+ (* v 2.5) 1.0) 0.5) (+ (* v 2.5) 1.0) 0.0)) x))
"""
    x = rng.standard_normal((6, 7)).astype(np.float32)
    save("chain_map", x=x, out=call(src, "chain", [A(FLOAT, 6, 7)], A(FLOAT, 6, 7), x))

    # Row sum of squares (the row_norms workload without its sqrt epilogue,
    # which is not a Remora primitive).
    x = rng.uniform(-1, 1, (16, 32)).astype(np.float32)
    src = """
(define/pi () (sumsq [row (Array Float 32)] Float) (fold + 0.0 (map (lambda (v) (* v v)) row)))
(define/pi () (rows [x (Array Float 16 32)] (Array Float 16)) (map sumsq x))
"""
    save("row_sumsq", x=x, out=call(src, "rows", [A(FLOAT, 16, 32)], A(FLOAT, 16), x))

    # Dense core: matmul as the lifted dot against B^T rows.
    a = rng.uniform(-1, 1, (6, 10)).astype(np.float32)
    bt = rng.uniform(-1, 1, (7, 10)).astype(np.float32)
    src = """
(define/pi () (dotrow [r (Array Float 10) c (Array Float 10)] Float) (fold + 0.0 (map * r c)))
(define/pi () (mm [a (Array Float 6 10) bt (Array Float 7 10)] (Array Float 6 7))
  (map (lambda (row) (map (lambda (col) (dotrow row col)) bt)) a))
"""
    save("lifted_matmul", a=a, bt=bt, out=call(src, "mm", [A(FLOAT, 6, 10), A(FLOAT, 7, 10)], A(FLOAT, 6, 7), a, bt))

    # Binary map with prefix-frame broadcasting: [3,4] + [3].  The program
    # typechecks (prefix agreement), but the interpreter evaluates it with
    # numpy's suffix broadcasting and raises; the CPU MLIR lowering keeps the
    # first k result dims for a rank-k operand
    # (remora/lowering/tensor_ops.py:708-715), which is the rule restated
    # here: out[i, j] = p[i, j] + q[i], one f32 add.
    p = rng.standard_normal((3, 4)).astype(np.float32)
    q = rng.standard_normal((3,)).astype(np.float32)
    src = "(define/pi () (bc [p (Array Float 3 4) q (Array Float 3)] (Array Float 3 4)) (+ p q))"
    try:
        out = call(src, "bc", [A(FLOAT, 3, 4), A(FLOAT, 3)], A(FLOAT, 3, 4), p, q)
    except ValueError:
        out = (p + q[:, None]).astype(np.float32)
    save("broadcast_add", p=p, q=q, out=out)

    # i32 maps and bool maps.
    ia = rng.integers(-50, 50, (5, 6)).astype(np.int32)
    ib = rng.integers(1, 9, (5, 6)).astype(np.int32)
    # `/` on ints is a Float result in Remora (remora/runtime.py:1537-1538).
    src = ("(define/pi () (idiv [a (Array Int 5 6) b (Array Int 5 6)] (Array Float 5 6))"
           " (map (lambda (u v) (/ u v)) a b))")
    save("i32_div", a=ia, b=ib, out=np.asarray(call(src, "idiv", [A(INT, 5, 6), A(INT, 5, 6)], A(FLOAT, 5, 6), ia, ib),
                                               dtype=np.float32))
    src = "(define/pi () (iadd [a (Array Int 5 6)] (Array Int 5 6)) (map (+ 2) a))"
    save("i32_add2", a=ia, out=call(src, "iadd", [A(INT, 5, 6)], A(INT, 5, 6), ia))
    ba = rng.integers(0, 2, (4, 5)).astype(np.bool_)
    bb = rng.integers(0, 2, (4, 5)).astype(np.bool_)
    src = "(define/pi () (band [a (Array Bool 4 5) b (Array Bool 4 5)] (Array Bool 4 5)) (map (lambda (u v) (&& u v)) a b))"
    save("bool_and", a=ba, b=bb, out=call(src, "band", [A(BOOL, 4, 5), A(BOOL, 4, 5)], A(BOOL, 4, 5), ba, bb))
    fz = rng.standard_normal((4, 5)).astype(np.float32)
    src = "(define/pi () (gt [a (Array Float 4 5)] (Array Bool 4 5)) (map (lambda (v) (> v 0.25)) a))"
    save("f32_gt_mask", a=fz, out=call(src, "gt", [A(FLOAT, 4, 5)], A(BOOL, 4, 5), fz))

    # Whole-array folds (the acceptance cases gpu_sum = 45.0 and
    # gpu_fold_i32 = 45, then seeded arrays).
    save("sum_iota10", out=np.asarray(evaluate_source("sum (iota 10)").value, dtype=np.float32))
    v = rng.uniform(-1, 1, 1000).astype(np.float32)
    src = "(define/pi () (s [v (Array Float 1000)] Float) (fold + 0.0 v))"
    save("fold_f32_1000", v=v, out=np.asarray(call(src, "s", [A(FLOAT, 1000)], FLOAT, v), dtype=np.float32))
    iv = rng.integers(-1000, 1000, 777).astype(np.int32)
    src = "(define/pi () (s [v (Array Int 777)] Int) (fold + 0 v))"
    save("fold_i32_777", v=iv, out=np.asarray(call(src, "s", [A(INT, 777)], INT, iv), dtype=np.int32))
    dv1 = rng.uniform(-1, 1, 256).astype(np.float32)
    dv2 = rng.uniform(-1, 1, 256).astype(np.float32)
    src = "(define/pi () (d [a (Array Float 256) b (Array Float 256)] Float) (fold + 0.0 (map * a b)))"
    save("dot_256", a=dv1, b=dv2, out=np.asarray(call(src, "d", [A(FLOAT, 256), A(FLOAT, 256)], FLOAT, dv1, dv2),
                                                  dtype=np.float32))

    # Scans: inclusive, exclusive, right.
    fs = rng.uniform(-1, 1, 100).astype(np.float32)
    isv = rng.integers(-100, 100, 100).astype(np.int32)
    outs = {}
    for tag, form in (("inc", "scan"), ("exc", "escan"), ("right", "trace-right")):
        outs[f"f32_{tag}"] = np.asarray(evaluate_source(f"({form} + 0.5 {lisp_list(fs)})", syntax="lisp").value,
                                        dtype=np.float32)
        outs[f"i32_{tag}"] = np.asarray(evaluate_source(f"({form} + 3 {lisp_list(isv)})", syntax="lisp").value,
                                        dtype=np.int32)
    outs["small_inc"] = np.asarray(evaluate_source("(scan + 0 [2 10 5])", syntax="lisp").value, dtype=np.int32)
    save("scans", f=fs, i=isv, **outs)
    m2 = rng.uniform(-1, 1, (9, 4)).astype(np.float32)
    src = "(define/pi () (sc [m (Array Float 9 4) z (Array Float 4)] (Array Float 9 4)) (scan + z m))"
    z = np.zeros(4, dtype=np.float32)
    save("scan_rank2", m=m2, out=call(src, "sc", [A(FLOAT, 9, 4), A(FLOAT, 4)], A(FLOAT, 9, 4), m2, z))

    # Leading-axis fold with an array accumulator.
    m3 = rng.uniform(-1, 1, (6, 5)).astype(np.float32)
    init = rng.uniform(-1, 1, 5).astype(np.float32)
    src = "(define/pi () (af [m (Array Float 6 5) i (Array Float 5)] (Array Float 5)) (fold + i m))"
    save("array_fold", m=m3, init=init, out=call(src, "af", [A(FLOAT, 6, 5), A(FLOAT, 5)], A(FLOAT, 5), m3, init))

    # im2col / col2im (reference-exact, single channel, no padding).
    img = rng.standard_normal((5, 6)).astype(np.float32)
    res = {"img": img}
    for s in (1, 2):
        oh, ow = (5 - 3) // s + 1, (6 - 3) // s + 1
        src = f"(define/pi () (ic [im (Array Float 5 6)] (Array Float {oh * ow} 9)) (im2col im [3 3] {s}))"
        cols = call(src, "ic", [A(FLOAT, 5, 6)], A(FLOAT, oh * ow, 9), img)
        res[f"cols_s{s}"] = np.asarray(cols, dtype=np.float32)
        cin = rng.standard_normal(cols.shape).astype(np.float32)
        src = f"(define/pi () (ci [c (Array Float {oh * ow} 9)] (Array Float 5 6)) (col2im c [5 6] [3 3] {s}))"
        res[f"cin_s{s}"] = cin
        res[f"img_s{s}"] = np.asarray(call(src, "ci", [A(FLOAT, oh * ow, 9)], A(FLOAT, 5, 6), cin), dtype=np.float32)
    save("im2col", **res)

    # The reference's single-channel conv2d with its gradients (tape AD):
    # loss = sum(conv2d(x, k, b) * cot).
    xi = rng.standard_normal((8, 8)).astype(np.float32)
    k = rng.standard_normal((3, 3)).astype(np.float32)
    b = np.float32(0.125)
    cot = rng.standard_normal(36).astype(np.float32)
    src = """
(define/pi () (dot-patch [patch (Array Float 9) flat-k (Array Float 9)] Float) (fold + 0.0 (map * patch flat-k)))
(define/pi () (conv2d [image (Array Float 8 8) kernel (Array Float 3 3) bias Float] (Array Float 36))
  (+ (map (lambda (p) (dot-patch p (ravel kernel))) (im2col image [3 3] 1)) bias))
(define/pi () (convloss [image (Array Float 8 8) kernel (Array Float 3 3) bias Float c (Array Float 36)] Float)
  (fold + 0.0 (map * (conv2d image kernel bias) c)))
"""
    y = call(src, "conv2d", [A(FLOAT, 8, 8), A(FLOAT, 3, 3), FLOAT], A(FLOAT, 36), xi, k, b)
    sp = specialise(src, "convloss", [A(FLOAT, 8, 8), A(FLOAT, 3, 3), FLOAT, A(FLOAT, 36)], FLOAT)
    tape, idx = trace_via_tape_multi(sp.body, [np.asarray(v, dtype=np.float64) for v in (xi, k, b, cot)],
                                     [p[0] for p in sp.params])
    adj = tape.reverse()
    save("conv_single", x=xi, k=k, b=np.asarray(b), cot=cot, y=np.asarray(y, dtype=np.float32),
         dx=np.asarray(adj[idx[0]], dtype=np.float64), dk=np.asarray(adj[idx[1]], dtype=np.float64),
         db=np.asarray(adj[idx[2]], dtype=np.float64))

    # Stable BCE and its gradient (examples/crater_train.py:50-54).
    zs = np.array([-6.0, -1.5, -0.2, 0.0, 0.3, 2.0, 7.5], dtype=np.float32)
    ys = np.array([1.0, 0.0, 1.0, 1.0, 0.0, 1.0, 0.0], dtype=np.float32)
    src = """
(define/pi () (bce [logit Float y Float] Float)
  (+ (select (> logit 0.0) logit 0.0)
     (+ (* -1.0 (* logit y))
        (log (+ 1.0 (exp (- 0.0 (select (> logit 0.0) logit (- 0.0 logit)))))))))
"""
    losses, grads = [], []
    for zz, yy in zip(zs, ys):
        sp = specialise(src, "bce", [FLOAT, FLOAT], FLOAT)
        losses.append(float(_lambda_callable(sp, {})(np.float32(zz), np.float32(yy))))
        tape, idx = trace_via_tape_multi(sp.body, [np.float64(zz), np.float64(yy)], [p[0] for p in sp.params])
        grads.append(float(tape.reverse()[idx[0]]))
    save("bce", z=zs, y=ys, loss=np.asarray(losses), dz=np.asarray(grads))


def runtime_helpers() -> None:
    """sort / grade / filter / replicate / rotate / append through the
    reference interpreter (remora/runtime.py:1135-1189): the reference's own
    known answers (tests/test_properties.py:450-500) plus seeded cases."""
    rng = np.random.default_rng(DATA_SEED + 7)

    def ev(src: str, dtype) -> np.ndarray:
        return np.asarray(evaluate_source(src, include_prelude=False, syntax="lisp").value, dtype=dtype)

    out: dict[str, np.ndarray] = {}
    # Known answers of the reference's tests.
    out["ka_sort"] = ev("(sort < [3 1 4 1])", np.int32)
    out["ka_grade"] = ev("(grade < [3 1 4 1])", np.int32)
    out["ka_filter"] = ev("(filter (> 0) [1 -2 3 -4])", np.int32)
    out["ka_filter_none"] = ev("(filter (> 0) [-1 -2 -3])", np.int32)
    out["ka_replicate"] = ev("(replicate [2 1 3] [10 20 30])", np.int32)
    out["ka_replicate_zero"] = ev("(replicate [0 1 0] [7 8 9])", np.int32)
    out["ka_rotate"] = ev("(rotate [1 2 3 4 5] 2)", np.int32)
    out["ka_rotate2"] = ev("(rotate [[1 2] [3 4] [5 6]] 1)", np.int32)
    out["ka_append"] = ev("(append [[1 2] [3 4]] [[5 6] [7 8]])", np.int32)
    # Seeded cases: floats (with repeats), ints with many ties, rank 2 rows.
    f = rng.standard_normal(300).astype(np.float32)
    f[::7] = f[3]
    i = rng.integers(-20, 20, 300).astype(np.int32)
    m = rng.integers(-9, 9, (6, 50)).astype(np.int32)
    out["f"], out["i"], out["m"] = f, i, m
    out["sort_f"] = ev(f"(sort < {lisp_list(f)})", np.float32)
    out["grade_f"] = ev(f"(grade < {lisp_list(f)})", np.int32)
    out["sort_i"] = ev(f"(sort < {lisp_list(i)})", np.int32)
    out["grade_i"] = ev(f"(grade < {lisp_list(i)})", np.int32)
    rows = "[" + " ".join(lisp_list(r) for r in m) + "]"
    out["sort_m"] = ev(f"(sort < {rows})", np.int32)
    out["grade_m"] = ev(f"(grade < {rows})", np.int32)
    out["filter_f"] = ev(f"(filter (> 0.25) {lisp_list(f)})", np.float32)
    out["filter_i"] = ev(f"(filter (> 3) {lisp_list(i)})", np.int32)
    c = rng.integers(0, 4, 300).astype(np.int32)
    out["c"] = c
    out["replicate_f"] = ev(f"(replicate {lisp_list(c)} {lisp_list(f)})", np.float32)
    out["rotate_f"] = ev(f"(rotate {lisp_list(f)} 37)", np.float32)
    out["rotate_m"] = ev(f"(rotate {rows} 4)", np.int32)
    out["append_f"] = ev(f"(append {lisp_list(f)} {lisp_list(f[:41])})", np.float32)
    save("rt_helpers", **out)


if __name__ == "__main__":
    if sys.argv[1:] == ["rt"]:
        runtime_helpers()
    else:
        main()
        runtime_helpers()
