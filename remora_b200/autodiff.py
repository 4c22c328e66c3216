"""Value and gradient of a scalar loss in one forward and one backward.

The reference differentiates a program by generating one gradient function
per input and compiling each separately (examples/crater_train.py:169-198;
its fused single-kernel form for ``fold + lit (elementwise expr of x)`` is
compile_gradient_function_source_to_supported_gpu_artifacts, exercised by
remora/tests/test_ad_source.py:553-605).  Here, for a loss

    loss(x_1 .. x_n) = fold (+) init (E(x_1 .. x_n))

with E an elementwise expression over the array parameters (primitives,
sections, lifted arithmetic on whole arrays, lambdas: + - * /, exp, log,
select, comparisons as values), ``value_and_grad_from_hir`` returns one
fused fold for the value and, per parameter, one map that computes
d loss / d x_k = dE/dx_k elementwise (the adjoint of a + fold is 1 at every
element).  The derivative programs come from the VJP rules of
remora/ad.py:85-179 applied symbolically to the expression tree
(``derivative``), simplified, and lowered like any map program.
"""

from __future__ import annotations

from typing import Any

from remora_b200 import _lib as L
from remora_b200.codegen import FoldSpec, KernelMeta, MapSpec, SpecModule, fold_spec
from remora_b200.errors import RemoraUnsupportedError
from remora_b200.program import (
    BinaryExpr,
    CmpExpr,
    ConstantExpr,
    Expr,
    InputExpr,
    LogicExpr,
    SelectExpr,
    UnaryExpr,
    compile_program,
)

_ZERO, _ONE = ConstantExpr(0.0), ConstantExpr(1.0)


def _is(e: Expr, v: float) -> bool:
    return isinstance(e, ConstantExpr) and float(e.value) == v


def _add(a: Expr, b: Expr) -> Expr:
    if _is(a, 0.0):
        return b
    if _is(b, 0.0):
        return a
    return BinaryExpr("+", a, b)


def _sub(a: Expr, b: Expr) -> Expr:
    if _is(b, 0.0):
        return a
    if _is(a, 0.0):
        return UnaryExpr("neg", b)
    return BinaryExpr("-", a, b)


def _mul(a: Expr, b: Expr) -> Expr:
    if _is(a, 0.0) or _is(b, 0.0):
        return _ZERO
    if _is(a, 1.0):
        return b
    if _is(b, 1.0):
        return a
    return BinaryExpr("*", a, b)


def _div(a: Expr, b: Expr) -> Expr:
    if _is(a, 0.0):
        return _ZERO
    if _is(b, 1.0):
        return a
    return BinaryExpr("/", a, b)


def derivative(e: Expr, k: int) -> Expr:
    """d e / d input_k, by the VJP rules of remora/ad.py:85-179 (add/sub
    pass the adjoint through, mul multiplies by the other operand, div by
    1/b and -a/b^2, exp by exp, log by 1/x, select routes the adjoint to the
    branch taken; comparisons and logic are locally constant)."""
    if isinstance(e, InputExpr):
        return _ONE if e.index == k else _ZERO
    if isinstance(e, ConstantExpr) or isinstance(e, (CmpExpr, LogicExpr)):
        return _ZERO
    if isinstance(e, BinaryExpr):
        da, db = derivative(e.left, k), derivative(e.right, k)
        if e.op == "+":
            return _add(da, db)
        if e.op == "-":
            return _sub(da, db)
        if e.op == "*":
            return _add(_mul(da, e.right), _mul(e.left, db))
        if e.op == "/":
            return _sub(_div(da, e.right), _div(_mul(e.left, db), _mul(e.right, e.right)))
    if isinstance(e, UnaryExpr):
        da = derivative(e.operand, k)
        if e.op == "neg":
            return UnaryExpr("neg", da) if not _is(da, 0.0) else _ZERO
        if e.op == "exp":
            return _mul(e, da)
        if e.op == "log":
            return _div(da, e.operand)
        if e.op == "sqrt":
            return _div(da, _mul(ConstantExpr(2.0), e))
    if isinstance(e, SelectExpr):
        dt, de = derivative(e.then_expr, k), derivative(e.else_expr, k)
        if _is(dt, 0.0) and _is(de, 0.0):
            return _ZERO
        return SelectExpr(e.condition, dt, de)
    raise RemoraUnsupportedError(f"no derivative for {e!r}")


# ------------------------------------------------------ from the reference
def _kind(node: object) -> str:
    return type(node).__name__


def _base_op(op: str) -> str:
    for base in ("&&", "||", "<=", ">=", "==", "!=", "exp", "log", "+", "-", "*", "/", "<", ">"):
        if op == base or (op.startswith(base) and op[len(base):] in ("f", "i", "b")):
            return base
    raise RemoraUnsupportedError(f"autodiff: primitive {op!r}")


def _apply(op: str, args: list[Expr]) -> Expr:
    if op in ("exp", "log"):
        return UnaryExpr(op, args[0])
    if op == "-" and len(args) == 1:
        return UnaryExpr("neg", args[0])
    if op in ("+", "-", "*", "/"):
        return BinaryExpr(op, *args)
    if op in ("<", "<=", ">", ">=", "==", "!="):
        return CmpExpr(op, *args)
    return LogicExpr(op, *args)


def _elementwise(node: object, env: dict[str, Expr]) -> Expr:
    """An elementwise HIR expression over the parameters as an Expr."""
    k = _kind(node)
    if k == "HIRVar":
        if node.name not in env:
            raise RemoraUnsupportedError(f"autodiff: free variable {node.name}")
        return env[node.name]
    if k == "HIRLit":
        return ConstantExpr(float(node.value))
    if k in ("HIRApply", "HIRMap"):
        if node.cell_shape:
            raise RemoraUnsupportedError("autodiff: maps over cells of rank >= 1")
        args = [_elementwise(a, env) for a in node.arrays]
        f = node.func
        if _kind(f) == "HIRPrimCallable":
            if f.left_arg is not None:
                args = [_elementwise(f.left_arg, env), *args]
            if f.right_arg is not None:
                args = [*args, _elementwise(f.right_arg, env)]
            return _apply(_base_op(f.op), args)
        if _kind(f) == "HIRLambda":
            return _elementwise(f.body, {**env, **{p.name: a for p, a in zip(f.params, args)}})
        raise RemoraUnsupportedError(f"autodiff: {_kind(f)} as a mapped function")
    if k == "HIRPrimOp":
        return _apply(_base_op(node.op), [_elementwise(a, env) for a in node.args])
    if k == "HIRIf":
        return SelectExpr(_elementwise(node.condition, env), _elementwise(node.then_branch, env),
                          _elementwise(node.else_branch, env))
    raise RemoraUnsupportedError(f"autodiff: {k} in a loss expression")


def value_and_grad_from_hir(function: object, name: str | None = None) -> tuple[SpecModule, list[KernelMeta]]:
    """Specs for the value (``<name>_value``, a fused fold) and the gradient
    with respect to every parameter (``<name>_grad_<param>``, one map each)
    of a loss ``fold (+) lit (E params)`` over f32 arrays of one shape."""
    name = name or f"remora_{function.name}"
    body = function.body
    if _kind(body) != "HIRFold" or _kind(body.func) != "HIRPrimCallable" or _base_op(body.func.op) != "+" or \
            body.func.left_arg is not None or body.func.right_arg is not None or _kind(body.init) != "HIRLit":
        raise RemoraUnsupportedError("autodiff: the loss must be fold (+) <literal> <elementwise expression>")
    params = list(function.params)
    shapes = set()
    for p in params:
        t = p.type
        if _kind(t) != "ArrayType" or _kind(t.element) != "ScalarType" or t.element.name != "float":
            raise RemoraUnsupportedError("autodiff: parameters must be f32 arrays")
        shapes.add(tuple(int(d.value) for d in t.shape))
    if len(shapes) != 1 or len(next(iter(shapes))) != 1 or len(params) > 2:
        raise RemoraUnsupportedError("autodiff: one or two rank-1 f32 parameters of one shape")
    shape = next(iter(shapes))
    expr = _elementwise(body.array, {p.name: InputExpr(i) for i, p in enumerate(params)})
    n = len(params)
    specs: dict[str, Any] = {}
    metas: list[KernelMeta] = []
    vname = f"{name}_value"
    specs[vname] = FoldSpec(fold_spec(op="+", init=float(body.init.value), mode="all", premap=expr, n_inputs=n))
    metas.append(KernelMeta(vname, 1, 0, n, 1, ["f32"] * n, ["f32"], (), "float32", True))
    for k, p in enumerate(params):
        gname = f"{name}_grad_{p.name}"
        d = derivative(expr, k)
        if not any(isinstance(x, InputExpr) for x in _walk(d)):
            d = BinaryExpr("+", d, BinaryExpr("*", InputExpr(0), ConstantExpr(0.0)))  # a map needs an input
        specs[gname] = MapSpec(compile_program(d, n, compute=L.F32))
        metas.append(KernelMeta(gname, 1, 0, n, 1, ["f32"] * n, ["f32"], shape, "float32"))
    return SpecModule(specs), metas


def _walk(e: Expr):
    yield e
    for attr in ("left", "right", "operand", "condition", "then_expr", "else_expr"):
        c = getattr(e, attr, None)
        if c is not None:
            yield from _walk(c)


def compile_value_and_grad_source(source: str, function_name: str, param_types: tuple[Any, ...], *,
                                  include_prelude: bool = False, syntax: str = "lisp",
                                  name: str | None = None) -> tuple[SpecModule, list[KernelMeta]]:
    """The reference's front end followed by ``value_and_grad_from_hir``."""
    from remora.compiler import compile_function_source  # the reference's front end

    artifact = compile_function_source(source, function_name, param_types, verify=False,
                                       include_prelude=include_prelude, syntax=syntax)
    return value_and_grad_from_hir(artifact.hir_function, name or f"remora_{function_name}")
