"""Value and gradient of a scalar loss in one forward and one backward.

The reference differentiates a program by generating one gradient function
per input and compiling each separately (examples/crater_train.py:169-198;
its fused single-kernel form for ``fold + lit (elementwise expr of x)`` is
compile_gradient_function_source_to_supported_gpu_artifacts, exercised by
tests/test_ad_source.py:553-605).  Here, for a loss

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

import numpy as np

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


def _elementwise(node: object, env: dict[str, Expr], on_fold=None, on_cellmap=None) -> Expr:
    """An elementwise HIR expression over the parameters as an Expr
    (``on_fold`` / ``on_cellmap`` turn a fold / a map over cells met on the
    way into an Expr, where allowed)."""
    k = _kind(node)
    if k == "HIRFold" and on_fold is not None:
        return on_fold(node, env)
    if k == "HIRLet":
        value = _elementwise(node.value, env, on_fold, on_cellmap)
        return _elementwise(node.body, {**env, node.name: value}, on_fold, on_cellmap)
    if k == "HIRVar":
        if node.name not in env:
            raise RemoraUnsupportedError(f"autodiff: free variable {node.name}")
        return env[node.name]
    if k == "HIRLit":
        return ConstantExpr(float(node.value))
    if k in ("HIRApply", "HIRMap"):
        if node.cell_shape:
            if on_cellmap is not None:
                return on_cellmap(node, env)
            raise RemoraUnsupportedError("autodiff: maps over cells of rank >= 1")
        args = [_elementwise(a, env, on_fold, on_cellmap) for a in node.arrays]
        f = node.func
        if _kind(f) == "HIRPrimCallable":
            if f.left_arg is not None:
                args = [_elementwise(f.left_arg, env, on_fold, on_cellmap), *args]
            if f.right_arg is not None:
                args = [*args, _elementwise(f.right_arg, env, on_fold, on_cellmap)]
            return _apply(_base_op(f.op), args)
        if _kind(f) == "HIRLambda":
            inner = {**env, **{p.name: a for p, a in zip(f.params, args)}}
            return _elementwise(f.body, inner, on_fold, on_cellmap)
        raise RemoraUnsupportedError(f"autodiff: {_kind(f)} as a mapped function")
    if k == "HIRPrimOp":
        return _apply(_base_op(node.op), [_elementwise(a, env, on_fold, on_cellmap) for a in node.args])
    if k == "HIRIf":
        return SelectExpr(_elementwise(node.condition, env, on_fold, on_cellmap),
                          _elementwise(node.then_branch, env, on_fold, on_cellmap),
                          _elementwise(node.else_branch, env, on_fold, on_cellmap))
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


# ------------------------------------------------- losses as device plans
def _walk_inputs(e: Expr) -> set[int]:
    return {x.index for x in _walk(e) if isinstance(x, InputExpr)}


def _substitute(e: Expr, slot: dict[int, int]) -> Expr:
    """``e`` with every ``InputExpr(i)`` renumbered to ``InputExpr(slot[i])``."""
    if isinstance(e, InputExpr):
        return InputExpr(slot[e.index])
    if isinstance(e, ConstantExpr):
        return e
    if isinstance(e, UnaryExpr):
        return UnaryExpr(e.op, _substitute(e.operand, slot))
    if isinstance(e, SelectExpr):
        return SelectExpr(_substitute(e.condition, slot), _substitute(e.then_expr, slot),
                          _substitute(e.else_expr, slot))
    return type(e)(e.op, _substitute(e.left, slot), _substitute(e.right, slot))


def _type_of(node: object) -> object:
    return getattr(node, "result_type", None) or getattr(node, "type", None)


def _dims(t: object) -> tuple[int, ...]:
    if _kind(t) == "ScalarType":
        return ()
    if _kind(t) != "ArrayType" or any(_kind(d) != "StaticDim" for d in t.shape):
        raise RemoraUnsupportedError("autodiff: arrays of static shape")
    return tuple(int(d.value) for d in t.shape)


class _LossPlanner:
    """Builds the plan of ``value_and_grad_plan_from_hir``.

    Slots number the scalar values and arrays an expression may read:
    0..P-1 are the parameters; the rest are added as the plan grows: the
    value of each fold of the loss (a rank-0 buffer), each layer's output
    (W x, or X W^T for a batch) and computed layer input, and each adjoint
    part or partial sum the backward needs.  Every Expr here is over
    slots; each map or fold step renumbers the slots it reads to its own
    inputs."""

    def __init__(self, params: list) -> None:
        from remora_b200.program_plan import _Planner

        self.pl = _Planner({})
        self.shapes: dict[int, tuple[int, ...]] = {}  # slot -> shape
        self.buf: dict[int, int] = {}  # slot -> plan buffer
        for k, p in enumerate(params):
            t = p.type
            elem = t if _kind(t) == "ScalarType" else getattr(t, "element", None)
            if _kind(elem) != "ScalarType" or elem.name != "float":
                raise RemoraUnsupportedError("autodiff: parameters must be f32 scalars or arrays")
            self.shapes[k] = _dims(t)
            self.buf[k] = self.pl.buf(self.shapes[k], L.F32, input=k)
        self.n_params = len(params)
        self.env = {p.name: InputExpr(k) for k, p in enumerate(params)}
        self.folds: list[tuple[float, Expr, tuple[int, ...]]] = []  # (init, summand, shape)
        # dense layers in forward order: (W, x, init) -> (kind, output slot,
        # W's slot, input's slot); kind "vec" for W x, "batch" for X W^T
        self.layers: dict[tuple, tuple[str, int, int, int]] = {}
        self.computed: dict[int, Expr] = {}  # slots of computed layer inputs -> their expression
        # convolution layers: slot of an im2col patch matrix -> (image slot,
        # kh, kw, stride); slot of a flattened kernel -> the kernel's slot
        self.im2col_of: dict[int, tuple[int, int, int, int]] = {}
        self.ravel_of: dict[int, int] = {}

    def new_slot(self, shape: tuple[int, ...], b: int) -> int:
        k = max(self.buf) + 1
        self.buf[k], self.shapes[k] = b, shape
        return k

    # ---- the loss: h(folds, scalar parameters)
    def on_fold(self, node: object, env: dict) -> Expr:
        f = node.func
        if _kind(f) != "HIRPrimCallable" or _base_op(f.op) != "+" or f.left_arg is not None or \
                f.right_arg is not None or _kind(node.init) != "HIRLit":
            raise RemoraUnsupportedError("autodiff: folds of the loss are fold (+) <literal> <expression>")
        e, shape, extra = self.summand(node.array, env)
        self.folds.append((float(node.init.value) + extra, e, shape))
        return InputExpr(-len(self.folds))  # renumbered once the folds are known

    def summand(self, node: object, env: dict) -> tuple[Expr, tuple[int, ...], float]:
        """(E, shape, c): the fold adds c and every element of E, an
        elementwise expression over arrays of ``shape``.  A map over cells
        whose body is itself ``fold (+) lit cell-expression`` (a sum over a
        rank >= 2 array) flattens into its elements, each cell adding lit."""
        if _kind(node) in ("HIRMap", "HIRApply") and node.cell_shape:
            f = node.func
            if _kind(f) != "HIRLambda" or _kind(f.body) != "HIRFold":
                raise RemoraUnsupportedError("autodiff: cell maps in a loss fold their cells")
            inner = f.body
            g = inner.func
            if _kind(g) != "HIRPrimCallable" or _base_op(g.op) != "+" or g.left_arg is not None or \
                    g.right_arg is not None or _kind(inner.init) != "HIRLit":
                raise RemoraUnsupportedError("autodiff: cell folds are fold (+) <literal> <expression>")
            shapes = {_dims(_type_of(a)) for a in node.arrays}
            if len(shapes) != 1:
                raise RemoraUnsupportedError("autodiff: cell maps over arrays of one shape")
            shape = next(iter(shapes))
            args = [_elementwise(a, env, on_cellmap=self.on_cellmap) for a in node.arrays]
            e, _, extra = self.summand(inner.array, {**env, **{p.name: a for p, a in zip(f.params, args)}})
            cells = int(np.prod(shape[:len(shape) - len(node.cell_shape)], dtype=np.int64))
            return e, shape, cells * (float(inner.init.value) + extra)
        return _elementwise(node, env, on_cellmap=self.on_cellmap), _dims(_type_of(node)), 0.0

    def on_cellmap(self, node: object, env: dict) -> Expr:
        """``map (\\row -> fold (+) lit (map (*) row x)) W`` (the lifted dot
        of stdlib/prelude.rem:14, W and x parameters) inside a summand: a
        matrix-vector product, computed in the forward as one cell fold and
        remembered for the backward; the Expr reads its result."""
        f = node.func
        if len(node.arrays) != 1 or _kind(f) != "HIRLambda" or len(f.params) != 1:
            raise RemoraUnsupportedError("autodiff: maps over cells other than rows times a vector")
        conv = self._conv_layer(node, env)
        if conv is not None:
            return conv
        batched = self._batched_layer(node, env)
        if batched is not None:
            return batched
        w = _elementwise(node.arrays[0], env)
        match = self.pl._match_dot(f.body)
        if not isinstance(w, InputExpr) or w.index >= self.n_params or len(self.shapes[w.index]) != 2 or \
                match is None or f.params[0].name not in match[0] or len(match[0]) != 2:
            raise RemoraUnsupportedError("autodiff: maps over cells other than rows times a vector")
        (other,) = match[0] - {f.params[0].name}
        x = env.get(other)
        n, c = self.shapes[w.index]
        if x is None or any(i < 0 or self.shapes[i] not in ((), (c,)) for i in _walk_inputs(x)):
            raise RemoraUnsupportedError("autodiff: rows times a vector of the row length")
        key = ("vec", w.index, repr(x), match[1])
        if key not in self.layers:
            if isinstance(x, InputExpr) and self.shapes[x.index] == (c,):
                xs = x.index  # a parameter vector, or an earlier layer's output
            else:
                # a vector computed from parameters and earlier layers (h = relu(W1 x + b1))
                xs = self.new_slot((c,), self.emit(x, (c,)))
                self.computed[xs] = x
            xv = self.pl.view(self.buf[xs], (n, c), 0, (0, 1))  # x repeated for every row
            sp = fold_spec(op="+", init=match[1], mode="cell", cell_rank=1, dtype=L.F32,
                           premap=BinaryExpr("*", InputExpr(0), InputExpr(1)), n_inputs=2)
            out = self.pl.buf((n,), L.F32)
            self.pl.plan.steps.append({"op": "fold", "spec": sp, "ins": [self.buf[w.index], xv], "out": out})
            self.layers[key] = ("vec", self.new_slot((n,), out), w.index, xs)
        return InputExpr(self.layers[key][1])

    def _dot_leaves(self, body: object) -> tuple[list, float] | None:
        """([leaf, leaf], init) when ``body`` is ``fold (+) init (map (*) a
        b)``: each leaf is ("free", name) for a name bound outside the body,
        or (node, names) for a computed operand; None for any other body."""
        pl = self.pl
        node, s = pl._resolve(body, {})
        if _kind(node) != "HIRFold":
            return None
        f = node.func
        if _kind(f) != "HIRPrimCallable" or _base_op(f.op) != "+" or f.left_arg is not None or \
                f.right_arg is not None:
            return None
        init, _ = pl._resolve(node.init, s)
        if _kind(init) != "HIRLit" or isinstance(init.value, bool):
            return None
        m, s2 = pl._resolve(node.array, s)
        if _kind(m) not in ("HIRMap", "HIRApply") or m.cell_shape or len(m.arrays) != 2:
            return None
        g = m.func
        if _kind(g) != "HIRPrimCallable" or _base_op(g.op) != "*" or g.left_arg is not None or \
                g.right_arg is not None:
            return None
        return [pl._resolve(a, s2) for a in m.arrays], float(init.value)

    def _conv_layer(self, node: object, env: dict) -> Expr | None:
        """``map (\\p -> dot p (ravel K)) (im2col X [kh kw] s)``: the
        reference's conv2d (examples/crater_train.py:30-36), every patch of
        the image X times the flattened kernel K.  The forward runs im2col
        once (the patch matrix stays for the backward) and then the rows of
        the patch matrix times ravel(K), a linear layer whose matrix is
        computed from X; the backward sends the layer's adjoint to K as
        patches^T g and to X through col2im, the im2col VJP of
        remora/ad.py:157-171.  None for a cell map over anything but im2col."""
        f, arr = node.func, node.arrays[0]
        if _kind(arr) != "HIRIm2col":
            return None
        img = _elementwise(arr.image, env)
        if not isinstance(img, InputExpr) or img.index >= self.n_params or len(self.shapes[img.index]) != 2:
            raise RemoraUnsupportedError("autodiff: im2col of a rank-2 image parameter")
        kh, kw = (int(v) for v in arr.kernel_shape)
        stride = int(arr.stride)
        dot = self._dot_leaves(f.body)
        if dot is None:
            raise RemoraUnsupportedError("autodiff: a map over im2col patches other than a dot with a kernel")
        (la, sa), (lb, sb) = dot[0]
        p = f.params[0].name
        if la == ("free", p):
            other, osub = lb, sb
        elif lb == ("free", p):
            other, osub = la, sa
        else:
            raise RemoraUnsupportedError("autodiff: a dot of each patch with a kernel")
        if not isinstance(other, tuple) and _kind(other) == "HIRRavel":
            other, _ = self.pl._resolve(other.array, osub)
            want = (kh, kw)
        else:
            want = (kh * kw,)
        kern = env.get(other[1]) if isinstance(other, tuple) and other[0] == "free" else None
        if not isinstance(kern, InputExpr) or kern.index >= self.n_params or self.shapes[kern.index] != want:
            raise RemoraUnsupportedError("autodiff: the kernel of a conv layer is a parameter of the patch size")
        key = ("conv", img.index, kern.index, kh, kw, stride, dot[1])
        if key not in self.layers:
            H, W = self.shapes[img.index]
            n, c = ((H - kh) // stride + 1) * ((W - kw) // stride + 1), kh * kw
            cols = self.pl.buf((n, c), L.F32)
            self.pl.plan.steps.append({"op": "im2col", "in": self.buf[img.index], "out": cols, "kh": kh, "kw": kw,
                                       "stride": stride})
            ws = self.new_slot((n, c), cols)
            self.im2col_of[ws] = (img.index, kh, kw, stride)
            if want == (kh, kw):
                xs = self.new_slot((c,), self.pl.view(self.buf[kern.index], (c,), 0, (1,)))  # ravel K
                self.ravel_of[xs] = kern.index
            else:
                xs = kern.index
            xv = self.pl.view(self.buf[xs], (n, c), 0, (0, 1))  # the kernel repeated for every patch
            sp = fold_spec(op="+", init=dot[1], mode="cell", cell_rank=1, dtype=L.F32,
                           premap=BinaryExpr("*", InputExpr(0), InputExpr(1)), n_inputs=2)
            out = self.pl.buf((n,), L.F32)
            self.pl.plan.steps.append({"op": "fold", "spec": sp, "ins": [cols, xv], "out": out})
            self.layers[key] = ("vec", self.new_slot((n,), out), ws, xs)
        return InputExpr(self.layers[key][1])

    def _batched_layer(self, node: object, env: dict) -> Expr | None:
        """``map (\\xi -> map (\\row -> dot row xi) W) X``: every row of the
        batch X [B, c] times W [n, c]'s rows, Z = X W^T [B, n], as one 3xTF32
        GEMM step; None for any other cell map."""
        f = node.func
        inner, s = self.pl._resolve(f.body, {})
        if isinstance(inner, tuple) or _kind(inner) not in ("HIRMap", "HIRApply") or len(inner.cell_shape) != 1 \
                or len(inner.arrays) != 1 or _kind(inner.func) != "HIRLambda" or len(inner.func.params) != 1:
            return None
        match = self.pl._match_dot(inner.func.body)
        if match is None or match[0] != {inner.func.params[0].name, f.params[0].name}:
            return None
        src, _ = self.pl._resolve(inner.arrays[0], s)
        x, w = _elementwise(node.arrays[0], env), env.get(src[1]) if isinstance(src, tuple) else None
        if not isinstance(w, InputExpr) or w.index >= self.n_params or len(self.shapes[w.index]) != 2:
            raise RemoraUnsupportedError("autodiff: a batch of rows times a parameter matrix")
        xshape = _dims(_type_of(node.arrays[0]))
        (n, c) = self.shapes[w.index]
        if len(xshape) != 2 or xshape[1] != c or \
                any(i < 0 or self.shapes[i] not in ((), xshape) for i in _walk_inputs(x)):
            raise RemoraUnsupportedError("autodiff: a batch of rows of the layer's row length")
        b = xshape[0]
        key = ("batch", w.index, repr(x), match[1])
        if key not in self.layers:
            if isinstance(x, InputExpr) and self.shapes[x.index] == xshape:
                xs = x.index  # a parameter batch, or an earlier layer's output
            else:
                xs = self.new_slot(xshape, self.emit(x, xshape))  # computed (H = relu(X W1^T))
                self.computed[xs] = x
            out = self.pl.buf((b, n), L.F32)
            wt = self.pl.view(self.buf[w.index], (c, n), 0, (1, c))  # W^T
            self.pl.plan.steps.append({"op": "gemm", "a": self.buf[xs], "b": wt, "out": out,
                                       "precision": L.PREC_3XTF32})
            if match[1] != 0.0:
                out = self.pl.emit_map(BinaryExpr("+", InputExpr(0), ConstantExpr(match[1])), [out], (b, n), L.F32)
            self.layers[key] = ("batch", self.new_slot((b, n), out), w.index, xs)
        return InputExpr(self.layers[key][1])

    # ---- steps
    def emit(self, e: Expr, shape: tuple[int, ...]) -> int:
        """A map step computing ``e`` over ``shape`` (rank-0 operands splat)."""
        used = sorted(_walk_inputs(e))
        for i in used:
            if self.shapes[i] not in ((), shape):
                raise RemoraUnsupportedError("autodiff: an expression over arrays of different shapes")
        operands = [self.buf[i] for i in used]
        expr = _substitute(e, {i: j for j, i in enumerate(used)})
        if not operands:
            # a constant (a parameter the loss ignores has gradient 0): a
            # rank-0 constant, or a map over a parameter of the shape that
            # reads none of it
            if shape == ():
                return self.pl.buf((), L.F32, const=np.asarray(_constant(expr), dtype=np.float32))
            operands = [next(self.buf[i] for i in range(self.n_params) if self.shapes[i] == shape)]
        return self.pl.emit_map(expr, operands, shape, L.F32)

    def fold_sum(self, e: Expr, shape: tuple[int, ...], init: float) -> int:
        """A rank-0 buffer holding init + the sum of every element of e."""
        used = sorted(_walk_inputs(e))
        if not used:
            raise RemoraUnsupportedError("autodiff: a fold of an expression of no parameter")
        arrays = [i for i in used if self.shapes[i] == shape and shape != ()]
        n = int(np.prod(shape, dtype=np.int64))
        flat = lambda b: self.pl.view(b, (n,), 0, (1,))  # noqa: E731  (every operand here is contiguous)
        if len(arrays) == len(used) and len(used) <= 2:
            ins = [flat(self.buf[i]) for i in used]
            premap = None if isinstance(e, InputExpr) else _substitute(e, {i: j for j, i in enumerate(used)})
        else:
            ins, premap = [flat(self.emit(e, shape))], None
        sp = fold_spec(op="+", init=init, mode="all", dtype=L.F32, premap=premap, n_inputs=len(ins))
        out = self.pl.buf((), L.F32)
        self.pl.plan.steps.append({"op": "fold", "spec": sp, "ins": ins, "out": out})
        return out


def _constant(e: Expr) -> np.float32:
    """The f32 value of an expression without inputs."""
    f = np.float32
    if isinstance(e, ConstantExpr):
        return f(e.value)
    if isinstance(e, UnaryExpr):
        v = _constant(e.operand)
        return {"neg": lambda: -v, "exp": lambda: f(np.exp(v)), "log": lambda: f(np.log(v))}[e.op]()
    if isinstance(e, BinaryExpr):
        a, b = _constant(e.left), _constant(e.right)
        return {"+": lambda: f(a + b), "-": lambda: f(a - b), "*": lambda: f(a * b), "/": lambda: f(a / b)}[e.op]()
    raise RemoraUnsupportedError(f"autodiff: a constant expression {e!r} as a result")


def value_and_grad_plan_from_hir(function: object):
    """One device plan for a loss and its gradient with respect to every
    parameter, from the reference's HIR function.

    The loss is any scalar expression h of f32 scalar parameters and of
    sums ``S_i = fold (+) lit_i E_i``, where E_i is elementwise over
    parameters (arrays of one shape, scalars broadcast); a sum over a rank
    >= 2 array written as a map of cell folds counts as one sum.  The plan's
    forward computes every S_i (one fold, fused with E_i where it reads at
    most two arrays) and the loss h; its backward applies the VJP rules of
    remora/ad.py:85-179 through the chain rule:

        dL/dx = sum_i dh/dS_i * dE_i/dx                      (x an array: one map)
        dL/dw = dh/dw + sum_i dh/dS_i * sum(dE_i/dw)         (w a scalar: folds, then a map)

    The folds' adjoint broadcasts along the folded axis (remora/ad.py:
    fold VJP) and a scalar's adjoint is the sum over the elements it was
    broadcast to (the unbroadcast rule).  E_i may also read a matrix-vector
    product of parameters, ``map (\\row -> dot row x) W`` (a linear layer,
    examples/crater_train.py:38-44): the forward computes it once, and its
    adjoint g reaches W as the outer product g x^T (one map over two
    stride-0 views) and x as W^T g (one cell fold over W's transposed view).
    x may itself be computed from parameters and earlier layers (a ``let``
    of ``relu (W1 x + b1)``): the forward computes it once, and the backward
    runs the layers last to first, passing W^T g through dx/d(inputs) to the
    earlier layers and parameters (a two-layer perceptron).  A batch of rows
    through a layer, ``map (\\xi -> map (\\row -> dot row xi) W) X``, is
    one 3xTF32 GEMM Z = X W^T forward and two backward, dW = G^T X and
    dX = G W, on the tensor cores.  ``plan.results`` lists the loss,
    then one gradient per parameter; run it with
    ``program_plan.execute_plan_results``."""
    lp = _LossPlanner(list(function.params))
    if _dims(function.return_type) != ():
        raise RemoraUnsupportedError("autodiff: the loss is a scalar")
    h = _elementwise(function.body, lp.env, lp.on_fold, lp.on_cellmap)
    if not lp.folds:
        raise RemoraUnsupportedError("autodiff: the loss sums an array with fold (+)")
    for i in _walk_inputs(h):
        if i >= 0 and lp.shapes[i] != ():
            raise RemoraUnsupportedError("autodiff: an array parameter outside the loss's folds")
    # folds became InputExpr(-1), InputExpr(-2), ...: give them slots
    fold_slot = {}
    for i, (init, e, shape) in enumerate(lp.folds):
        for j in _walk_inputs(e):
            if lp.shapes[j] not in ((), shape):
                raise RemoraUnsupportedError("autodiff: a fold over arrays of different shapes")
        fold_slot[-(i + 1)] = lp.new_slot((), lp.fold_sum(e, shape, init))
    h = _substitute(h, {**fold_slot, **{k: k for k in range(lp.n_params)}})
    results = [lp.buf[next(iter(_walk_inputs(h)))] if isinstance(h, InputExpr) else lp.emit(h, ())]
    adj = [derivative(h, fold_slot[-(i + 1)]) for i in range(len(lp.folds))]
    # Dense layers go last to first: a layer's adjoint g is complete once
    # every later layer that reads its output (through a computed input) has
    # added to it.  W x: g reaches W as the outer product g x^T and x as
    # W^T g; X W^T: dW = g^T X and dX = g W, two 3xTF32 GEMMs.
    contrib: dict[int, list[int]] = {}  # parameter slot -> gradient parts
    later: dict[int, list[int]] = {}  # layer output slot -> adjoint parts from later layers
    outputs = {z for _, z, _, _ in lp.layers.values()}
    prod = BinaryExpr("*", InputExpr(0), InputExpr(1))
    for kind, z, wk, xk in reversed(list(lp.layers.values())):
        gz: Expr = _ZERO
        for i, (_, e, fshape) in enumerate(lp.folds):
            if fshape == lp.shapes[z]:
                gz = _add(gz, _mul(adj[i], derivative(e, z)))
        for part in later.get(z, []):
            gz = _add(gz, InputExpr(lp.new_slot(lp.shapes[z], part)))
        if _is(gz, 0.0):
            continue
        # a single part handed on by a later layer is already a buffer
        single = isinstance(gz, InputExpr) and lp.shapes[gz.index] == lp.shapes[z]
        gzb = lp.buf[gz.index] if single else lp.emit(gz, lp.shapes[z])
        n, c = lp.shapes[wk]
        xshape = lp.shapes[xk]
        dx = lp.pl.buf(xshape, L.F32)
        if kind == "vec":
            dw = lp.pl.emit_map(prod, [lp.pl.view(gzb, (n, c), 0, (1, 0)), lp.pl.view(lp.buf[xk], (n, c), 0, (0, 1))],
                                (n, c), L.F32)
            sp = fold_spec(op="+", init=0.0, mode="cell", cell_rank=1, dtype=L.F32, premap=prod, n_inputs=2)
            lp.pl.plan.steps.append({"op": "fold", "spec": sp, "out": dx, "ins": [
                lp.pl.view(lp.buf[wk], (c, n), 0, (1, c)), lp.pl.view(gzb, (c, n), 0, (0, 1))]})  # W^T, g per row
        else:
            b = xshape[0]
            dw = lp.pl.buf((n, c), L.F32)
            lp.pl.plan.steps.append({"op": "gemm", "a": lp.pl.view(gzb, (n, b), 0, (1, n)), "b": lp.buf[xk],
                                     "out": dw, "precision": L.PREC_3XTF32})
            lp.pl.plan.steps.append({"op": "gemm", "a": gzb, "b": lp.buf[wk], "out": dx,
                                     "precision": L.PREC_3XTF32})
        if wk in lp.im2col_of:
            # a patch matrix: its adjoint reaches the image through col2im
            img, kh, kw, stride = lp.im2col_of[wk]
            dimg = lp.pl.buf(lp.shapes[img], L.F32)
            lp.pl.plan.steps.append({"op": "col2im", "in": dw, "out": dimg, "kh": kh, "kw": kw, "stride": stride})
            contrib.setdefault(img, []).append(dimg)
        else:
            contrib.setdefault(wk, []).append(dw)
        if xk in lp.ravel_of:
            # a flattened kernel: its adjoint is the kernel's, reshaped
            k = lp.ravel_of[xk]
            ks = lp.shapes[k]
            contrib.setdefault(k, []).append(lp.pl.view(dx, ks, 0, (ks[1], 1)))
            continue
        if xk not in lp.computed:
            contrib.setdefault(xk, []).append(dx)
            continue
        # a computed input x = X(...): its adjoint dx flows on through dX/dq
        X, ds = lp.computed[xk], lp.new_slot(xshape, dx)
        for q in sorted(_walk_inputs(X)):
            dq = _mul(InputExpr(ds), derivative(X, q))
            if _is(dq, 0.0):
                continue
            if q in outputs:
                later.setdefault(q, []).append(lp.emit(dq, xshape))
            elif lp.shapes[q] == ():
                contrib.setdefault(q, []).append(lp.fold_sum(dq, xshape, 0.0))
            else:
                contrib.setdefault(q, []).append(lp.emit(dq, xshape))
    for k in range(lp.n_params):
        shape = lp.shapes[k]
        if shape != ():
            g: Expr = _ZERO
            for i, (_, e, fshape) in enumerate(lp.folds):
                if fshape == shape:
                    g = _add(g, _mul(adj[i], derivative(e, k)))
            parts = contrib.get(k, [])
            if _is(g, 0.0) and len(parts) == 1 and lp.pl.plan.buffers[parts[0]].view is None:
                results.append(parts[0])
                continue
            for b in parts:
                g = _add(g, InputExpr(lp.new_slot(shape, b)))
            results.append(lp.emit(g, shape))
        else:
            g = derivative(h, k)
            for i, (_, e, fshape) in enumerate(lp.folds):
                de = derivative(e, k)
                if not _is(de, 0.0):
                    g = _add(g, _mul(adj[i], InputExpr(lp.new_slot((), lp.fold_sum(de, fshape, 0.0)))))
            for b in contrib.get(k, []):
                g = _add(g, InputExpr(lp.new_slot((), b)))
            results.append(lp.emit(g, ()))
    lp.pl.plan.result = results[0]
    lp.pl.plan.results = results
    return lp.pl.plan


def compile_value_and_grad_plan_source(source: str, function_name: str, param_types: tuple[Any, ...], *,
                                       include_prelude: bool = True, syntax: str = "lisp"):
    """The reference's front end followed by ``value_and_grad_plan_from_hir``
    (ML sources see the prelude's ``sum``, ``dot``, ``scale`` ... unless
    ``include_prelude`` is False)."""
    from remora.compiler import compile_function_source  # the reference's front end

    artifact = compile_function_source(source, function_name, param_types, verify=False,
                                       include_prelude=include_prelude, syntax=syntax)
    return value_and_grad_plan_from_hir(artifact.hir_function)


def execute_value_and_grad(plan, inputs: list[Any], device: int | None = None):
    """(loss, [gradient per parameter]) of a value-and-grad plan on the device."""
    from remora_b200.program_plan import execute_plan_results

    out = execute_plan_results(plan, [np.asarray(a, dtype=np.float32) for a in inputs], device)
    return float(out[0]), out[1:]
