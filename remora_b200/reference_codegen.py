"""Specs for this backend from the reference compiler's HIR.

The reference turns one type-checked function into descriptor-ABI PTX plus
``KernelMeta`` in ``generate_mlir_descriptor_abi_ptx``
(remora/codegen.py:116-257), reached from
``compile_function_source_to_supported_gpu_artifacts``
(remora/compiler.py:226-272); what it accepts is the set its builders
recognise (f32 / i32 / bool maps, f32 whole-array folds and their dot form,
rank-1 f32 scans and appends).  ``specs_from_hir`` is the same step for this
backend: it reads the HIR (nodes matched by class name and field, as
``program.from_reference_expr`` does, so importing this module does not
import the reference) and returns a ``SpecModule`` and the ``KernelMeta``
list that ``RemoraExecutor`` / ``B200Executor`` run.  It accepts

- maps over the parameters, rank 1 to 10, f32 / i32 / bool: a primitive
  (binary, or a section with a literal) or a lambda whose body is a scalar
  expression (+ - * /, comparisons, && ||, exp, log, select / if), fused
  into one program (remora/_gpu_map_support.py:85-295 is the reference's
  analysis of the same shapes);
- cell folds: ``map (lambda (cell ...) (fold op lit <cell or map over the
  cells>))`` over the parameters, the inner map fused in
  (remora/lowering/tensor_ops.py:802-874);
- whole-array folds with + or * and a literal init, of a parameter or of a
  map over the parameters (the reference's dot form,
  remora/gpu_lowering.py:928-982);
- scans with + or * and a literal init (remora/lowering/tensor_ops.py:
  2301-2482): rank 1 inclusive, exclusive or right; higher ranks inclusive;
- append, rotate, sort and grade of parameters.

Anything else raises ``RemoraUnsupportedError``, the counterpart of the
reference's ``CodegenUnavailable``.
"""

from __future__ import annotations

from typing import Any

from remora_b200 import _lib as L
from remora_b200.codegen import (
    AppendSpec,
    FoldSpec,
    KernelMeta,
    MapSpec,
    RotateSpec,
    ScanSpec,
    SortSpec,
    SpecModule,
    fold_spec,
    scan_spec,
)
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

_ELEM = {"float": L.F32, "int": L.I32, "bool": L.BOOL}
_ELEM_NAME = {L.F32: "f32", L.I32: "i32", L.BOOL: "i8"}
_NP_NAME = {L.F32: "float32", L.I32: "int32", L.BOOL: "bool"}
_ARITH = {"+", "-", "*", "/"}
_CMP = {"<", "<=", ">", ">=", "==", "!="}
_LOGIC = {"&&", "||"}
_UNARY = {"exp", "log"}


def _kind(node: object) -> str:
    return type(node).__name__


def _unsupported(msg: str) -> RemoraUnsupportedError:
    return RemoraUnsupportedError(f"B200 codegen: {msg}")


def _scalar_code(t: object) -> int:
    if _kind(t) != "ScalarType" or t.name not in _ELEM:
        raise _unsupported(f"element type {t!r} (float, int and bool only)")
    return _ELEM[t.name]


def _array(t: object) -> tuple[int, tuple[int, ...]]:
    """(element code, static shape) of an ArrayType."""
    if _kind(t) != "ArrayType":
        raise _unsupported(f"{t!r} is not an array type")
    dims = []
    for d in t.shape:
        if _kind(d) != "StaticDim":
            raise _unsupported("shapes must be static")
        dims.append(int(d.value))
    return _scalar_code(t.element), tuple(dims)


def _param_index(node: object, params: list) -> int:
    if _kind(node) != "HIRVar":
        raise _unsupported("operands must be the function's parameters")
    for k, p in enumerate(params):
        if p.name == node.name:
            return k
    raise _unsupported(f"{node.name} is not a parameter")


def _base_op(op: str) -> str:
    """HIR primitive names carry a result-type suffix ('+f', '>b', 'expf')."""
    for base in sorted(_ARITH | _CMP | _LOGIC | _UNARY, key=len, reverse=True):
        if op == base or (op.startswith(base) and op[len(base):] in ("f", "i", "b")):
            return base
    raise _unsupported(f"primitive {op!r}")


def _lit(node: object) -> ConstantExpr:
    v = node.value
    return ConstantExpr(int(v) if isinstance(v, bool) else v)


def _scalar_expr(node: object, env: dict[str, Expr]) -> Expr:
    """A lambda body over scalar parameters as an expression tree."""
    k = _kind(node)
    if k == "HIRVar":
        if node.name not in env:
            raise _unsupported(f"free variable {node.name} in a map body")
        return env[node.name]
    if k == "HIRLit":
        return _lit(node)
    if k == "HIRIf":
        return SelectExpr(_scalar_expr(node.condition, env), _scalar_expr(node.then_branch, env),
                          _scalar_expr(node.else_branch, env))
    if k == "HIRPrimOp":
        op = _base_op(node.op)
        args = [_scalar_expr(a, env) for a in node.args]
        return _apply(op, args)
    if k == "HIRApply" and _kind(getattr(node, "func", None)) == "HIRPrimCallable":
        return _apply_callable(node.func, [_scalar_expr(a, env) for a in node.args])
    raise _unsupported(f"{k} in a map body")


def _apply(op: str, args: list[Expr]) -> Expr:
    if op in _UNARY and len(args) == 1:
        return UnaryExpr(op, args[0])
    if op == "-" and len(args) == 1:
        return UnaryExpr("neg", args[0])
    if len(args) != 2:
        raise _unsupported(f"{op} with {len(args)} operands")
    if op in _ARITH:
        return BinaryExpr(op, *args)
    if op in _CMP:
        return CmpExpr(op, *args)
    if op in _LOGIC:
        return LogicExpr(op, *args)
    raise _unsupported(f"primitive {op!r}")


def _apply_callable(c: object, args: list[Expr]) -> Expr:
    """A primitive callable, possibly a section with a literal operand."""
    op = _base_op(c.op)
    if c.left_arg is not None:
        args = [_section_operand(c.left_arg), *args]
    if c.right_arg is not None:
        args = [*args, _section_operand(c.right_arg)]
    return _apply(op, args)


def _section_operand(node: object) -> Expr:
    if _kind(node) != "HIRLit":
        raise _unsupported("sections must hold a literal")
    return _lit(node)


def _map_expr(mapnode: object, operands: list[Expr]) -> Expr:
    """The elementwise function of a map applied to operand expressions."""
    f = mapnode.func
    if _kind(f) == "HIRPrimCallable":
        return _apply_callable(f, operands)
    if _kind(f) == "HIRLambda":
        if len(f.params) != len(operands):
            raise _unsupported("lambda arity differs from the mapped arrays")
        return _scalar_expr(f.body, {p.name: e for p, e in zip(f.params, operands)})
    raise _unsupported(f"{_kind(f)} as a mapped function")


def _meta(name: str, in_codes: list[int], out_code: int, shape: tuple[int, ...], *,
          reduction: bool = False) -> KernelMeta:
    return KernelMeta(name=name, grid_dims=1, block_size=0, num_inputs=len(in_codes), num_outputs=1,
                      input_elem_types=[_ELEM_NAME[c] for c in in_codes], output_elem_types=[_ELEM_NAME[out_code]],
                      output_shape=shape, output_dtype=_NP_NAME[out_code], is_reduction=reduction)


def _compute_type(codes: list[int]) -> int:
    if L.F32 in codes:
        return L.F32
    if L.I32 in codes:
        return L.I32
    return L.BOOL


def _fold_parts(fold: object) -> tuple[str, float | int]:
    f = fold.func
    if _kind(f) != "HIRPrimCallable" or f.left_arg is not None or f.right_arg is not None:
        raise _unsupported("folds take a primitive binary operator")
    op = _base_op(f.op)
    if op not in ("+", "*"):
        raise _unsupported(f"fold with {op} (+ and * only)")
    if _kind(fold.init) != "HIRLit":
        raise _unsupported("fold initial values must be literals")
    return op, fold.init.value


def specs_from_hir(function: object, kernel_name: str | None = None) -> tuple[SpecModule, list[KernelMeta]]:
    """SpecModule and KernelMeta for one reference HIRFunction."""
    name = kernel_name or f"remora_{function.name}"
    params = list(function.params)
    body = function.body
    k = _kind(body)
    in_types = [_array(p.type) for p in params] if all(_kind(p.type) == "ArrayType" for p in params) else None
    if in_types is None:
        raise _unsupported("every parameter must be an array")
    in_codes = [c for c, _ in in_types]

    if k == "HIRMap":
        arrays = [_param_index(a, params) for a in body.arrays]
        if arrays != list(range(len(params))):
            raise _unsupported("a map must take the parameters in order")
        out_code, out_shape = _array(function.return_type)
        f = body.func
        if body.cell_shape and _kind(f) == "HIRLambda" and _kind(f.body) == "HIRFold":
            return _cell_fold(name, params, in_types, f, out_code, out_shape)
        if body.cell_shape:
            raise _unsupported("maps over cells of rank >= 1 other than folds")
        expr = _map_expr(body, [InputExpr(i) for i in range(len(params))])
        for _, shape in in_types:
            if shape != out_shape[: len(shape)]:
                raise _unsupported("operand shapes must be prefixes of the result shape")
        prog = compile_program(expr, len(params), compute=_compute_type(in_codes + [out_code]), out=out_code,
                               in_dtypes=in_codes)
        return SpecModule({name: MapSpec(prog)}), [_meta(name, in_codes, out_code, out_shape)]

    if k == "HIRFold":
        op, init = _fold_parts(body)
        out_code = _scalar_code(function.return_type)
        arr = body.array
        if _kind(arr) == "HIRVar":
            premap, n_in = None, 1
            if _param_index(arr, params) != 0 or len(params) != 1:
                raise _unsupported("a fold must take its one parameter")
        elif _kind(arr) == "HIRMap":
            if [_param_index(a, params) for a in arr.arrays] != list(range(len(params))):
                raise _unsupported("the folded map must take the parameters in order")
            if arr.cell_shape:
                raise _unsupported("folds of cell maps")
            premap, n_in = _map_expr(arr, [InputExpr(i) for i in range(len(params))]), len(params)
        else:
            raise _unsupported(f"fold of {_kind(arr)}")
        shapes = {s for _, s in in_types}
        if len(shapes) != 1 or len(next(iter(shapes))) != 1:
            raise _unsupported("whole-array folds take rank-1 operands of one shape")
        sp = fold_spec(op=op, init=init, mode="all", dtype=out_code, premap=premap, n_inputs=n_in,
                       premap_in_dtypes=in_codes if premap is not None else None)
        return SpecModule({name: FoldSpec(sp)}), [_meta(name, in_codes, out_code, (), reduction=True)]

    if k == "HIRScan":
        op, init = _fold_parts(body)
        if len(params) != 1 or _param_index(body.array, params) != 0:
            raise _unsupported("a scan must take its one parameter")
        code, shape = in_types[0]
        if code not in (L.F32, L.I32):
            raise _unsupported("scans of f32 or i32")
        if len(shape) > 1 and (body.exclusive or body.right):
            raise _unsupported("exclusive and right scans of rank >= 2")
        sp = scan_spec(op=op, init=init, dtype=code, exclusive=bool(body.exclusive), right=bool(body.right))
        return SpecModule({name: ScanSpec(sp)}), [_meta(name, in_codes, code, shape)]

    if k == "HIRAppend":
        if len(params) != 2:
            raise _unsupported("append of two parameters")
        left, right = _param_index(body.left, params), _param_index(body.right, params)
        if {left, right} != {0, 1} or in_codes[0] != in_codes[1]:
            raise _unsupported("append of the two parameters, same element type")
        out_code, out_shape = _array(function.return_type)
        return (SpecModule({name: AppendSpec(out_code, left)}), [_meta(name, in_codes, out_code, out_shape)])

    if k == "HIRRotate":
        if len(params) != 1 or _param_index(body.array, params) != 0:
            raise _unsupported("rotate of its one parameter")
        if _kind(body.shift) != "StaticDim":
            raise _unsupported("rotate by a static shift")
        code, shape = in_types[0]
        return SpecModule({name: RotateSpec(code, int(body.shift.value))}), [_meta(name, in_codes, code, shape)]

    if k in ("HIRSort", "HIRGrade"):
        if len(params) != 1 or _param_index(body.array, params) != 0:
            raise _unsupported(f"{k[3:].lower()} of its one parameter")
        code, shape = in_types[0]
        if code not in (L.F32, L.I32) or len(shape) not in (1, 2):
            raise _unsupported("sort and grade of rank-1 or rank-2 f32 / i32 arrays")
        grade = k == "HIRGrade"
        out_code = L.I32 if grade else code
        return SpecModule({name: SortSpec(code, grade)}), [_meta(name, in_codes, out_code, shape)]

    raise _unsupported(f"function bodies of kind {k}")


def _cell_fold(name: str, params: list, in_types: list, lam: object, out_code: int,
               out_shape: tuple[int, ...]) -> tuple[SpecModule, list[KernelMeta]]:
    fold = lam.body
    op, init = _fold_parts(fold)
    cell_names = [p.name for p in lam.params]
    arr = fold.array
    in_codes = [c for c, _ in in_types]
    if _kind(arr) == "HIRVar":
        if len(params) != 1 or arr.name != cell_names[0]:
            raise _unsupported("a cell fold folds its cell")
        premap, n_in = None, 1
    elif _kind(arr) == "HIRMap":
        if [a.name if _kind(a) == "HIRVar" else None for a in arr.arrays] != cell_names:
            raise _unsupported("the cell map must take the cells in order")
        if arr.cell_shape:
            raise _unsupported("nested cell maps")
        premap, n_in = _map_expr(arr, [InputExpr(i) for i in range(len(params))]), len(params)
    else:
        raise _unsupported(f"cell fold of {_kind(arr)}")
    shapes = {s for _, s in in_types}
    if len(shapes) != 1:
        raise _unsupported("cell-fold operands of one shape")
    shape = next(iter(shapes))
    cell_rank = len(shape) - len(out_shape)
    if cell_rank < 1 or shape[: len(out_shape)] != out_shape:
        raise _unsupported("the result must be the frame of the operands")
    sp = fold_spec(op=op, init=init, mode="cell", cell_rank=cell_rank, dtype=out_code, premap=premap, n_inputs=n_in,
                   premap_in_dtypes=in_codes if premap is not None else None)
    return SpecModule({name: FoldSpec(sp)}), [_meta(name, in_codes, out_code, out_shape)]


def compile_function_source_to_b200_artifacts(source: str, function_name: str, param_types: tuple[Any, ...], *,
                                              include_prelude: bool = True, kernel_name: str | None = None,
                                              syntax: str = "ml") -> tuple[SpecModule, list[KernelMeta], Any]:
    """The reference's front end (remora.compiler.compile_function_source)
    followed by ``specs_from_hir``: the counterpart of
    compile_function_source_to_supported_gpu_artifacts
    (remora/compiler.py:226-272).  Needs the reference package on the path."""
    from remora.compiler import compile_function_source  # the reference's front end

    artifact = compile_function_source(source, function_name, param_types, verify=False,
                                       include_prelude=include_prelude, syntax=syntax)
    module, metas = specs_from_hir(artifact.hir_function, kernel_name or f"remora_{function_name}")
    return module, metas, artifact.hir_function
