"""Whole-program execution on the device.

The reference runs a whole compiled program on the GPU with
``execute_program_from_ptx`` (remora/executor.py:192-306): every kernel of
the IREE module in order over two ping-pong buffers, a synchronisation after
each launch, and, for a scalar result, the last nonzero word of the buffer.
Here a program becomes a ``Plan``: device buffers (constants, inputs, views
of other buffers) and an ordered list of library calls over them.
``plan_from_hir`` builds it from the reference compiler's HIR program
(nodes matched by class name and field, as in ``reference_codegen``);
``execute_plan`` uploads the constants and inputs once, enqueues every call on
one stream, synchronises once and copies the result back.  Intermediates
stay in device memory for the whole program.

What the planner accepts (anything else raises ``RemoraUnsupportedError``):
let bindings, array literals and ``iota``; maps over arrays and captured
scalars with primitive, section, lambda or named-function bodies (fused into
one program each), including cell maps whose body folds its cell; whole and
leading-axis (array-accumulator) folds with + or * (and && / || over bools);
scans; append, rotate, sort, grade; reverse, transpose, static indexing and
slices as strided views; ``if`` on a scalar condition known at plan time, and
an elementwise ``if`` over arrays.  Scalar arithmetic on literals is folded
when the plan is built, as a compiler folds constants.

Plans are plain data (``Plan.to_record`` / ``Plan.from_record``), so a plan
built where the reference compiler is importable can be run where it is not.
"""

from __future__ import annotations

import ctypes
import dataclasses
from dataclasses import dataclass, field
from typing import Any

import numpy as np

from remora_b200 import _lib as L
from remora_b200.codegen import fold_spec, scan_spec
from remora_b200.errors import RemoraShapeError, RemoraUnsupportedError
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

_NP = {L.F32: np.float32, L.I32: np.int32, L.BOOL: np.bool_}
_NAME = {L.F32: "float32", L.I32: "int32", L.BOOL: "bool"}
_CODE = {v: k for k, v in _NAME.items()}
_ELEM = {"float": L.F32, "int": L.I32, "bool": L.BOOL}
_ARITH, _CMP, _LOGIC, _UNARY = {"+", "-", "*", "/"}, {"<", "<=", ">", ">=", "==", "!="}, {"&&", "||"}, {"exp", "log"}


def _unsupported(msg: str) -> RemoraUnsupportedError:
    return RemoraUnsupportedError(f"B200 program plan: {msg}")


def _kind(node: object) -> str:
    return type(node).__name__


# ------------------------------------------------------------------ plans
@dataclass
class Buffer:
    shape: tuple[int, ...]
    dtype: int
    const: np.ndarray | None = None  # uploaded once
    input: int | None = None  # filled from the caller's k-th input
    # a strided view of another buffer: (base id, element offset, element strides)
    view: tuple[int, int, tuple[int, ...]] | None = None


@dataclass
class Plan:
    buffers: list[Buffer] = field(default_factory=list)
    steps: list[dict] = field(default_factory=list)
    result: int = -1
    # a plan with several results (a loss and its gradients) lists them all
    results: list[int] = field(default_factory=list)

    def to_record(self) -> dict:
        bufs = []
        for b in self.buffers:
            r: dict[str, Any] = {"shape": list(b.shape), "dtype": _NAME[b.dtype]}
            if b.const is not None:
                r["const"] = np.ascontiguousarray(b.const, dtype=_NP[b.dtype]).tobytes().hex()
            if b.input is not None:
                r["input"] = b.input
            if b.view is not None:
                r["view"] = [b.view[0], b.view[1], list(b.view[2])]
            bufs.append(r)
        steps = []
        for s in self.steps:
            t = dict(s)
            for key in ("program", "spec"):
                if key in t:
                    t[key] = bytes(t[key]).hex()
            steps.append(t)
        rec = {"buffers": bufs, "steps": steps, "result": self.result}
        if self.results:
            rec["results"] = list(self.results)
        return rec

    @classmethod
    def from_record(cls, rec: dict) -> "Plan":
        p = cls()
        for r in rec["buffers"]:
            code = _CODE[r["dtype"]]
            shape = tuple(r["shape"])
            const = None
            if "const" in r:
                const = np.frombuffer(bytes.fromhex(r["const"]), dtype=_NP[code]).reshape(shape).copy()
            view = None
            if "view" in r:
                view = (int(r["view"][0]), int(r["view"][1]), tuple(int(v) for v in r["view"][2]))
            p.buffers.append(Buffer(shape, code, const, r.get("input"), view))
        for s in rec["steps"]:
            t = dict(s)
            if "program" in t:
                t["program"] = L.RemoraMapProgram.from_buffer_copy(bytes.fromhex(t["program"]))
            if "spec" in t:
                cls_ = {"fold": L.RemoraFoldSpec, "array_fold": L.RemoraFoldSpec, "scan": L.RemoraScanSpec}[t["op"]]
                t["spec"] = cls_.from_buffer_copy(bytes.fromhex(t["spec"]))
            p.steps.append(t)
        p.result = int(rec["result"])
        p.results = [int(r) for r in rec.get("results", [])]
        return p


# --------------------------------------------------------------- planner
# Values while planning: ("buf", id) an array (or a rank-0 device scalar),
# ("const", value, code) a scalar known at plan time, ("func", params, body)
# a function value.
def _scalar_code(t: object) -> int:
    if _kind(t) != "ScalarType" or t.name not in _ELEM:
        raise _unsupported(f"element type {t!r}")
    return _ELEM[t.name]


def _shape(t: object) -> tuple[int, ...]:
    if _kind(t) == "ScalarType":
        return ()
    if _kind(t) != "ArrayType":
        raise _unsupported(f"type {t!r}")
    out = []
    for d in t.shape:
        if _kind(d) != "StaticDim":
            raise _unsupported("shapes must be static")
        out.append(int(d.value))
    return tuple(out)


def _elem(t: object) -> int:
    return _scalar_code(t.element if _kind(t) == "ArrayType" else t)


def _base_op(op: str) -> str:
    for base in sorted(_ARITH | _CMP | _LOGIC | _UNARY, key=len, reverse=True):
        if op == base or (op.startswith(base) and op[len(base):] in ("f", "i", "b")):
            return base
    raise _unsupported(f"primitive {op!r}")


def _const_eval(op: str, args: list[tuple[Any, int]], out_code: int) -> tuple[Any, int]:
    """Plan-time folding of a scalar primitive on literals, in the result's
    element type (f32 ops rounded once, like the device)."""
    vals = [np.asarray(v, dtype=_NP[c]) for v, c in args]
    if op in _ARITH:
        a, b = (v.astype(_NP[out_code]) for v in vals)
        if op == "/" and out_code == L.I32:
            r = np.int32(0) if b == 0 else np.int32(int(a) // int(b) if a * b >= 0 else -(abs(int(a)) // abs(int(b))))
        else:
            r = {"+": np.add, "-": np.subtract, "*": np.multiply, "/": np.divide}[op](a, b)
        return r.astype(_NP[out_code]).item(), out_code
    if op in _CMP:
        ct = L.F32 if any(c == L.F32 for _, c in args) else L.I32
        a, b = (v.astype(_NP[ct]) for v in vals)
        fn = {"<": np.less, "<=": np.less_equal, ">": np.greater, ">=": np.greater_equal, "==": np.equal,
              "!=": np.not_equal}[op]
        return bool(fn(a, b)), L.BOOL
    if op in _LOGIC:
        a, b = (bool(v) for v in vals)
        return (a and b) if op == "&&" else (a or b), L.BOOL
    if op == "-" and len(vals) == 1:
        return (-vals[0]).astype(_NP[out_code]).item(), out_code
    raise _unsupported(f"plan-time folding of {op}")


class _Planner:
    def __init__(self, functions: dict[str, Any]) -> None:
        self.functions = functions
        self.plan = Plan()

    # -------------------------------------------------------- buffers
    def buf(self, shape: tuple[int, ...], code: int, **kw: Any) -> int:
        self.plan.buffers.append(Buffer(tuple(shape), code, **kw))
        return len(self.plan.buffers) - 1

    def shape_of(self, b: int) -> tuple[int, ...]:
        return self.plan.buffers[b].shape

    def code_of(self, b: int) -> int:
        return self.plan.buffers[b].dtype

    def as_buf(self, v: tuple) -> int:
        if v[0] == "buf":
            return v[1]
        if v[0] == "const":
            return self.buf((), v[2], const=np.asarray(v[1], dtype=_NP[v[2]]))
        raise _unsupported("a function where an array is needed")

    def strides_of(self, b: int) -> tuple[int, tuple[int, ...], int]:
        """(base buffer, element offset, element strides) of b."""
        bb = self.plan.buffers[b]
        if bb.view is not None:
            return bb.view
        shape, st, acc = bb.shape, [], 1
        for d in reversed(shape):
            st.append(acc)
            acc *= d
        return b, 0, tuple(reversed(st))

    def view(self, b: int, shape: tuple[int, ...], offset: int, strides: tuple[int, ...]) -> int:
        base, off0, _ = self.strides_of(b)
        return self.buf(shape, self.code_of(b), view=(base, off0 + offset, tuple(strides)))

    # ------------------------------------------------------- lowering
    def lower(self, node: object, env: dict[str, tuple]) -> tuple:
        k = _kind(node)
        if k == "HIRLit":
            return ("const", node.value, _scalar_code(node.type))
        if k == "HIRVar":
            if node.name in env:
                return env[node.name]
            if node.name in self.functions:
                f = self.functions[node.name]
                return ("func", [p.name for p in f.params], f.body)
            raise _unsupported(f"unbound name {node.name}")
        if k == "HIRLet":
            return self.lower(node.body, {**env, node.name: self.lower(node.value, env)})
        if k == "HIRArrayLit":
            return ("buf", self.buf(_shape(node.result_type), _elem(node.result_type),
                                    const=self._literal(node, env)))
        if k == "HIRIota":
            n = int(node.size.value) if _kind(node.size) == "StaticDim" else None
            if n is None:
                raise _unsupported("iota of a static size")
            return ("buf", self.buf((n,), L.I32, const=np.arange(n, dtype=np.int32)))
        if k == "HIRCall":
            f = self.functions.get(node.func_name)
            if f is None:
                raise _unsupported(f"call of unknown function {node.func_name}")
            args = [self.lower(a, env) for a in node.args]
            return self.lower(f.body, {**env, **{p.name: a for p, a in zip(f.params, args)}})
        if k in ("HIRPrimOp", "HIRIf", "HIRCast"):
            return self.scalar_or_elementwise(node, env)
        if k == "HIRMap":
            return self.lower_map(node, env)
        if k == "HIRFold":
            return self.lower_fold(node, env)
        if k == "HIRScan":
            return self.lower_scan(node, env)
        if k == "HIRAppend":
            a, b = self.as_buf(self.lower(node.left, env)), self.as_buf(self.lower(node.right, env))
            out = self.buf(_shape(node.result_type), _elem(node.result_type))
            self.plan.steps.append({"op": "append", "a": a, "b": b, "out": out})
            return ("buf", out)
        if k == "HIRRotate":
            a = self.as_buf(self.lower(node.array, env))
            out = self.buf(self.shape_of(a), self.code_of(a))
            self.plan.steps.append({"op": "rotate", "in": a, "out": out, "shift": int(node.shift.value)})
            return ("buf", out)
        if k in ("HIRSort", "HIRGrade"):
            a = self.as_buf(self.lower(node.array, env))
            grade = k == "HIRGrade"
            out = self.buf(self.shape_of(a), L.I32 if grade else self.code_of(a))
            self.plan.steps.append({"op": "grade" if grade else "sort", "in": a, "out": out})
            return ("buf", out)
        if k == "HIRReverse":
            a = self.as_buf(self.lower(node.array, env))
            shape = self.shape_of(a)
            _, _, st = self.strides_of(a)
            return ("buf", self.view(a, shape, (shape[0] - 1) * st[0], (-st[0], *st[1:])))
        if k == "HIRTranspose":
            a = self.as_buf(self.lower(node.array, env))
            shape = self.shape_of(a)
            _, _, st = self.strides_of(a)
            return ("buf", self.view(a, tuple(reversed(shape)), 0, tuple(reversed(st))))
        if k == "HIRIndex":
            return self.lower_index(node, env)
        if k == "HIRReshape":
            a = self.as_buf(self.lower(node.array, env))
            shape = _shape(node.result_type)
            base, off, st = self.strides_of(a)
            contiguous = st == self.strides_of(self.buf(self.shape_of(a), self.code_of(a)))[2]
            if not contiguous:
                a = self.emit_map(InputExpr(0), [a], self.shape_of(a), self.code_of(a))
            strides, acc = [], 1
            for d in reversed(shape):
                strides.append(acc)
                acc *= d
            return ("buf", self.view(a, shape, 0, tuple(reversed(strides))))
        raise _unsupported(f"{k} nodes")

    def _literal(self, node: object, env: dict) -> np.ndarray:
        def rec(n: object) -> Any:
            if _kind(n) == "HIRArrayLit":
                return [rec(e) for e in n.elements]
            v = self.lower(n, env)
            if v[0] != "const":
                raise _unsupported("array literals of plan-time scalars")
            return v[1]

        return np.asarray(rec(node), dtype=_NP[_elem(node.result_type)])

    def lower_index(self, node: object, env: dict) -> tuple:
        a = self.as_buf(self.lower(node.array, env))
        shape = self.shape_of(a)
        _, _, st = self.strides_of(a)
        off, out_shape, out_st = 0, [], []
        for d, ix in enumerate(node.indices):
            if _kind(ix) == "HIRSlice":
                start, end = int(ix.start), int(ix.end)
                off += start * st[d]
                out_shape.append(end - start)
                out_st.append(st[d])
            else:
                v = self.lower(ix, env)
                if v[0] != "const":
                    raise _unsupported("indices known at plan time")
                i = int(v[1])
                if not 0 <= i < shape[d]:
                    raise _unsupported(f"index {i} outside axis of {shape[d]}")
                off += i * st[d]
        for d in range(len(node.indices), len(shape)):
            out_shape.append(shape[d])
            out_st.append(st[d])
        return ("buf", self.view(a, tuple(out_shape), off, tuple(out_st)))

    # ---- elementwise expressions over buffers and constants
    def expr(self, node: object, env: dict, operands: list[int]) -> tuple[Expr, int]:
        """(expression, element code) of a scalar-valued HIR node; array or
        device-scalar operands are appended to `operands` as inputs."""
        k = _kind(node)
        if k == "HIRLit":
            return ConstantExpr(int(node.value) if isinstance(node.value, bool) else node.value), \
                _scalar_code(node.type)
        if k == "HIRVar" and node.name in env and env[node.name][0] == "expr":
            return env[node.name][1], env[node.name][2]
        if k == "HIRVar" and node.name in env and env[node.name][0] == "const":
            v = env[node.name]
            return ConstantExpr(int(v[1]) if isinstance(v[1], bool) else v[1]), v[2]
        if k == "HIRVar" and node.name in env and env[node.name][0] == "buf":
            b = env[node.name][1]
            operands.append(b)
            return InputExpr(len(operands) - 1), self.code_of(b)
        cell = self._cell_operand(node, env)
        if cell is not None:
            operands.append(cell)
            return InputExpr(len(operands) - 1), self.code_of(cell)
        if k == "HIRIf":
            c, _ = self.expr(node.condition, env, operands)
            t, tc = self.expr(node.then_branch, env, operands)
            e, _ = self.expr(node.else_branch, env, operands)
            return SelectExpr(c, t, e), tc
        if k == "HIRPrimOp":
            op = _base_op(node.op)
            args = [self.expr(a, env, operands) for a in node.args]
            code = _elem(node.result_type)
            es = [a for a, _ in args]
            if op in _UNARY:
                return UnaryExpr(op, es[0]), code
            if op == "-" and len(es) == 1:
                return UnaryExpr("neg", es[0]), code
            if op in _ARITH:
                return BinaryExpr(op, *es), code
            if op in _CMP:
                return CmpExpr(op, *es), code
            if op in _LOGIC:
                return LogicExpr(op, *es), code
            raise _unsupported(f"primitive {op}")
        # any other array-valued node: computed first, then an operand
        v = self.lower(node, env)
        if v[0] == "const":
            return ConstantExpr(int(v[1]) if isinstance(v[1], bool) else v[1]), v[2]
        if v[0] == "buf":
            operands.append(v[1])
            return InputExpr(len(operands) - 1), self.code_of(v[1])
        raise _unsupported(f"{k} in an elementwise expression")

    def const_of(self, node: object, env: dict) -> tuple | None:
        """The value of a scalar node if it is known at plan time."""
        k = _kind(node)
        if k == "HIRLit":
            return ("const", node.value, _scalar_code(node.type))
        if k == "HIRVar":
            v = env.get(node.name)
            return v if v is not None and v[0] == "const" else None
        if k == "HIRPrimOp":
            args = [self.const_of(a, env) for a in node.args]
            if all(a is not None for a in args):
                return ("const", *_const_eval(_base_op(node.op), [a[1:] for a in args], _elem(node.result_type)))
            return None
        if k == "HIRIf":
            c = self.const_of(node.condition, env)
            if c is None:
                return None
            return self.const_of(node.then_branch if c[1] else node.else_branch, env)
        if k == "HIRCast":
            v = self.const_of(node.value, env)
            if v is None:
                return None
            to = _scalar_code(node.to_type)
            return ("const", np.asarray(v[1], dtype=_NP[v[2]]).astype(_NP[to]).item(), to)
        return None

    def apply_func(self, func: object, env: dict, arg_exprs: list[tuple[Expr, int]], operands: list[int],
                   result_code: int) -> Expr:
        """The expression of a scalar function (primitive, section, lambda or
        named function) applied to argument expressions."""
        k = _kind(func)
        if k == "HIRPrimCallable":
            op = _base_op(func.op)
            args = [e for e, _ in arg_exprs]
            if func.left_arg is not None:
                args = [self.expr(func.left_arg, env, operands)[0], *args]
            if func.right_arg is not None:
                args = [*args, self.expr(func.right_arg, env, operands)[0]]
            if op in _UNARY:
                return UnaryExpr(op, args[0])
            if op == "-" and len(args) == 1:
                return UnaryExpr("neg", args[0])
            make = BinaryExpr if op in _ARITH else CmpExpr if op in _CMP else LogicExpr
            return make(op, *args)
        if k == "HIRLambda":
            names, body = [p.name for p in func.params], func.body
        elif k == "HIRVar":
            v = self.lower(func, env)
            if v[0] != "func":
                raise _unsupported("mapping a non-function")
            names, body = v[1], v[2]
        else:
            raise _unsupported(f"{k} as a scalar function")
        inner = {**env, **{n: ("expr", e, c) for n, (e, c) in zip(names, arg_exprs)}}
        return self.expr(body, inner, operands)[0]

    def emit_map(self, expr: Expr, operands: list[int], shape: tuple[int, ...], out_code: int) -> int:
        in_codes = [self.code_of(b) for b in operands]
        compute = L.F32 if L.F32 in in_codes + [out_code] else L.I32 if L.I32 in in_codes + [out_code] else L.BOOL
        if not operands:
            raise _unsupported("a map with no array operand")
        prog = compile_program(expr, len(operands), compute=compute, out=out_code, in_dtypes=in_codes)
        out = self.buf(shape, out_code)
        self.plan.steps.append({"op": "map", "program": prog, "ins": list(operands), "out": out})
        return out

    def scalar_or_elementwise(self, node: object, env: dict) -> tuple:
        c = self.const_of(node, env)
        if c is not None:
            return c
        if _kind(node) == "HIRIf":
            cond = self.const_of(node.condition, env)
            if cond is not None:
                return self.lower(node.then_branch if cond[1] else node.else_branch, env)
        # elementwise over arrays and device scalars: one fused map
        operands: list[int] = []
        e, code = self.expr(node, env, operands)
        return ("buf", self.emit_map(e, operands, _shape(node.result_type), code))

    def lower_map(self, node: object, env: dict) -> tuple:
        arrays = [self.as_buf(self.lower(a, env)) for a in node.arrays]
        shape = _shape(node.result_type)
        func = node.func
        if node.cell_shape:
            return self.lower_cell_map(node, env, arrays, shape)
        operands = list(arrays)
        arg_exprs = [(InputExpr(i), self.code_of(b)) for i, b in enumerate(arrays)]
        # captured scalars and arrays of the body become extra operands
        expr = self.apply_func(func, env, arg_exprs, operands, _elem(node.result_type))
        return ("buf", self.emit_map(expr, operands, shape, _elem(node.result_type)))

    def _func_parts(self, func: object, env: dict) -> tuple[list[str], object]:
        if _kind(func) == "HIRLambda":
            return [p.name for p in func.params], func.body
        v = self.lower(func, env)
        if v[0] != "func":
            raise _unsupported("a cell map of a non-function")
        return v[1], v[2]

    def lower_cell_map(self, node: object, env: dict, arrays: list[int], shape: tuple[int, ...]) -> tuple:
        """``map f xs`` over cells of rank >= 1 whose result per cell is a
        scalar: f's body is a fold of the cell, or an elementwise expression
        of folds of the cell and of its elements at indices known at plan
        time (``\\row -> row[0] + row[1]``).  The cell parameter stands for
        the whole array; each use of it becomes a frame-shaped operand (a
        cell-fold step, or a strided view), and the body one fused map."""
        names, body = self._func_parts(node.func, env)
        if len(arrays) != 1:
            raise _unsupported("cell maps of one array")
        cell_rank = len(node.cell_shape)
        frame = self.shape_of(arrays[0])[:len(self.shape_of(arrays[0])) - cell_rank]
        dot = self.lifted_dot(names[0], body, env, arrays[0], cell_rank)
        if dot is not None:
            return ("buf", dot)
        if tuple(shape) != tuple(frame):
            raise _unsupported("cell maps other than one scalar per cell")
        inner = {**env, names[0]: ("cell", arrays[0], cell_rank)}
        if _kind(body) == "HIRFold":
            return ("buf", self.cell_fold(body, inner))
        operands: list[int] = []
        e, code = self.expr(body, inner, operands)
        if not operands:
            raise _unsupported("a cell map whose body does not use its cell")
        return ("buf", self.emit_map(e, operands, tuple(frame), code))

    # ---- lifted dot products: rows times a vector, rows times rows
    def _resolve(self, node: object, subst: dict) -> tuple[object, dict]:
        """What ``node`` stands for once let-bound and argument names are
        followed (the front end inlines ``dot``/``sum`` as a chain of lets):
        (node, its names) or (("free", name), ...) for a name bound outside."""
        while True:
            k = _kind(node)
            if k == "HIRVar":
                if node.name not in subst:
                    return ("free", node.name), subst
                node, subst = subst[node.name]
            elif k == "HIRLet":
                subst = {**subst, node.name: (node.value, subst)}
                node = node.body
            elif k == "HIRCall" and node.func_name in self.functions:
                f = self.functions[node.func_name]
                subst = {p.name: (a, subst) for p, a in zip(f.params, node.args)}
                node = f.body
            else:
                return node, subst

    def _match_dot(self, body: object) -> tuple[set[str], float] | None:
        """({a, b}, init) when ``body`` is ``fold (+) init (map (*) a b)`` of
        two names bound outside it (the prelude's ``dot a b``), else None."""
        node, s = self._resolve(body, {})
        if not _kind(node) == "HIRFold":
            return None
        f = node.func
        if _kind(f) != "HIRPrimCallable" or _base_op(f.op) != "+" or f.left_arg is not None or \
                f.right_arg is not None:
            return None
        init, _ = self._resolve(node.init, s)
        if _kind(init) != "HIRLit" or isinstance(init.value, bool):
            return None
        m, s2 = self._resolve(node.array, s)
        if _kind(m) not in ("HIRMap", "HIRApply") or m.cell_shape or len(m.arrays) != 2:
            return None
        g = m.func
        if _kind(g) == "HIRPrimCallable":
            if _base_op(g.op) != "*" or g.left_arg is not None or g.right_arg is not None:
                return None
        elif _kind(g) == "HIRLambda":
            b = g.body
            if _kind(b) != "HIRPrimOp" or _base_op(b.op) != "*" or \
                    sorted(getattr(a, "name", "") for a in b.args) != sorted(p.name for p in g.params):
                return None
        else:
            return None
        leaves = [self._resolve(a, s2)[0] for a in m.arrays]
        if not all(isinstance(x, tuple) and x[0] == "free" for x in leaves):
            return None
        return {leaves[0][1], leaves[1][1]}, float(init.value)

    def lifted_dot(self, cell: str, body: object, env: dict, arr: int, cell_rank: int) -> int | None:
        """``map (\\row -> dot row v) A`` (a vector per row of A: a cell fold
        whose premap multiplies the row by a stride-0 view of v) or
        ``map (\\r -> map (\\c -> dot r c) B) A`` (A times B's rows: one
        3xTF32 GEMM step, the f32-accurate form of the tensor-core GEMM),
        as remora/lowering/tensor_ops.py lowers the lifted dot of the prelude
        (stdlib/prelude.rem:14); None for any other body."""
        if cell_rank != 1 or self.code_of(arr) != L.F32 or len(self.shape_of(arr)) != 2:
            return None
        m_rows, k = self.shape_of(arr)
        inner, s = self._resolve(body, {})
        if _kind(inner) in ("HIRMap", "HIRApply") and len(inner.cell_shape) == 1 and len(inner.arrays) == 1 \
                and _kind(inner.func) == "HIRLambda" and len(inner.func.params) == 1:
            match = self._match_dot(inner.func.body)
            if match is None or match[0] != {cell, inner.func.params[0].name}:
                return None
            src, s2 = self._resolve(inner.arrays[0], s)
            if isinstance(src, tuple):
                v = env.get(src[1])
                if v is None or v[0] != "buf":
                    return None
                b = v[1]
            elif not s2:
                b = self.as_buf(self.lower(src, env))
            else:
                return None
            if self.code_of(b) != L.F32 or len(self.shape_of(b)) != 2 or self.shape_of(b)[1] != k:
                return None
            n = self.shape_of(b)[0]
            _, _, st = self.strides_of(b)
            bt = self.view(b, (k, n), 0, (st[1], st[0]))  # the GEMM's B: columns are the rows of b
            out = self.buf((m_rows, n), L.F32)
            self.plan.steps.append({"op": "gemm", "a": arr, "b": bt, "out": out, "precision": L.PREC_3XTF32})
            init = match[1]
        else:
            match = self._match_dot(body)
            if match is None or cell not in match[0] or len(match[0]) != 2:
                return None
            (other,) = match[0] - {cell}
            v = env.get(other)
            if v is None or v[0] != "buf" or self.code_of(v[1]) != L.F32 or self.shape_of(v[1]) != (k,):
                return None
            _, _, st = self.strides_of(v[1])
            vb = self.view(v[1], (m_rows, k), 0, (0, st[0]))  # v repeated for every row
            sp = fold_spec(op="+", init=match[1], mode="cell", cell_rank=1, dtype=L.F32,
                           premap=BinaryExpr("*", InputExpr(0), InputExpr(1)), n_inputs=2)
            out = self.buf((m_rows,), L.F32)
            self.plan.steps.append({"op": "fold", "spec": sp, "ins": [arr, vb], "out": out})
            return out
        if init != 0.0:
            out = self.emit_map(BinaryExpr("+", InputExpr(0), ConstantExpr(init)), [out], self.shape_of(out), L.F32)
        return out

    def _cell_operand(self, node: object, env: dict) -> int | None:
        """A frame-shaped buffer for a use of a cell parameter inside a cell
        map's body (an index at plan-time positions, or a fold), else None."""
        k = _kind(node)
        arr = getattr(node, "array", None)
        if k == "HIRFold":
            return self.cell_fold(node, env) if self._cell_of(arr, env)[0] is not None else None
        if k != "HIRIndex" or _kind(arr) != "HIRVar" or env.get(arr.name, ("",))[0] != "cell":
            return None
        _, b, cell_rank = env[arr.name]
        shape = self.shape_of(b)
        fr = len(shape) - cell_rank
        if len(node.indices) != cell_rank or any(_kind(ix) == "HIRSlice" for ix in node.indices):
            raise _unsupported("cell indices that pick one element of the cell")
        _, _, st = self.strides_of(b)
        off = 0
        for d, ix in enumerate(node.indices):
            v = self.const_of(ix, env)
            if v is None:
                raise _unsupported("cell indices known at plan time")
            i = int(v[1])
            if not 0 <= i < shape[fr + d]:
                raise _unsupported(f"index {i} outside axis of {shape[fr + d]}")
            off += i * st[fr + d]
        return self.view(b, shape[:fr], off, st[:fr])

    def _cell_of(self, node: object, env: dict) -> tuple[tuple | None, Expr | None]:
        """(cell, premap) for the array a cell fold folds: the cell parameter
        itself (premap None), or an elementwise map over it alone
        (``map (\\v -> v * v) row``), whose function becomes the fold's
        premap; (None, None) for anything else."""
        k = _kind(node)
        if k == "HIRVar":
            cell = env.get(node.name)
            return (cell, None) if cell is not None and cell[0] == "cell" else (None, None)
        if k not in ("HIRMap", "HIRApply") or node.cell_shape or not node.arrays or \
                any(_kind(a) != "HIRVar" or env.get(a.name, ("",))[0] != "cell" for a in node.arrays) or \
                len({env[a.name][1] for a in node.arrays}) != 1:
            return None, None
        cell = env[node.arrays[0].name]
        code = self.code_of(cell[1])
        if code == L.BOOL:
            raise _unsupported("a fold of a map over a bool cell")
        operands: list[int] = []
        e = self.apply_func(node.func, env, [(InputExpr(0), code)] * len(node.arrays), operands,
                            _elem(node.result_type))
        if operands:
            raise _unsupported("a map inside a cell fold that reads more than its cell")
        return cell, e

    def cell_fold(self, body: object, env: dict) -> int:
        """A fold of a cell parameter, or of an elementwise map over it: one
        cell-fold step over the whole array (the map fused as its premap)."""
        op, init, code = self.fold_op(body, env)
        cell, premap = self._cell_of(body.array, env)
        if cell is None:
            raise _unsupported("a cell fold folds its cell")
        if init[0] != "const" or op not in ("+", "*"):
            raise _unsupported("cell folds with + or * and a literal init")
        _, b, cell_rank = cell
        in_code = self.code_of(b)
        if premap is None and in_code != code:
            premap = InputExpr(0)
        sp = fold_spec(op=op, init=init[1], mode="cell", cell_rank=cell_rank, dtype=code, premap=premap,
                       premap_in_dtypes=[in_code] if premap is not None else None)
        shape = self.shape_of(b)
        out = self.buf(shape[:len(shape) - cell_rank], code)
        self.plan.steps.append({"op": "fold", "spec": sp, "ins": [b], "out": out})
        return out

    def fold_op(self, node: object, env: dict) -> tuple[str, Any, int]:
        """(op, init, accumulator code) of a fold with a + / * / && / || step."""
        func = node.func
        code = _elem(node.result_type)
        if _kind(func) == "HIRPrimCallable" and func.left_arg is None and func.right_arg is None:
            op = _base_op(func.op)
        else:
            names, body = self._func_parts(func, env)
            if _kind(body) == "HIRPrimOp" and len(body.args) == 2 and \
                    [getattr(a, "name", None) for a in body.args] == names:
                op = _base_op(body.op)
            elif _kind(body) == "HIRMap" and _kind(body.func) == "HIRPrimCallable" and \
                    [getattr(a, "name", None) for a in body.arrays] == names:
                op = _base_op(body.func.op)  # an elementwise accumulator step (array fold)
            else:
                raise _unsupported("fold steps other than acc op x")
        init = self.lower(node.init, env)
        if op not in ("+", "*", "&&", "||"):
            raise _unsupported(f"fold with {op}")
        return op, init, code

    def lower_fold(self, node: object, env: dict) -> tuple:
        op, init, code = self.fold_op(node, env)
        arr = self.as_buf(self.lower(node.array, env))
        in_code = self.code_of(arr)
        if op in ("&&", "||"):
            # over bools: && is a product and || a sum of 0/1 in i32, then != 0
            acc_code, op2 = L.I32, ("*" if op == "&&" else "+")
        else:
            acc_code, op2 = code, op
        if in_code == L.BOOL:
            # the fold kernels read f32 / i32: widen the bools first
            arr = self.emit_map(InputExpr(0), [arr], self.shape_of(arr), L.I32)
            in_code = L.I32
        if init[0] == "buf" and self.shape_of(init[1]) == () and len(self.shape_of(arr)) == 1:
            # a scalar init known only at run time (a parameter, an earlier
            # result): fold from the identity, then combine with the init
            ib = init[1]
            if self.code_of(ib) != acc_code:
                raise _unsupported("a fold init of another element type")
            sp = fold_spec(op=op2, init=(0 if op2 == "+" else 1), mode="all", dtype=acc_code,
                           premap=InputExpr(0) if in_code != acc_code else None,
                           premap_in_dtypes=[in_code] if in_code != acc_code else None)
            total = self.buf((), acc_code)
            self.plan.steps.append({"op": "fold", "spec": sp, "ins": [arr], "out": total})
            out = self.emit_map(BinaryExpr(op2, InputExpr(0), InputExpr(1)), [ib, total], (), acc_code)
        elif init[0] == "const":
            if len(self.shape_of(arr)) != 1:
                raise _unsupported("scalar-init folds of rank >= 2 arrays")
            premap = InputExpr(0) if in_code != acc_code else None
            sp = fold_spec(op=op2, init=int(init[1]) if acc_code != L.F32 else float(init[1]), mode="all",
                           dtype=acc_code, premap=premap, premap_in_dtypes=[in_code] if premap is not None else None)
            out = self.buf((), acc_code)
            self.plan.steps.append({"op": "fold", "spec": sp, "ins": [arr], "out": out})
        else:
            ib = self.as_buf(init)
            if in_code != acc_code or self.code_of(ib) != acc_code:
                raise _unsupported("array folds in one element type")
            sp = fold_spec(op=op2, dtype=acc_code)
            out = self.buf(self.shape_of(ib), acc_code)
            self.plan.steps.append({"op": "array_fold", "spec": sp, "in": arr, "init": ib, "out": out})
        if acc_code != code:
            out = self.emit_map(CmpExpr("!=", InputExpr(0), ConstantExpr(0)), [out], self.shape_of(out), code)
        return ("buf", out)

    def lower_scan(self, node: object, env: dict) -> tuple:
        op, init, code = self.fold_op(node, env)
        arr = self.as_buf(self.lower(node.array, env))
        if init[0] != "const" or op not in ("+", "*") or self.code_of(arr) != code:
            raise _unsupported("scans with + or *, a literal init, one element type")
        sp = scan_spec(op=op, init=init[1], dtype=code, exclusive=bool(node.exclusive), right=bool(node.right))
        out = self.buf(self.shape_of(arr), code)
        self.plan.steps.append({"op": "scan", "spec": sp, "in": arr, "out": out})
        return ("buf", out)


def plan_from_hir(program: object) -> Plan:
    """A plan for the reference's HIRProgram (its `main` expression, with
    the program's lifted functions)."""
    if getattr(program, "main", None) is None:
        raise _unsupported("a program without a main expression")
    pl = _Planner({f.name: f for f in program.functions})
    v = pl.lower(program.main, {})
    out = pl.as_buf(v)
    if pl.plan.buffers[out].view is not None or pl.plan.buffers[out].input is not None:
        # the result is a view: one copy makes it a buffer of its own
        out = pl.emit_map(InputExpr(0), [out], pl.shape_of(out), pl.code_of(out))
    pl.plan.result = out
    return pl.plan


# ------------------------------------------------- let inlining (functions)
def _is_node(v: object) -> bool:
    return dataclasses.is_dataclass(v) and not isinstance(v, type) and type(v).__name__.startswith("HIR")


def _fields(node: object):
    """(field name, value) of the fields of a HIR node that hold nodes or lists of nodes."""
    for f in dataclasses.fields(node):
        v = getattr(node, f.name)
        if _is_node(v) or (isinstance(v, list) and any(_is_node(x) for x in v)):
            yield f.name, v


def _binds(node: object) -> set[str] | None:
    """Names a binding node binds over its ``body`` (a let its name, a
    lambda its parameters, an unbox its value and hidden index names); None
    for a node that binds nothing.  The bound names scope over ``body``
    only, never over the let's value or the unbox's boxed operand."""
    k = _kind(node)
    if k == "HIRLet":
        return {node.name}
    if k == "HIRLambda":
        return {p.name for p in node.params}
    if k == "HIRUnbox":
        return {node.value_name, *node.hidden_names}
    return None


def _children(node: object):
    for _, v in _fields(node):
        for x in (v if isinstance(v, list) else [v]):
            if _is_node(x):
                yield x


def _free(node: object) -> set[str]:
    """Names read by ``node`` that it does not bind itself."""
    if _kind(node) == "HIRVar":
        return {node.name}
    bound = _binds(node)
    out: set[str] = set()
    for fname, v in _fields(node):
        for x in (v if isinstance(v, list) else [v]):
            if _is_node(x):
                out |= (_free(x) - bound) if bound is not None and fname == "body" else _free(x)
    return out


def _uses(node: object, name: str) -> int:
    if _kind(node) == "HIRVar":
        return int(node.name == name)
    bound = _binds(node)
    n = 0
    for fname, v in _fields(node):
        if bound is not None and fname == "body" and name in bound:
            continue
        for x in (v if isinstance(v, list) else [v]):
            if _is_node(x):
                n += _uses(x, name)
    return n


def _substitute_name(node: object, name: str, value: object, value_free: set[str]) -> object | None:
    """``node`` with the free uses of ``name`` replaced by ``value``; None
    where a binder on the way would capture a name ``value`` reads, or
    where a use sits inside a lambda and ``value`` is more than a name or a
    literal (substituting it there would move array work into the
    per-cell body)."""
    k = _kind(node)
    if k == "HIRVar":
        return value if node.name == name else node
    bound = _binds(node)
    if k == "HIRLambda" and _uses(node, name) and _kind(value) not in ("HIRVar", "HIRLit"):
        return None
    changes = {}
    for fname, v in _fields(node):
        if bound is not None and fname == "body":
            if name in bound or not _uses(v, name):
                continue
            if bound & value_free:
                return None
        if isinstance(v, list):
            new = [(_substitute_name(x, name, value, value_free) if _is_node(x) else x) for x in v]
            if any(x is None for x in new):
                return None
            if any(a is not b for a, b in zip(new, v)):
                changes[fname] = new
        else:
            new = _substitute_name(v, name, value, value_free)
            if new is None:
                return None
            if new is not v:
                changes[fname] = new
    return dataclasses.replace(node, **changes) if changes else node


def _inline_lets(node: object) -> object:
    """The front end inlines called functions (the prelude's ``sum``,
    ``dot``) as chains of lets binding their parameters.  A let whose value
    is a plain name, or whose name is read once, is substituted into its
    body (unless a binder on the way rebinds a name the value reads, or the
    one use sits inside a lambda and the value is more than a name or a
    literal), so ``let xs = row in fold (+) 0.0 xs`` plans like
    ``fold (+) 0.0 row``, while ``let r = map (*) v v in map (\\row -> ... r ...) m``
    keeps ``r`` as one array computed once."""
    changes = {}
    for fname, v in _fields(node):
        changes[fname] = [(_inline_lets(x) if _is_node(x) else x) for x in v] if isinstance(v, list) \
            else _inline_lets(v)
    node = dataclasses.replace(node, **changes) if changes else node
    if _kind(node) == "HIRLet" and (_kind(node.value) == "HIRVar" or _uses(node.body, node.name) <= 1):
        inlined = _substitute_name(node.body, node.name, node.value, _free(node.value))
        if inlined is not None:
            return inlined
    return node


def plan_from_function(function: object, functions: dict[str, Any] | None = None) -> Plan:
    """A plan for one of the reference's HIR functions (``HIRFunction``, as
    remora/compiler.py:compile_function_source builds it): parameter k is
    the plan's input k (arrays, and scalars as rank-0 buffers), the body its
    steps.  ``functions`` holds other functions the body calls, by name."""
    pl = _Planner(dict(functions or {}))
    env = {}
    for k, p in enumerate(function.params):
        env[p.name] = ("buf", pl.buf(_shape(p.type), _elem(p.type), input=k))
    out = pl.as_buf(pl.lower(_inline_lets(function.body), env))
    if pl.plan.buffers[out].view is not None or pl.plan.buffers[out].input is not None:
        out = pl.emit_map(InputExpr(0), [out], pl.shape_of(out), pl.code_of(out))
    pl.plan.result = out
    return pl.plan


def compile_function_source_to_plan(source: str, function_name: str, param_types: tuple[Any, ...], *,
                                    include_prelude: bool = True, syntax: str = "ml") -> Plan:
    """The reference's function front end (remora/compiler.py:
    compile_function_source: parse, type check, specialise to
    ``param_types``, lower to HIR) followed by ``plan_from_function``."""
    from remora.compiler import compile_function_source  # the reference's front end

    artifact = compile_function_source(source, function_name, param_types, verify=False,
                                       include_prelude=include_prelude, syntax=syntax)
    return plan_from_function(artifact.hir_function)


# -------------------------------------------------------------- execution
_TORCH = {L.F32: "float32", L.I32: "int32", L.BOOL: "bool"}


def execute_plan(plan: Plan, inputs: list[np.ndarray] | None = None, device: int | None = None) -> np.ndarray:
    """Run a plan on the device and return its result as a numpy array."""
    return PlanRunner(plan, device, results=[plan.result]).run(inputs)[0]


def execute_plan_results(plan: Plan, inputs: list[np.ndarray] | None = None,
                         device: int | None = None) -> list[np.ndarray]:
    """Run a plan on the device and return every one of its results."""
    return PlanRunner(plan, device).run(inputs)


def _check_inputs(plan: Plan, inputs: list[np.ndarray] | None) -> list[np.ndarray]:
    """The caller's inputs, converted to the plan's element types; their
    count and shapes must be the plan's, since the device reads exactly the
    planned extents."""
    want = sorted({b.input for b in plan.buffers if b.input is not None})
    inputs = list(inputs or [])
    if want != list(range(len(inputs))):
        raise RemoraShapeError(f"the plan takes {len(want)} inputs, got {len(inputs)}")
    out = []
    for k, a in enumerate(inputs):
        b = next(b for b in plan.buffers if b.input == k)
        arr = np.array(a, dtype=_NP[b.dtype], order="C")  # rank 0 stays rank 0
        if arr.shape != tuple(b.shape):
            raise RemoraShapeError(f"plan input {k} has shape {arr.shape}, the plan wants {tuple(b.shape)}")
        out.append(arr)
    return out


class PlanRunner:
    """A plan bound to device memory, for one run or many.

    Construction allocates every buffer of the plan on the device, uploads
    its constants and builds each step's descriptors and arguments once.
    It runs on the caller's current stream, or with ``graph=True`` on a
    stream of its own.  The plan's inputs share one device arena
    and its results another, each staged through one pinned host buffer.
    ``run(inputs)`` writes the inputs into the staging buffer, then on that
    stream copies them in (one copy), enqueues every step, copies the
    results out (one copy), and synchronises once, reading the library's
    device error flags (remora_b200_synchronize).  With ``graph=True`` the
    first run, eager, also sizes the stream's workspace and compiles the
    kernels; the copies and steps are then recorded as one CUDA graph, and
    later runs replay it: one launch per run instead of one library call per
    step, for plans run many times (a training loop's value and gradient)."""

    def __init__(self, plan: Plan, device: int | None = None, *, graph: bool = False,
                 results: list[int] | None = None) -> None:
        import torch

        from remora_b200.abi import make_memref_descriptor
        from remora_b200.runtime import context

        self.torch, self.plan, self.graph_wanted, self.graph = torch, plan, graph, None
        self.dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
        self.ctx = context(self.dev.index)
        self.lib = L.lib()
        # One-shot runs use the caller's stream (the library keeps a
        # workspace per stream until shutdown); a graph is captured on a
        # stream of the runner's own.
        self.stream = torch.cuda.Stream(self.dev) if graph else torch.cuda.current_stream(self.dev)
        self._s = ctypes.c_void_p(self.stream.cuda_stream)
        self.results = list(results or plan.results or [plan.result])
        for r in self.results:
            if plan.buffers[r].view is not None:
                raise _unsupported("a plan result that is a view")
        self.launches_per_run: int | None = None
        self.store: dict[int, Any] = {}
        # Inputs and results live in one device arena each, staged through
        # one pinned host buffer each: a run copies once in and once out.
        ins = [i for i, b in enumerate(plan.buffers) if b.input is not None and b.view is None]
        outs = list(dict.fromkeys(r for r in self.results if plan.buffers[r].input is None
                                  and plan.buffers[r].const is None))
        self._in_arena, self._in_host, self._in_np = self._arena(ins)
        self._out_arena, self._out_host, self._out_np = self._arena(outs)
        with torch.cuda.stream(self.stream):
            for i, b in enumerate(plan.buffers):
                if b.view is not None or i in self.store:
                    continue
                if b.const is not None:
                    host = torch.from_numpy(np.array(b.const, dtype=_NP[b.dtype], order="C").reshape(b.shape))
                    self.store[i] = host.to(self.dev)
                else:
                    self.store[i] = torch.empty(b.shape, dtype=getattr(torch, _TORCH[b.dtype]), device=self.dev)
        self._keep: list = []

        def desc(i: int) -> int:
            b = plan.buffers[i]
            if b.view is not None:
                base, off, st = b.view
                d = make_memref_descriptor(self.store[base].data_ptr(), b.shape, st, None, off)
            else:
                st, acc = [], 1
                for n in reversed(b.shape):
                    st.append(acc)
                    acc *= n
                d = make_memref_descriptor(self.store[i].data_ptr(), b.shape, tuple(reversed(st)), None, 0)
            self._keep.append(d)
            return ctypes.addressof(d)

        def rank(i: int) -> int:
            return len(plan.buffers[i].shape)

        def descs(ids: list[int]) -> tuple:
            ptrs = (ctypes.c_void_p * len(ids))(*[desc(i) for i in ids])
            ranks = (ctypes.c_int32 * len(ids))(*[rank(i) for i in ids])
            self._keep += [ptrs, ranks]
            return ptrs, ranks

        lib, ctx, s = self.lib, self.ctx.ptr, self._s
        self.calls: list[tuple[str, Any, tuple]] = []
        for st in plan.steps:
            op = st["op"]
            if op == "map":
                ptrs, ranks = descs(st["ins"])
                self._keep.append(st["program"])
                call = (lib.remora_b200_map, (ctx, ctypes.byref(st["program"]), ptrs, ranks, len(st["ins"]),
                                              desc(st["out"]), rank(st["out"]), s))
            elif op == "fold":
                ptrs, ranks = descs(st["ins"])
                call = (lib.remora_b200_fold, (ctx, ctypes.byref(st["spec"]), ptrs, ranks, len(st["ins"]),
                                               desc(st["out"]), rank(st["out"]), s))
            elif op == "array_fold":
                call = (lib.remora_b200_array_fold, (ctx, ctypes.byref(st["spec"]), desc(st["in"]), rank(st["in"]),
                                                     desc(st["init"]), desc(st["out"]), s))
            elif op == "scan":
                call = (lib.remora_b200_scan, (ctx, ctypes.byref(st["spec"]), desc(st["in"]), desc(st["out"]),
                                               rank(st["in"]), s))
            elif op == "append":
                call = (lib.remora_b200_append, (ctx, plan.buffers[st["a"]].dtype, desc(st["a"]), desc(st["b"]),
                                                 desc(st["out"]), rank(st["out"]), s))
            elif op == "rotate":
                call = (lib.remora_b200_rotate, (ctx, plan.buffers[st["in"]].dtype, int(st["shift"]), desc(st["in"]),
                                                 desc(st["out"]), rank(st["in"]), s))
            elif op in ("sort", "grade"):
                fn = lib.remora_b200_grade if op == "grade" else lib.remora_b200_sort
                call = (fn, (ctx, plan.buffers[st["in"]].dtype, desc(st["in"]), desc(st["out"]), rank(st["in"]), s))
            elif op == "gemm":
                spec = L.RemoraGemmSpec()
                spec.precision = int(st["precision"])
                self._keep.append(spec)
                call = (lib.remora_b200_gemm, (ctx, ctypes.byref(spec), desc(st["a"]), desc(st["b"]), desc(st["out"]),
                                               2, s))
            elif op in ("im2col", "col2im"):
                spec = L.RemoraIm2colSpec(int(st["kh"]), int(st["kw"]), int(st["stride"]), 0)
                self._keep.append(spec)
                fn = lib.remora_b200_im2col if op == "im2col" else lib.remora_b200_col2im
                call = (fn, (ctx, ctypes.byref(spec), desc(st["in"]), desc(st["out"]), s))
            else:
                raise _unsupported(f"plan step {op}")
            self.calls.append((op, *call))

    def _arena(self, ids: list[int]) -> tuple[Any, Any, dict[int, np.ndarray]]:
        """One device arena and one pinned host buffer holding the buffers
        ``ids`` at 256-byte aligned offsets; the device slices become the
        buffers' storage, the host slices their numpy staging views."""
        torch = self.torch
        offs, total = {}, 0
        for i in ids:
            b = self.plan.buffers[i]
            offs[i] = total
            total += (int(np.prod(b.shape, dtype=np.int64)) * np.dtype(_NP[b.dtype]).itemsize + 255) & ~255
        dev = torch.empty(max(total, 256), dtype=torch.uint8, device=self.dev)
        host = torch.empty(max(total, 256), dtype=torch.uint8, pin_memory=True)
        views = {}
        for i in ids:
            b = self.plan.buffers[i]
            n = int(np.prod(b.shape, dtype=np.int64)) * np.dtype(_NP[b.dtype]).itemsize
            dt = getattr(torch, _TORCH[b.dtype])
            self.store[i] = dev[offs[i]:offs[i] + n].view(dt).view(b.shape)
            views[i] = host[offs[i]:offs[i] + n].numpy().view(_NP[b.dtype]).reshape(b.shape)
        return dev, host, views

    def _enqueue(self) -> None:
        """The input copy, every step and the result copy, on the runner's
        stream (the copies are plain cudaMemcpyAsync between the arenas and
        their pinned staging buffers, which a graph records as copy nodes)."""
        ctx, s, lib = self.ctx.ptr, self._s, self.lib
        L.check(lib.remora_b200_memcpy_h2d(ctx, ctypes.c_void_p(self._in_arena.data_ptr()),
                                           ctypes.c_void_p(self._in_host.data_ptr()), self._in_arena.numel(), s),
                "plan inputs")
        for op, fn, args in self.calls:
            L.check(fn(*args), f"plan step {op}")
        L.check(lib.remora_b200_memcpy_d2h(ctx, ctypes.c_void_p(self._out_host.data_ptr()),
                                           ctypes.c_void_p(self._out_arena.data_ptr()), self._out_arena.numel(), s),
                "plan results")

    def run(self, inputs: list[np.ndarray] | None = None) -> list[np.ndarray]:
        """Copy the inputs in, run every step, and return the results."""
        torch = self.torch
        inputs = _check_inputs(self.plan, inputs)
        for i, view in self._in_np.items():
            view[...] = inputs[self.plan.buffers[i].input]
        with torch.cuda.stream(self.stream):
            if self.graph is not None:
                self.graph.replay()
            else:
                n0 = L.launch_count()
                self._enqueue()
                self.launches_per_run = L.launch_count() - n0
        L.check(self.lib.remora_b200_synchronize(self.ctx.ptr, self._s), "plan")
        out = []
        for r in self.results:
            if r in self._out_np:
                out.append(self._out_np[r].copy())
            else:  # a result that is an input or a constant of the plan
                out.append(self.store[r].cpu().numpy().reshape(self.plan.buffers[r].shape))
        if self.graph_wanted and self.graph is None and self.calls:
            self._capture()
        return out

    def _capture(self) -> None:
        """Record the input copy, the steps and the result copy as one CUDA
        graph on the runner's stream (after an eager run: kernels compiled,
        the stream's workspace sized)."""
        torch = self.torch
        g = torch.cuda.CUDAGraph()
        n0 = L.launch_count()
        with torch.cuda.graph(g, stream=self.stream):
            self._enqueue()
        self.launches_per_run = L.launch_count() - n0
        self.graph = g


def compile_source_to_plan(source: str, *, include_prelude: bool = True, syntax: str = "ml") -> Plan:
    """The reference's front end (parse, type check, elaborate, erase to HIR,
    defunctionalise, as remora/compiler.py:106-143 does before its MLIR
    lowering) followed by ``plan_from_hir``.  Needs the reference package."""
    from remora.compiler import _parse_source  # the reference's front end
    from remora.defunc import defunctionalize
    from remora.elaborate import elaborate_program
    from remora.erase import erase_to_hir
    from remora.prelude import with_prelude
    from remora.typechecker import TypeChecker

    text = with_prelude(source) if include_prelude and syntax == "ml" else source
    typed = TypeChecker().check_program(_parse_source(text, syntax))
    return plan_from_hir(defunctionalize(erase_to_hir(elaborate_program(typed))))
