"""Map programs: expression trees lowered to the library's register code.

The expression vocabulary is the reference's fused-map analysis result
(remora/_gpu_map_support.py:22-60: Input, Constant, Binary + - * /, Cmp
< <= > >= == !=, Select) plus the remaining primitives of
remora/operators.py:17-23 (exp, log, && ||), negation and the sqrt epilogue.
``from_reference_expr`` converts the reference's own dataclasses (matched by
class name and fields, so the reference package is not imported) into these.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Union

from remora_b200 import _lib as L
from remora_b200.errors import RemoraB200Error, RemoraLimitError


@dataclass(frozen=True)
class InputExpr:
    index: int


@dataclass(frozen=True)
class ConstantExpr:
    value: float | int


@dataclass(frozen=True)
class BinaryExpr:
    op: str  # + - * /
    left: "Expr"
    right: "Expr"


@dataclass(frozen=True)
class CmpExpr:
    op: str  # < <= > >= == !=
    left: "Expr"
    right: "Expr"


@dataclass(frozen=True)
class SelectExpr:
    condition: "Expr"
    then_expr: "Expr"
    else_expr: "Expr"


@dataclass(frozen=True)
class LogicExpr:
    op: str  # && ||
    left: "Expr"
    right: "Expr"


@dataclass(frozen=True)
class UnaryExpr:
    op: str  # neg exp log sqrt
    operand: "Expr"


Expr = Union[InputExpr, ConstantExpr, BinaryExpr, CmpExpr, SelectExpr, LogicExpr, UnaryExpr]

_BIN = {"+": L.OP_ADD, "-": L.OP_SUB, "*": L.OP_MUL, "/": L.OP_DIV}
_CMP = {"<": L.OP_LT, "<=": L.OP_LE, ">": L.OP_GT, ">=": L.OP_GE, "==": L.OP_EQ, "!=": L.OP_NE}
_LOGIC = {"&&": L.OP_AND, "||": L.OP_OR}
_UNARY = {"neg": L.OP_NEG, "exp": L.OP_EXP, "log": L.OP_LOG, "sqrt": L.OP_SQRT}

DTYPES = {"f32": L.F32, "float32": L.F32, "i32": L.I32, "int32": L.I32, "bool": L.BOOL, "i1": L.BOOL, "i8": L.BOOL}


def dtype_code(dtype: object) -> int:
    if isinstance(dtype, int):
        return dtype
    name = str(dtype).replace("torch.", "").replace("numpy.", "")
    if name in DTYPES:
        return DTYPES[name]
    raise RemoraB200Error(f"unsupported element type {dtype!r} (f32, i32, bool)")


def compile_program(
    expr: Expr,
    n_inputs: int,
    *,
    compute: object = L.F32,
    out: object | None = None,
    in_dtypes: list[object] | None = None,
) -> L.RemoraMapProgram:
    """Lower an expression tree to register code (common subexpressions
    computed once).  ``compute`` is the arithmetic type, ``out`` the stored
    element type (defaults to ``compute``), ``in_dtypes`` per input."""
    compute_c = dtype_code(compute)
    out_c = compute_c if out is None else dtype_code(out)
    ins = [compute_c] * n_inputs if in_dtypes is None else [dtype_code(d) for d in in_dtypes]
    if len(ins) != n_inputs:
        raise RemoraB200Error("in_dtypes must give one dtype per input")
    if n_inputs > L.MAP_MAX_INPUTS:
        raise RemoraLimitError(f"at most {L.MAP_MAX_INPUTS} inputs per map program")
    code: list[tuple] = []
    memo: dict[Expr, int] = {}

    def emit(op: int, a: int = 0, b: int = 0, c: int = 0, imm_f: float = 0.0, imm_i: int = 0) -> int:
        dst = len(code)
        if dst >= L.MAP_MAX_REGS or dst >= L.MAP_MAX_INSTR:
            raise RemoraLimitError(f"map program exceeds {L.MAP_MAX_INSTR} instructions")
        code.append((op, dst, a, b, c, imm_f, imm_i))
        return dst

    def walk(e: Expr) -> int:
        if e in memo:
            return memo[e]
        if isinstance(e, InputExpr):
            if not 0 <= e.index < n_inputs:
                raise RemoraB200Error(f"input {e.index} out of range for {n_inputs} inputs")
            r = emit(L.OP_INPUT, imm_i=e.index)
        elif isinstance(e, ConstantExpr):
            if compute_c == L.F32:
                r = emit(L.OP_CONST, imm_f=float(e.value))
            else:
                r = emit(L.OP_CONST, imm_i=int(e.value))
        elif isinstance(e, BinaryExpr):
            r = emit(_BIN[e.op], walk(e.left), walk(e.right))
        elif isinstance(e, CmpExpr):
            r = emit(_CMP[e.op], walk(e.left), walk(e.right))
        elif isinstance(e, LogicExpr):
            r = emit(_LOGIC[e.op], walk(e.left), walk(e.right))
        elif isinstance(e, SelectExpr):
            r = emit(L.OP_SELECT, walk(e.condition), walk(e.then_expr), walk(e.else_expr))
        elif isinstance(e, UnaryExpr):
            r = emit(_UNARY[e.op], walk(e.operand))
        else:
            raise RemoraB200Error(f"unsupported expression node {e!r}")
        memo[e] = r
        return r

    result = walk(expr)
    prog = L.RemoraMapProgram()
    prog.n_instr = len(code)
    prog.n_inputs = n_inputs
    prog.compute_dtype = compute_c
    prog.out_dtype = out_c
    prog.result = result
    for k, d in enumerate(ins):
        prog.in_dtype[k] = d
    for k, (op, dst, a, b, c, imm_f, imm_i) in enumerate(code):
        ins_ = prog.code[k]
        ins_.op, ins_.dst, ins_.a, ins_.b, ins_.c = op, dst, a, b, c
        ins_.imm_f = imm_f
        ins_.imm_i = imm_i
    return prog


def from_reference_expr(node: object) -> Expr:
    """Convert the reference's F32Expr dataclasses (F32InputExpr,
    F32ConstantExpr, F32BinaryExpr, F32CmpExpr, F32SelectExpr of
    remora/_gpu_map_support.py:29-60) into this module's nodes."""
    name = type(node).__name__
    if name == "F32InputExpr":
        return InputExpr(int(node.index))
    if name == "F32ConstantExpr":
        return ConstantExpr(float(node.value))
    if name == "F32BinaryExpr":
        return BinaryExpr(node.op, from_reference_expr(node.left), from_reference_expr(node.right))
    if name == "F32CmpExpr":
        return CmpExpr(node.op, from_reference_expr(node.left), from_reference_expr(node.right))
    if name == "F32SelectExpr":
        return SelectExpr(
            from_reference_expr(node.condition),
            from_reference_expr(node.then_expr),
            from_reference_expr(node.else_expr),
        )
    raise RemoraB200Error(f"not a reference map expression: {name}")


def section_expr(op: str, constant: float | int | None, side: str | None, n_inputs: int) -> Expr:
    """The simple map shapes of the reference's map analysis
    (remora/_gpu_map_support.py:187-197): a binary op over two inputs, or a
    literal section ``(op c)`` / ``(c op)`` over one input."""
    if n_inputs == 2:
        return BinaryExpr(op, InputExpr(0), InputExpr(1)) if op in _BIN else LogicExpr(op, InputExpr(0), InputExpr(1)) if op in _LOGIC else CmpExpr(op, InputExpr(0), InputExpr(1))
    if constant is None:
        raise RemoraB200Error("a unary map needs a literal section constant")
    c = ConstantExpr(constant)
    x = InputExpr(0)
    make = BinaryExpr if op in _BIN else LogicExpr if op in _LOGIC else CmpExpr
    return make(op, c, x) if side == "left" else make(op, x, c)


# ------------------------------------------------------------ conveniences
def x(i: int = 0) -> InputExpr:
    return InputExpr(i)


def const(v: float | int) -> ConstantExpr:
    return ConstantExpr(v)


def stable_bce(z: Expr, y: Expr) -> Expr:
    """The reference's overflow-free binary cross-entropy on a logit
    (examples/crater_train.py:50-54):
    select(z > 0, z, 0) + (-1 * (z * y) + log(1 + exp(0 - select(z > 0, z, 0 - z))))."""
    zero = ConstantExpr(0.0)
    pos = SelectExpr(CmpExpr(">", z, zero), z, zero)
    absz = SelectExpr(CmpExpr(">", z, zero), z, BinaryExpr("-", zero, z))
    soft = UnaryExpr("log", BinaryExpr("+", ConstantExpr(1.0), UnaryExpr("exp", BinaryExpr("-", zero, absz))))
    return BinaryExpr("+", pos, BinaryExpr("+", BinaryExpr("*", ConstantExpr(-1.0), BinaryExpr("*", z, y)), soft))
