"""Kernel specs: what this backend produces where the reference produces PTX.

The reference's code generator returns ``(ptx, [KernelMeta])``
(remora/codegen.py:116-257).  Here the same ``KernelMeta`` (field for field,
remora/codegen.py:50-61) travels with a ``SpecModule`` mapping each kernel
name to an op spec; ``B200Runtime.load_ptx`` accepts that module and each
spec knows which C-ABI entry point runs it.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Any

from remora_b200 import _lib as L
from remora_b200.abi import descriptor_rank
from remora_b200.errors import RemoraExecutorError
from remora_b200.program import Expr, compile_program


@dataclass(frozen=True)
class KernelMeta:
    name: str
    grid_dims: int
    block_size: int
    num_inputs: int
    num_outputs: int
    input_elem_types: list[str]
    output_elem_types: list[str]
    output_shape: tuple[int, ...] | None = None
    output_dtype: str | None = None
    is_reduction: bool = False


def _ptrs(descs: list[ctypes.Structure]):
    ptrs = (ctypes.c_void_p * max(1, len(descs)))()
    ranks = (ctypes.c_int32 * max(1, len(descs)))()
    for k, d in enumerate(descs):
        ptrs[k] = ctypes.addressof(d)
        ranks[k] = descriptor_rank(d)
    return ptrs, ranks


@dataclass
class MapSpec:
    program: L.RemoraMapProgram

    def launch(self, ctx: Any, ins: list, out: ctypes.Structure, stream: Any = None) -> None:
        ptrs, ranks = _ptrs(ins)
        L.check(
            L.lib().remora_b200_map(ctx.ptr, ctypes.byref(self.program), ptrs, ranks, len(ins),
                                    ctypes.addressof(out), descriptor_rank(out), stream),
            "remora_b200_map",
        )


@dataclass
class FoldSpec:
    spec: L.RemoraFoldSpec

    def launch(self, ctx: Any, ins: list, out: ctypes.Structure, stream: Any = None) -> None:
        ptrs, ranks = _ptrs(ins)
        L.check(
            L.lib().remora_b200_fold(ctx.ptr, ctypes.byref(self.spec), ptrs, ranks, len(ins),
                                     ctypes.addressof(out), descriptor_rank(out), stream),
            "remora_b200_fold",
        )


@dataclass
class ScanSpec:
    spec: L.RemoraScanSpec

    def launch(self, ctx: Any, ins: list, out: ctypes.Structure, stream: Any = None) -> None:
        if len(ins) != 1:
            raise RemoraExecutorError("a scan takes one input")
        L.check(
            L.lib().remora_b200_scan(ctx.ptr, ctypes.byref(self.spec), ctypes.addressof(ins[0]),
                                     ctypes.addressof(out), descriptor_rank(out), stream),
            "remora_b200_scan",
        )


@dataclass
class GemmSpec:
    precision: int = L.PREC_3XTF32

    def launch(self, ctx: Any, ins: list, out: ctypes.Structure, stream: Any = None) -> None:
        if len(ins) != 2:
            raise RemoraExecutorError("a matmul takes two inputs")
        spec = L.RemoraGemmSpec(self.precision, 0)
        L.check(
            L.lib().remora_b200_gemm(ctx.ptr, ctypes.byref(spec), ctypes.addressof(ins[0]),
                                     ctypes.addressof(ins[1]), ctypes.addressof(out),
                                     descriptor_rank(out), stream),
            "remora_b200_gemm",
        )


@dataclass
class AppendSpec:
    """out = inputs[left] followed by inputs[1 - left] along axis 0."""

    dtype: int = L.F32
    left: int = 0

    def launch(self, ctx: Any, ins: list, out: ctypes.Structure, stream: Any = None) -> None:
        if len(ins) != 2:
            raise RemoraExecutorError("an append takes two inputs")
        a, b = ins[self.left], ins[1 - self.left]
        L.check(
            L.lib().remora_b200_append(ctx.ptr, self.dtype, ctypes.addressof(a), ctypes.addressof(b),
                                       ctypes.addressof(out), descriptor_rank(out), stream),
            "remora_b200_append",
        )


@dataclass
class RotateSpec:
    dtype: int = L.F32
    shift: int = 0

    def launch(self, ctx: Any, ins: list, out: ctypes.Structure, stream: Any = None) -> None:
        if len(ins) != 1:
            raise RemoraExecutorError("a rotate takes one input")
        L.check(
            L.lib().remora_b200_rotate(ctx.ptr, self.dtype, int(self.shift), ctypes.addressof(ins[0]),
                                       ctypes.addressof(out), descriptor_rank(out), stream),
            "remora_b200_rotate",
        )


@dataclass
class SortSpec:
    """Ascending sort, or with grade the stable argsort, of rank 1 or rows."""

    dtype: int = L.F32
    grade: bool = False

    def launch(self, ctx: Any, ins: list, out: ctypes.Structure, stream: Any = None) -> None:
        if len(ins) != 1:
            raise RemoraExecutorError("a sort takes one input")
        fn = L.lib().remora_b200_grade if self.grade else L.lib().remora_b200_sort
        L.check(fn(ctx.ptr, self.dtype, ctypes.addressof(ins[0]), ctypes.addressof(out), descriptor_rank(out),
                   stream), "remora_b200_grade" if self.grade else "remora_b200_sort")


@dataclass
class SpecModule:
    kernels: dict[str, Any] = field(default_factory=dict)


# ------------------------------------------------- records (plain data)
def spec_record(spec: Any) -> dict:
    """A spec as plain data (json-able): the C structs as hex bytes."""
    if isinstance(spec, MapSpec):
        return {"kind": "map", "bytes": bytes(spec.program).hex()}
    if isinstance(spec, FoldSpec):
        return {"kind": "fold", "bytes": bytes(spec.spec).hex()}
    if isinstance(spec, ScanSpec):
        return {"kind": "scan", "bytes": bytes(spec.spec).hex()}
    if isinstance(spec, GemmSpec):
        return {"kind": "gemm", "precision": int(spec.precision)}
    if isinstance(spec, AppendSpec):
        return {"kind": "append", "dtype": int(spec.dtype), "left": int(spec.left)}
    if isinstance(spec, RotateSpec):
        return {"kind": "rotate", "dtype": int(spec.dtype), "shift": int(spec.shift)}
    if isinstance(spec, SortSpec):
        return {"kind": "sort", "dtype": int(spec.dtype), "grade": bool(spec.grade)}
    raise RemoraExecutorError(f"no record form for {type(spec).__name__}")


def spec_from_record(rec: dict) -> Any:
    kind = rec["kind"]
    if kind in ("map", "fold", "scan"):
        cls = {"map": L.RemoraMapProgram, "fold": L.RemoraFoldSpec, "scan": L.RemoraScanSpec}[kind]
        raw = bytes.fromhex(rec["bytes"])
        if len(raw) != ctypes.sizeof(cls):
            raise RemoraExecutorError(f"{kind} record holds {len(raw)} bytes, the struct has {ctypes.sizeof(cls)}")
        st = cls.from_buffer_copy(raw)
        return {"map": MapSpec, "fold": FoldSpec, "scan": ScanSpec}[kind](st)
    if kind == "gemm":
        return GemmSpec(int(rec["precision"]))
    if kind == "append":
        return AppendSpec(int(rec["dtype"]), int(rec["left"]))
    if kind == "rotate":
        return RotateSpec(int(rec["dtype"]), int(rec["shift"]))
    if kind == "sort":
        return SortSpec(int(rec["dtype"]), bool(rec["grade"]))
    raise RemoraExecutorError(f"unknown spec kind {kind!r}")


def meta_record(meta: KernelMeta) -> dict:
    d = dict(meta.__dict__)
    d["output_shape"] = None if meta.output_shape is None else list(meta.output_shape)
    return d


def meta_from_record(rec: dict) -> KernelMeta:
    d = dict(rec)
    if d.get("output_shape") is not None:
        d["output_shape"] = tuple(d["output_shape"])
    return KernelMeta(**d)


_DT = {L.F32: "f32", L.I32: "i32", L.BOOL: "i8"}
_NP = {L.F32: "float32", L.I32: "int32", L.BOOL: "bool"}


def map_kernel(name: str, expr: Expr, n_inputs: int, *, shape: tuple[int, ...] | None = None,
               compute: object = L.F32, out: object | None = None,
               in_dtypes: list[object] | None = None) -> tuple[MapSpec, KernelMeta]:
    prog = compile_program(expr, n_inputs, compute=compute, out=out, in_dtypes=in_dtypes)
    meta = KernelMeta(
        name=name, grid_dims=1, block_size=0, num_inputs=n_inputs, num_outputs=1,
        input_elem_types=[_DT[prog.in_dtype[k]] for k in range(n_inputs)],
        output_elem_types=[_DT[prog.out_dtype]], output_shape=shape, output_dtype=_NP[prog.out_dtype],
    )
    return MapSpec(prog), meta


def fold_spec(*, op: str = "+", init: float | int = 0, mode: str = "cell", cell_rank: int = 1,
              dtype: object = L.F32, premap: Expr | None = None, n_inputs: int = 1,
              epilogue: str | None = None, premap_in_dtypes: list[object] | None = None) -> L.RemoraFoldSpec:
    from remora_b200.program import dtype_code

    sp = L.RemoraFoldSpec()
    sp.op = {"+": L.FOLD_ADD, "*": L.FOLD_MUL}[op]
    sp.mode = {"cell": L.FOLD_CELL, "all": L.FOLD_ALL}[mode]
    sp.cell_rank = int(cell_rank)
    sp.dtype = dtype_code(dtype)
    sp.epilogue = {None: L.EPI_NONE, "sqrt": L.EPI_SQRT}[epilogue]
    if sp.dtype == L.F32:
        sp.init_f = float(init)
    else:
        sp.init_i = int(init)
    if premap is not None:
        sp.has_premap = 1
        sp.premap = compile_program(premap, n_inputs, compute=sp.dtype, out=sp.dtype, in_dtypes=premap_in_dtypes)
    return sp


def fold_kernel(name: str, *, shape: tuple[int, ...] | None = None, **kw: Any) -> tuple[FoldSpec, KernelMeta]:
    sp = fold_spec(**kw)
    n_in = int(kw.get("n_inputs", 1))
    meta = KernelMeta(
        name=name, grid_dims=1, block_size=0, num_inputs=n_in, num_outputs=1,
        input_elem_types=[_DT[sp.dtype]] * n_in, output_elem_types=[_DT[sp.dtype]],
        output_shape=shape if sp.mode == L.FOLD_CELL else (), output_dtype=_NP[sp.dtype],
        is_reduction=sp.mode == L.FOLD_ALL,
    )
    return FoldSpec(sp), meta


def scan_spec(*, op: str = "+", init: float | int = 0, dtype: object = L.F32, exclusive: bool = False,
              right: bool = False) -> L.RemoraScanSpec:
    from remora_b200.program import dtype_code

    sp = L.RemoraScanSpec()
    sp.op = {"+": L.FOLD_ADD, "*": L.FOLD_MUL}[op]
    sp.dtype = dtype_code(dtype)
    sp.exclusive = int(bool(exclusive))
    sp.right = int(bool(right))
    if sp.dtype == L.F32:
        sp.init_f = float(init)
    else:
        sp.init_i = int(init)
    return sp
