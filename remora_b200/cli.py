"""Command line for the B200 backend: the reference CLI's two GPU paths.

``python -m remora_b200.cli FILE --call NAME --input a.npy [--input b.npy]``
is the reference's ``remorac FILE --call NAME --input ...``
(remora/cli.py:141-187): the named function is typed from the .npy inputs
(a 0-d input is a scalar parameter), compiled by the reference front end,
lowered to this backend's specs (``reference_codegen``) and run through
``B200Executor``; a function no single kernel computes runs as a device plan
(``program_plan.plan_from_function``).

``python -m remora_b200.cli FILE`` runs a whole program, as
``remorac FILE --target gpu-nvidia`` does (remora/cli.py:190-212,
remora/executor.py:192-306), through a device-resident plan
(``program_plan``).  ``--emit-plan`` prints that plan as JSON instead, and
``--plan PLAN.json`` runs a recorded plan, which needs neither the source nor
the reference front end.

Results print the way remora/display.py:10-44 formats them, and failures
print ``remorac: <message>`` on stderr with exit status 1, as the reference
CLI does (remora/cli.py:130-132,159-187).
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np

from remora_b200.errors import RemoraB200Error


# ------------------------------------------------------------- formatting
def format_scalar(value: object, kind: str) -> str:
    """One element: ``true``/``false``, a plain integer, or a float with six
    significant digits that always shows it is a float (remora/display.py:32-44)."""
    if isinstance(value, np.generic):
        value = value.item()
    if kind == "bool":
        return "true" if bool(value) else "false"
    if kind == "int":
        return str(int(value))
    text = f"{float(value):.6g}"
    return text if ("e" in text or "." in text) else text + ".0"


def _kind(dtype: np.dtype) -> str:
    if dtype == np.bool_:
        return "bool"
    return "int" if np.issubdtype(dtype, np.integer) else "float"


def format_result(value: np.ndarray) -> str:
    """A result array as remora/display.py:10-29 prints it: rank 0 as a scalar,
    higher ranks through numpy's array printer with ``, `` separators."""
    arr = np.asarray(value)
    kind = _kind(arr.dtype)
    if arr.ndim == 0:
        return format_scalar(arr.item(), kind)
    fmt = {"bool": lambda v: format_scalar(v, "bool"), "int_kind": lambda v: format_scalar(v, "int"),
           "float_kind": lambda v: format_scalar(v, "float")}
    return np.array2string(arr, separator=", ", formatter=fmt)


# ----------------------------------------------------------------- --call
def _param_type(arr: np.ndarray):
    from remora.types import BOOL, FLOAT, INT, ArrayType, StaticDim  # the reference's front end

    if arr.dtype == np.float32:
        elem = FLOAT
    elif arr.dtype == np.bool_:
        elem = BOOL
    elif np.issubdtype(arr.dtype, np.integer):
        elem = INT
    else:
        raise RemoraB200Error(f"input of dtype {arr.dtype}: save --input arrays as float32, int32 or bool")
    if arr.ndim == 0:
        return elem  # a 0-d input is a scalar parameter
    return ArrayType(elem, tuple(StaticDim(int(d)) for d in arr.shape))


def call_function(source: str, name: str, arrays: list[np.ndarray], *, syntax: str = "ml") -> np.ndarray:
    """Compile function ``name`` of ``source`` for the argument shapes and
    dtypes of ``arrays`` and run it on the device: as one kernel where the
    codegen takes the function whole (``reference_codegen``), else as a
    device plan of several steps (``program_plan.plan_from_function``)."""
    from remora_b200.errors import RemoraUnsupportedError
    from remora_b200.program_plan import compile_function_source_to_plan
    from remora_b200.reference_codegen import compile_function_source_to_b200_artifacts

    arrays = [a.astype(np.int32) if np.issubdtype(a.dtype, np.integer) else a for a in arrays]
    plan = None
    try:
        types = tuple(_param_type(a) for a in arrays)
        try:
            module, kernels, _hir = compile_function_source_to_b200_artifacts(source, name, types, syntax=syntax)
        except RemoraUnsupportedError:
            plan = compile_function_source_to_plan(source, name, types, syntax=syntax)
    except Exception as exc:
        raise _CliError(f"GPU function compilation failed: {exc}") from exc
    if plan is not None:
        return run_plan(plan, arrays)
    try:
        from remora_b200.executor import B200Executor

        executor = B200Executor(module, kernels)
        names = [k.name for k in kernels]
        kernel = name if name in names else names[0]
        return executor.execute(kernel, arrays)
    except Exception as exc:
        raise _CliError(f"GPU execution failed: {exc}") from exc


# --------------------------------------------------------- whole programs
def run_plan(plan, arrays: list[np.ndarray]) -> np.ndarray:
    from remora_b200.program_plan import execute_plan

    n_in = sum(1 for b in plan.buffers if b.input is not None)
    if n_in != len(arrays):
        raise _CliError(f"the plan takes {n_in} --input arrays, got {len(arrays)}")
    try:
        return execute_plan(plan, arrays)
    except Exception as exc:
        raise _CliError(f"GPU execution failed: {exc}") from exc


class _CliError(Exception):
    pass


def main(argv: list[str] | None = None) -> int:
    parser = argparse.ArgumentParser(prog="remora_b200.cli", description="Remora programs on the B200 backend")
    parser.add_argument("file", type=Path, nargs="?", help="Remora source file")
    parser.add_argument("--syntax", choices=("ml", "lisp"), default="ml",
                        help="syntax for reading source files; ml (default) or lisp")
    parser.add_argument("--call", type=str, default=None,
                        help="call a named function with descriptor ABI (requires --input for each param)")
    parser.add_argument("--input", type=Path, action="append", default=None,
                        help="load a .npy file as input to a --call function or a --plan")
    parser.add_argument("--emit-plan", action="store_true", help="print the program's device plan as JSON and exit")
    parser.add_argument("--plan", type=Path, default=None, help="run a plan recorded with --emit-plan")
    args = parser.parse_args(argv)
    try:
        arrays = [np.load(str(p)) for p in (args.input or [])]
        if args.plan is not None:
            from remora_b200.program_plan import Plan

            print(format_result(run_plan(Plan.from_record(json.loads(args.plan.read_text())), arrays)))
            return 0
        if args.file is None:
            raise _CliError("a source file (or --plan) is required")
        source = args.file.read_text(encoding="utf-8")
        if args.call is not None:
            if not arrays:
                raise _CliError("--call requires at least one --input FILE.npy")
            print(format_result(call_function(source, args.call, arrays, syntax=args.syntax)))
            return 0
        from remora_b200.program_plan import compile_source_to_plan

        try:
            plan = compile_source_to_plan(source, syntax=args.syntax)
        except RemoraB200Error:
            raise
        except Exception as exc:  # the reference front end rejects the program
            raise _CliError(str(exc)) from exc
        if args.emit_plan:
            print(json.dumps(plan.to_record()))
            return 0
        print(format_result(run_plan(plan, arrays)))
        return 0
    except (OSError, ValueError, RemoraB200Error, _CliError) as exc:
        print(f"remorac: {exc}", file=sys.stderr)
        return 1


if __name__ == "__main__":
    raise SystemExit(main())
