"""Host-only tests of the boundary: descriptor layout (the reference's
tests/test_abi.py strategy), the C library's exports, the program compiler
and its NVRTC code generation (no GPU needed)."""

from __future__ import annotations

import ctypes
import re

import numpy as np
import pytest

from conftest import ROOT
from remora_b200 import _lib as L
from remora_b200.abi import (DESCRIPTORS, descriptor_rank, descriptor_shape, descriptor_strides, element_strides,
                             make_memref_descriptor, numpy_descriptor)
from remora_b200.errors import RemoraB200Error, RemoraLimitError
from remora_b200.program import (BinaryExpr, CmpExpr, ConstantExpr, InputExpr, LogicExpr, SelectExpr, UnaryExpr,
                                 compile_program, const, from_reference_expr, stable_bce, x)


def test_descriptor_sizes_and_field_order():
    for rank, cls in DESCRIPTORS.items():
        assert ctypes.sizeof(cls) == 24 + 16 * rank
        names = [f[0] for f in cls._fields_]
        assert names[:3] == ["allocated", "aligned", "offset"]
        assert names[3:3 + rank] == [f"size{d}" for d in range(rank)]
        assert names[3 + rank:] == [f"stride{d}" for d in range(rank)]
        assert descriptor_rank(cls) == rank


def test_descriptor_from_views():
    base = np.arange(60, dtype=np.float32).reshape(3, 4, 5)
    d = numpy_descriptor(base)
    assert descriptor_shape(d) == (3, 4, 5) and descriptor_strides(d) == (20, 5, 1) and d.offset == 0
    v = base[1:, ::2, ::-1]
    d = numpy_descriptor(v)
    assert descriptor_shape(d) == v.shape
    assert descriptor_strides(d) == element_strides(v) == (20, 10, -1)
    assert d.offset == 20 + 4 and d.aligned == base.ctypes.data
    t = base.transpose(2, 0, 1)
    assert descriptor_strides(numpy_descriptor(t)) == (1, 20, 5)


def test_descriptor_rejects_bad_input():
    with pytest.raises(RemoraB200Error):
        make_memref_descriptor(0, [2, -1], [1, 1])
    with pytest.raises(RemoraB200Error):
        make_memref_descriptor(0, [2, 2], [1])
    with pytest.raises(RemoraB200Error):
        make_memref_descriptor(0, [1] * 11, [1] * 11)


def _header_symbols() -> set[str]:
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"\b(remora_b200_\w+)\s*\(", text))
    return names


def test_library_loads_and_exports_every_declared_symbol():
    lib = L.lib()
    declared = _header_symbols()
    assert declared, "no entry points found in include/*.h"
    missing = sorted(n for n in declared if not hasattr(lib, n))
    assert not missing, f"declared but not exported: {missing}"
    assert b"sm_100a" in lib.remora_b200_version()


def test_launch_counter_is_exported_and_untouched_by_rejected_calls():
    n0 = L.launch_count()
    assert isinstance(n0, int) and n0 >= 0
    # a call with no context is rejected before any kernel is enqueued
    assert L.lib().remora_b200_memset_d32(None, None, 0, 16, None) != 0
    assert L.launch_count() == n0


def test_header_struct_sizes_match_ctypes():
    # RemoraMapProgram: 5 int32 + 8 int32 + 48 x 16-byte instructions
    assert ctypes.sizeof(L.RemoraMapInstr) == 16
    assert ctypes.sizeof(L.RemoraMapProgram) == 4 * 5 + 4 * 8 + 16 * 48
    assert ctypes.sizeof(L.RemoraScanSpec) == 24


def test_compile_program_cse_and_limits():
    y = BinaryExpr("+", BinaryExpr("*", x(0), const(2.5)), const(1.0))
    chain = SelectExpr(CmpExpr(">", y, const(0.5)), y, const(0.0))
    p = compile_program(chain, 1)
    # y is computed once: input, 2.5, mul, 1.0, add, 0.5, cmp, 0.0, select
    assert p.n_instr == 9 and p.result == 8
    deep = x(0)
    for _ in range(30):
        deep = BinaryExpr("+", deep, ConstantExpr(float(_)))
    with pytest.raises(RemoraLimitError):
        compile_program(deep, 1)
    with pytest.raises(RemoraB200Error):
        compile_program(x(2), 1)


def test_from_reference_expr_by_shape():
    # stand-ins with the reference's class names and fields
    def mk(name, **kw):
        return type(name, (), {"__init__": lambda self: self.__dict__.update(kw)})()

    node = mk("F32BinaryExpr", op="+", left=mk("F32InputExpr", index=0), right=mk("F32ConstantExpr", value=1.0))
    assert from_reference_expr(node) == BinaryExpr("+", InputExpr(0), ConstantExpr(1.0))


@pytest.mark.parametrize("case", ["chain", "i32", "bool", "bce", "div", "cmp_bool_out", "sqrt"])
def test_generated_kernels_compile_for_sm100a(case):
    y = BinaryExpr("+", BinaryExpr("*", x(0), const(2.5)), const(1.0))
    progs = {
        "chain": (compile_program(SelectExpr(CmpExpr(">", y, const(0.5)), y, const(0.0)), 1), L.FOLD_ADD),
        "i32": (compile_program(BinaryExpr("*", x(0), BinaryExpr("-", x(1), const(3))), 2, compute="i32"), L.FOLD_MUL),
        "bool": (compile_program(LogicExpr("||", x(0), x(1)), 2, compute="bool"), -1),
        "bce": (compile_program(stable_bce(x(0), x(1)), 2), L.FOLD_ADD),
        "div": (compile_program(BinaryExpr("/", x(0), x(1)), 2, compute="f32", in_dtypes=["i32", "i32"]), L.FOLD_ADD),
        "cmp_bool_out": (compile_program(CmpExpr("<=", x(0), const(0.0)), 1, out="bool"), -1),
        "sqrt": (compile_program(UnaryExpr("sqrt", x(0)), 1), L.FOLD_ADD),
    }
    prog, fold_op = progs[case]
    buf = ctypes.create_string_buffer(1 << 18)
    st = L.lib().remora_b200_jit_check(ctypes.byref(prog), fold_op, buf, len(buf))
    assert st == 0, L.last_error()
    src = buf.value.decode()
    assert "remora_map_vec" in src and "remora_map_strided" in src
    if fold_op >= 0:
        assert "remora_fold_cell_vec" in src and "remora_fold_all" in src
    # every kernel may run as a programmatic dependent of the previous one
    assert src.count("PDL_PROLOGUE();") == (5 if fold_op >= 0 else 2)
    # no unrounded f32 arithmetic that the compiler could contract into FMA
    body = src.split("remora_expr(")[1].split("return")[0]
    assert "fmaf" not in body


def test_jit_check_rejects_bad_programs():
    p = compile_program(BinaryExpr("+", x(0), x(1)), 2)
    p.code[2].a = 40  # read an unwritten register
    assert L.lib().remora_b200_jit_check(ctypes.byref(p), -1, None, 0) == L.ERR_ARG
    assert "before it is written" in L.last_error()
    p = compile_program(UnaryExpr("exp", x(0)), 1, compute="i32")
    assert L.lib().remora_b200_jit_check(ctypes.byref(p), -1, None, 0) == L.ERR_UNSUPPORTED


def _c_member(cname: str, field: str) -> str:
    m = re.fullmatch(r"(size|stride)(\d+)", field)
    if cname.startswith("RemoraMemRef") and m:
        return f"{m.group(1)}s[{m.group(2)}]"
    return field


def test_headers_compile_as_c_and_cxx_with_the_ctypes_layouts(tmp_path):
    """include/*.h is plain C (what a cgo or C caller includes) and C++, and a
    C compiler lays every struct out exactly as the ctypes mirrors the Python
    binding passes by pointer: same size, same offset for every field."""
    import shutil
    import subprocess

    from remora_b200 import abi
    from remora_b200.cnn import RemoraCnnStepSpec

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    structs = [abi.DESCRIPTORS[r] for r in range(abi.MAX_RANK + 1)] + [
        L.RemoraMapInstr, L.RemoraMapProgram, L.RemoraFoldSpec, L.RemoraScanSpec, L.RemoraGemmSpec,
        L.RemoraConvSpec, L.RemoraIm2colSpec, L.RemoraFilterPred, RemoraCnnStepSpec]
    lines = ["#include <stddef.h>", "#include <stdio.h>", '#include "remora_b200.h"', '#include "remora_b200_cnn.h"',
             "int main(void) {"]
    for s in structs:
        c = s.__name__
        lines.append(f'  printf("{c} %zu\\n", sizeof({c}));')
        for f, _ in s._fields_:
            lines.append(f'  printf("{c}.{f} %zu\\n", offsetof({c}, {_c_member(c, f)}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    r = subprocess.run([cc, "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", f"-I{ROOT / 'include'}",
                        str(src), "-o", str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    got = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                       check=True).stdout.splitlines())
    for s in structs:
        c = s.__name__
        assert int(got[c]) == ctypes.sizeof(s), c
        for f, _ in s._fields_:
            assert int(got[f"{c}.{f}"]) == getattr(s, f).offset, f"{c}.{f}"
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is not None:
        for h in sorted((ROOT / "include").glob("*.h")):
            r = subprocess.run([cxx, "-std=c++11", "-Wall", "-Wextra", "-Werror", "-fsyntax-only", "-x", "c++",
                                f"-I{ROOT / 'include'}", str(h)], capture_output=True, text=True)
            assert r.returncode == 0, (h.name, r.stderr)


def test_a_c_caller_links_and_calls_the_library(tmp_path):
    """The library as a C (or cgo) binding sees it: linked by name, no Python
    in between.  Calls that need no GPU: the version, a call rejected before
    any work (no context) with its status and message."""
    import shutil
    import subprocess

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    so = L.library_path()
    src = tmp_path / "caller.c"
    src.write_text(r"""
#include <stdio.h>
#include <string.h>
#include "remora_b200.h"
int main(void) {
  char msg[512];
  int st;
  printf("version %s\n", remora_b200_version());
  st = remora_b200_memset_d32(NULL, NULL, 0u, 16, NULL);
  remora_b200_last_error(msg, sizeof msg);
  printf("status %d\n", st);
  printf("message %s\n", msg);
  return 0;
}
""")
    exe = tmp_path / "caller"
    r = subprocess.run([cc, "-std=c99", "-Wall", "-Werror", f"-I{ROOT / 'include'}", str(src), "-o", str(exe),
                        f"-L{so.parent}", f"-l:{so.name}", f"-Wl,-rpath,{so.parent}"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True, timeout=60).stdout
    lines = dict(line.split(" ", 1) for line in out.splitlines())
    assert "sm_100a" in lines["version"]
    assert int(lines["status"]) == L.ERR_ARG
    assert lines["message"].strip()
