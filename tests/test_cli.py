"""The command line (remora_b200.cli) without a GPU.

Device execution is replaced by the oracle here (the plan's steps, or each
recorded spec, run on the CPU restatement), so these tests check what the
command line adds: argument handling, typing of --call inputs, the way
results print and the way failures report.  The printed text of every
recorded acceptance program is compared with the stdout the reference's own
acceptance manifest expects of its CLI.  tests/test_gpu_cli.py runs the same
command line on the device."""

from __future__ import annotations

import json
import os
import sys

import numpy as np
import pytest

from conftest import REFERENCE, GOLDEN
from remora_b200 import cli
from remora_b200.codegen import meta_from_record, spec_from_record
from remora_b200.program_plan import Plan

from test_program_plan import run_plan_on_oracle
from test_reference_codegen import oracle_run

REF = REFERENCE or ""
have_ref = REFERENCE is not None
needs_ref = pytest.mark.skipif(not have_ref, reason="the reference front end is not importable here")
if have_ref and REF not in sys.path:
    sys.path.insert(0, REF)  # the CLI compiles through the reference's front end


def plans() -> list[dict]:
    return json.loads((GOLDEN / "program_plans.json").read_text())["programs"]


def run(argv: list[str], capsys) -> tuple[int, str, str]:
    code = cli.main(argv)
    out, err = capsys.readouterr()
    return code, out.strip(), err.strip()


@pytest.fixture
def on_oracle(monkeypatch, oracle_mod):
    """Device execution replaced by the oracle."""
    monkeypatch.setattr("remora_b200.program_plan.execute_plan",
                        lambda plan, inputs=None, device=None: run_plan_on_oracle(oracle_mod, plan, inputs))

    class OracleExecutor:
        def __init__(self, module, kernels):
            self.specs, self.metas = module.kernels, {k.name: k for k in kernels}

        def execute(self, name, arrays):
            return oracle_run(oracle_mod, self.specs[name], self.metas[name], arrays)

    monkeypatch.setattr("remora_b200.executor.B200Executor", OracleExecutor)
    return oracle_mod


# ------------------------------------------------------------- formatting
@pytest.mark.parametrize("value, text", [
    (np.float32(3.0), "3.0"), (np.float32(0.1), "0.1"), (np.float32(1e-7), "1e-07"),
    (np.float32(123456789.0), "1.23457e+08"), (np.float32(np.inf), "inf.0"), (np.int32(-7), "-7"),
    (np.bool_(True), "true"), (np.array([1.5, 2.0], np.float32), "[1.5, 2.0]"),
    (np.array([[1, 2], [3, 4]], np.int32), "[[1, 2],\n [3, 4]]"), (np.array([True, False]), "[true, false]"),
])
def test_format_result(value, text):
    assert cli.format_result(np.asarray(value)) == text


@needs_ref
def test_format_result_matches_the_reference_display():
    sys.path.insert(0, REF)
    from remora.display import format_result
    from remora.types import BOOL, FLOAT, INT, ArrayType, StaticDim

    rng = np.random.default_rng(5)
    cases = [(rng.standard_normal((3, 4)).astype(np.float32) * 1e3, FLOAT),
             (rng.standard_normal(7).astype(np.float32) * 1e-5, FLOAT),
             (rng.integers(-100, 100, (2, 3, 2)).astype(np.int32), INT), (rng.random(9) < 0.5, BOOL),
             (np.arange(40, dtype=np.float32), FLOAT)]
    for arr, elem in cases:
        t = ArrayType(elem, tuple(StaticDim(d) for d in arr.shape))
        assert cli.format_result(arr) == format_result(arr, t)
    for v, elem in [(np.float32(2.5), FLOAT), (np.float32(-0.0), FLOAT), (np.int32(3), INT), (np.bool_(False), BOOL)]:
        assert cli.format_result(np.asarray(v)) == format_result(np.asarray(v), elem)


# ------------------------------------------------------------------ plans
@pytest.mark.parametrize("rec", [r for r in plans() if "stdout" in r], ids=lambda r: r["name"])
def test_recorded_plan_prints_what_the_reference_cli_prints(rec, tmp_path, capsys, on_oracle):
    path = tmp_path / "plan.json"
    path.write_text(json.dumps(rec["plan"]))
    code, out, err = run(["--plan", str(path)], capsys)
    assert code == 0, err
    assert out == rec["stdout"].strip()


@needs_ref
@pytest.mark.parametrize("rec", [r for r in plans() if "stdout" in r][:12], ids=lambda r: r["name"])
def test_source_file_runs_as_a_whole_program(rec, tmp_path, capsys, on_oracle):
    src = tmp_path / "p.remora"
    src.write_text(rec["source"] + "\n")
    code, out, err = run([str(src), "--syntax", rec["syntax"]], capsys)
    assert code == 0, err
    assert out == rec["stdout"].strip()
    code, out, err = run([str(src), "--syntax", rec["syntax"], "--emit-plan"], capsys)
    assert code == 0, err
    assert Plan.from_record(json.loads(out)).to_record() == rec["plan"]


def test_plan_with_the_wrong_number_of_inputs_fails(tmp_path, capsys, on_oracle):
    path = tmp_path / "plan.json"
    path.write_text(json.dumps(plans()[0]["plan"]))
    arr = tmp_path / "a.npy"
    np.save(arr, np.zeros(3, np.float32))
    code, out, err = run(["--plan", str(path), "--input", str(arr)], capsys)
    assert code == 1 and err.startswith("remorac: the plan takes 0 --input arrays, got 1")


# ------------------------------------------------------------------ --call
def reference_programs() -> list[dict]:
    return json.loads((GOLDEN / "reference_programs.json").read_text())


@needs_ref
@pytest.mark.parametrize("rec", reference_programs(), ids=lambda r: r["name"])
def test_call_compiles_and_runs_the_named_function(rec, tmp_path, capsys, on_oracle):
    sys.path.insert(0, str(GOLDEN))
    import make_reference_programs as mk

    with np.load(GOLDEN / "reference_programs.npz") as f:
        ins = [f[f"{rec['name']}__in{k}"] for k in range(rec["n_inputs"])]
        want = f[f"{rec['name']}__out"]
    src = tmp_path / "f.remora"
    src.write_text(rec["source"] + "\n")
    argv = [str(src), "--syntax", rec["syntax"], "--call", next(p[3] for p in mk.PROGRAMS if p[0] == rec["name"])]
    for k, a in enumerate(ins):
        np.save(tmp_path / f"in{k}.npy", a)
        argv += ["--input", str(tmp_path / f"in{k}.npy")]
    code, out, err = run(argv, capsys)
    assert code == 0, err
    # the oracle on the recorded spec gives the interpreter's value; printed
    # the way the reference prints it
    meta = meta_from_record(rec["meta"])
    got = oracle_run(on_oracle, spec_from_record(rec["spec"]), meta, ins)
    np.testing.assert_allclose(got.astype(np.float64), want.astype(np.float64), rtol=1e-5,
                               atol=1e-6 * float(np.abs(want).max() if want.size else 0))
    assert out == cli.format_result(got)


def test_call_without_inputs_fails(tmp_path, capsys):
    src = tmp_path / "f.remora"
    src.write_text("def scale xs = map (* 2.0) xs\n")
    code, out, err = run([str(src), "--call", "scale"], capsys)
    assert (code, out) == (1, "")
    assert err == "remorac: --call requires at least one --input FILE.npy"


@needs_ref
@pytest.mark.parametrize("rec", __import__("test_program_plan").function_records(), ids=lambda r: r["name"])
def test_call_runs_a_multi_step_function_as_a_plan(rec, tmp_path, capsys, on_oracle):
    """Functions no single kernel computes (several steps, scalar parameters
    given as 0-d .npy inputs) run through --call as device plans."""
    from test_program_plan import close, function_io

    ins, want = function_io(rec)
    src = tmp_path / "f.remora"
    src.write_text(rec["source"] + "\n")
    argv = [str(src), "--syntax", rec["syntax"], "--call", rec["function"]]
    for k, a in enumerate(ins):
        np.save(tmp_path / f"in{k}.npy", a)
        argv += ["--input", str(tmp_path / f"in{k}.npy")]
    code, out, err = run(argv, capsys)
    assert code == 0, err
    # printed as the oracle's run of the recorded plan prints (numpy elides
    # the middle of arrays above 1000 elements, as the reference's display does)
    assert out == cli.format_result(run_plan_on_oracle(on_oracle, Plan.from_record(rec["plan"]), ins))
    if want.size <= 1000:
        got = np.asarray(eval(out.replace("true", "True").replace("false", "False")), dtype=want.dtype)
        close(got.reshape(want.shape), want)


@needs_ref
def test_call_of_an_unsupported_function_fails_at_compilation(tmp_path, capsys):
    src = tmp_path / "f.remora"
    src.write_text("def f xs = fold (\\acc x -> acc * x + 1.0) 1.0 xs\n")
    np.save(tmp_path / "a.npy", np.arange(4, dtype=np.float32))
    code, _, err = run([str(src), "--call", "f", "--input", str(tmp_path / "a.npy")], capsys)
    assert code == 1 and err.startswith("remorac: GPU function compilation failed:")


@needs_ref
def test_call_rejects_float64_inputs(tmp_path, capsys):
    src = tmp_path / "f.remora"
    src.write_text("def scale xs = map (* 2.0) xs\n")
    np.save(tmp_path / "a.npy", np.arange(4, dtype=np.float64))
    code, _, err = run([str(src), "--call", "scale", "--input", str(tmp_path / "a.npy")], capsys)
    assert code == 1 and "float64" in err and err.startswith("remorac:")


def test_missing_file_fails(tmp_path, capsys):
    code, _, err = run([str(tmp_path / "absent.remora")], capsys)
    assert code == 1 and err.startswith("remorac:")


@needs_ref
def test_without_a_device_execution_fails_loudly(tmp_path, capsys):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    src = tmp_path / "p.remora"
    src.write_text("fold (+) 0 (iota 10)\n")
    code, out, err = run([str(src)], capsys)
    assert (code, out) == (1, "") and err.startswith("remorac: GPU execution failed:")
