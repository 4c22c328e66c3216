"""Generate tests/golden/program_plans.{json,npz}: whole Remora programs —
the reference's own acceptance programs (tests/acceptance/pass/
*.remora) plus a few more — compiled by the reference's front end and
planned by remora_b200.program_plan, with the result the reference
interpreter gives (remora/runtime.py:evaluate_source).  Where the acceptance
manifest holds the expected stdout of the reference's compiled CPU path, the
interpreter's value is checked against it here, and the text is recorded
for the command-line tests.  The tests replay the
recorded plans, so neither the reference nor its front end is needed to run
them.  Regenerate with:

    REMORA_REFERENCE=/path/to/remorac python tests/golden/make_program_plans.py
"""

from __future__ import annotations

import ast
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(Path(__file__).resolve().parents[2] / "oracle"))
from oracle import reference_root  # noqa: E402  (REMORA_REFERENCE, or where the oracle's build found it)

if reference_root() is None:
    raise SystemExit("set REMORA_REFERENCE to the reference checkout (the directory holding remora/)")
REF = reference_root()
sys.path.insert(0, str(REF))
sys.path.insert(0, str(ROOT))

from remora.runtime import evaluate_source  # noqa: E402

from remora_b200.errors import RemoraUnsupportedError  # noqa: E402
from remora_b200.program_plan import compile_source_to_plan  # noqa: E402

# (source, syntax): programs for the shapes the acceptance set does not reach
EXTRA = {
    "extra_scan": ("scan (+) 0.0 (map (* 0.5) (iota 20))", "ml"),
    "extra_rows": ("let xs = reshape [6, 5] (map (* 0.5) (iota 30)) in map (\\row -> fold (+) 0.0 row) xs", "ml"),
    "extra_sort": ("(sort < (map (lambda (x) (- 7 (* x 3))) (iota 9)))", "lisp"),
    "extra_grade": ("(grade < [3 1 4 1 5 9 2 6])", "lisp"),
    "extra_append": ("(append (iota 4) (map (lambda (x) (* x 10)) (iota 3)))", "lisp"),
    "extra_rotate": ("(rotate (map (lambda (x) (* x 2)) (iota 10)) 3)", "lisp"),
    "extra_row_mean": ("let xs = reshape [6, 5] (map (* 0.5) (iota 30)) in map (\\row -> fold (+) 0.0 row / 5.0) xs",
                       "ml"),
    "extra_row_span": ("let xs = reshape [4, 6] (map (\\v -> v * v - 3 * v) (iota 24)) in\n"
                       "map (\\row -> row[5] - row[0] + fold (+) 0 row) xs", "ml"),
    "extra_row_sumsq": ("let xs = reshape [8, 16] (map (* 0.25) (iota 128)) in map (\\row -> fold (+) 0.0 (map (*) row row)) xs",
                        "ml"),
    "extra_row_meansq": ("let xs = reshape [8, 16] (map (* 0.25) (iota 128)) in\n"
                         "map (\\row -> fold (+) 0.0 (map (*) row row) / 16.0) xs", "ml"),
    "extra_cell_index2": ("let m = reshape [3, 2, 2] (map (* 1.5) (iota 12)) in map (\\c -> c[1, 0] * 2.0 - c[0, 1]) m",
                          "ml"),
}


def manifest_stdout() -> dict[str, str]:
    m = json.loads((REF / "tests" / "acceptance" / "manifest.json").read_text())
    items = m if isinstance(m, list) else m.get("cases", [])
    out = {}
    for c in items:
        if isinstance(c, dict) and c.get("target") == "cpu" and "expect_stdout" in c:
            out[Path(c["path"]).stem] = c["expect_stdout"].strip()
    return out


def main() -> None:
    expected_stdout = manifest_stdout()
    sources = {p.stem: (p.read_text(), "ml")
               for p in sorted((REF / "tests" / "acceptance" / "pass").glob("*.remora"))}
    sources.update(EXTRA)
    records, arrays, skipped = [], {}, []
    for name, (src, syntax) in sources.items():
        try:
            plan = compile_source_to_plan(src, syntax=syntax)
        except RemoraUnsupportedError as exc:
            skipped.append((name, f"unsupported: {exc}"))
            continue
        except Exception as exc:  # the reference's own front end rejects it
            skipped.append((name, f"front end: {type(exc).__name__}: {str(exc)[:80]}"))
            continue
        res = plan.buffers[plan.result]
        np_t = {0: np.float32, 1: np.int32, 2: np.bool_}[res.dtype]
        try:
            value = np.asarray(evaluate_source(src, syntax=syntax).value)
        except Exception:
            # the interpreter defers some forms (slices); the manifest's
            # expected stdout of the compiled CPU path is the reference value
            if name not in expected_stdout:
                skipped.append((name, "no reference value"))
                continue
            text = expected_stdout[name].replace("true", "True").replace("false", "False")
            value = np.asarray(ast.literal_eval(text))
        want = value.astype(np_t).reshape(res.shape)
        if name in expected_stdout:
            text = expected_stdout[name].replace("true", "True").replace("false", "False")
            stated = np.asarray(ast.literal_eval(text)).astype(np_t).reshape(res.shape)
            if not np.array_equal(stated, want):
                raise SystemExit(f"{name}: the reference value {want.tolist()} differs from the manifest's {text}")
        arrays[f"{name}__out"] = want
        rec = {"name": name, "source": src.strip(), "syntax": syntax, "plan": plan.to_record(),
               "steps": [s["op"] for s in plan.steps]}
        if name in expected_stdout:
            rec["stdout"] = expected_stdout[name]  # what the reference CLI prints for it
        records.append(rec)
        print(f"{name:28s} {len(plan.steps)} steps {[s['op'] for s in plan.steps]}")
    for name, why in skipped:
        print(f"{name:28s} skipped ({why})")
    (HERE / "program_plans.json").write_text(json.dumps({"programs": records, "skipped": skipped}, indent=1) + "\n")
    np.savez(HERE / "program_plans.npz", **arrays)


if __name__ == "__main__":
    main()
