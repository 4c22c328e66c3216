"""The command line on the device: every recorded acceptance plan runs
through ``python -m remora_b200.cli --plan`` (argument handling, device plan,
result printing), and what it prints must be the reference CLI's stdout from
the acceptance manifest: the same text for integer and bool results, the same
shape and values within the fold tolerance for f32 results (the device adds
in a different order than the reference's sequential loop, which can move the
sixth printed digit)."""

from __future__ import annotations

import ast
import json

import numpy as np
import pytest

from remora_b200 import cli
from test_program_plan import programs

pytestmark = pytest.mark.gpu


def parse_printed(text: str) -> np.ndarray:
    return np.asarray(ast.literal_eval(text.replace("true", "True").replace("false", "False")))


@pytest.mark.parametrize("rec", [r for r in programs() if "stdout" in r], ids=lambda r: r["name"])
def test_cli_plan_on_device(cuda, rec, tmp_path, capsys):
    path = tmp_path / "plan.json"
    path.write_text(json.dumps(rec["plan"]))
    code = cli.main(["--plan", str(path)])
    out, err = capsys.readouterr()
    assert code == 0, err
    got, want = out.strip(), rec["stdout"].strip()
    g, w = parse_printed(got), parse_printed(want)
    assert g.shape == w.shape
    if w.dtype.kind == "f" or g.dtype.kind == "f":
        scale = float(np.abs(w).max()) if w.size else 0.0
        np.testing.assert_allclose(g.astype(np.float64), w.astype(np.float64), rtol=1e-5, atol=1e-6 * scale)
    else:
        assert got == want
