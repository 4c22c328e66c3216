"""Programs compiled by the reference's front end and lowered by
remora_b200.reference_codegen (recorded in tests/golden/reference_programs.
{json,npz} by tests/golden/make_reference_programs.py), run on the device
through B200Executor: the same execute(kernel, host arrays) call the
reference's RemoraExecutor makes (remora/executor.py:34-117).  Outputs are
checked against the reference interpreter's: exact for int and bool, rtol
1e-5 for f32 (the interpreter computes in Python floats)."""

from __future__ import annotations

import numpy as np
import pytest

from remora_b200.codegen import SpecModule, meta_from_record, spec_from_record
from remora_b200.executor import B200Executor
from test_reference_codegen import arrays, close, records

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rec", records(), ids=lambda r: r["name"])
def test_reference_program_on_device(cuda, rec):
    a = arrays()
    spec, meta = spec_from_record(rec["spec"]), meta_from_record(rec["meta"])
    ins = [a[f"{rec['name']}__in{k}"] for k in range(rec["n_inputs"])]
    with B200Executor(SpecModule({rec["kernel"]: spec}), [meta]) as ex:
        got = ex.execute(rec["kernel"], ins)
        again = ex.execute_main(ins)
    close(got, a[f"{rec['name']}__out"])
    np.testing.assert_array_equal(got, again)
