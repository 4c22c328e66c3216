"""Value and gradients of fold-of-elementwise losses on the device
(remora_b200.autodiff specs recorded in tests/golden/reference_gradients.json
from the reference's front end), through B200Executor: the value against the
reference interpreter, the gradients against the reference's tape AD and,
for the reference's own three GPU gradient cases, their closed forms, at
the reference's tolerance (rtol 1e-5, atol 1e-6)."""

from __future__ import annotations

import math

import numpy as np
import pytest

from remora_b200.codegen import SpecModule, meta_from_record, spec_from_record
from remora_b200.executor import B200Executor
from test_autodiff import arrays, records

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rec", records(), ids=lambda r: r["name"])
def test_value_and_grad_on_device(cuda, rec):
    a = arrays()
    ins = [a[f"{rec['name']}__in{k}"] for k in range(rec["n_inputs"])]
    specs = {k: spec_from_record(v["spec"]) for k, v in rec["kernels"].items()}
    metas = [meta_from_record(v["meta"]) for v in rec["kernels"].values()]
    with B200Executor(SpecModule(specs), metas) as ex:
        for kname in rec["kernels"]:
            got = ex.execute(kname, ins)
            if kname.endswith("_value"):
                want = float(a[f"{rec['name']}__value"])
                if not math.isnan(want):
                    assert float(got) == pytest.approx(want, rel=1e-5, abs=1e-6)
                continue
            k = 0 if kname.endswith("_grad_x") else 1
            np.testing.assert_allclose(got, a[f"{rec['name']}__grad{k}"], rtol=1e-5, atol=1e-6)
            if k == 0 and f"{rec['name']}__closed" in a:
                np.testing.assert_allclose(got, a[f"{rec['name']}__closed"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("rec", __import__("test_autodiff").plan_records(), ids=lambda r: r["name"])
def test_value_and_grad_plan_on_device(cuda, rec):
    """The wider losses as one device plan each (forward folds, backward maps
    and folds, one stream, one synchronisation), at the tolerances the CPU
    test of the same plans states."""
    from remora_b200.autodiff import execute_value_and_grad
    from remora_b200.program_plan import Plan
    from test_autodiff import check_value_and_grads, plan_arrays

    a = plan_arrays()
    ins = [a[f"{rec['name']}__in{k}"] for k in range(len(rec["shapes"]))]
    loss, grads = execute_value_and_grad(Plan.from_record(rec["plan"]), ins)
    check_value_and_grads(rec, [np.float32(loss), *grads])


@pytest.mark.parametrize("rec", __import__("test_autodiff").plan_records(), ids=lambda r: r["name"])
def test_value_and_grad_plan_replayed_on_new_inputs(cuda, oracle_mod, rec):
    """A training loop's use: one PlanRunner with a CUDA graph, run on the
    fixture's inputs and then on new ones; each replay equals a fresh eager
    run bit for bit, and the oracle run of the same plan on the new inputs
    within the tolerances above."""
    from remora_b200.program_plan import Plan, PlanRunner, execute_plan_results
    from test_autodiff import plan_arrays
    from test_program_plan import run_plan_on_oracle

    a = plan_arrays()
    plan = Plan.from_record(rec["plan"])
    ins = [a[f"{rec['name']}__in{k}"] for k in range(len(rec["shapes"]))]
    runner = PlanRunner(plan, graph=True)
    runner.run(ins)
    rng = np.random.default_rng(11)
    for step in range(3):
        new = [np.asarray(x * np.float32(1.0 + 0.1 * (step + 1)) + np.float32(0.01) * rng.standard_normal(
            np.shape(x)).astype(np.float32), dtype=np.float32) for x in ins]
        got = runner.run(new)
        for g, e in zip(got, execute_plan_results(plan, new)):
            np.testing.assert_array_equal(g, e)
        want = run_plan_on_oracle(oracle_mod, plan, new, all_results=True)
        assert float(got[0]) == pytest.approx(float(want[0]), rel=1e-4)
        for g, w in zip(got[1:], want[1:]):
            if g.ndim == 0:
                assert float(g) == pytest.approx(float(w), rel=1e-4, abs=1e-6)
            else:
                np.testing.assert_allclose(g, w, rtol=1e-5, atol=1e-6 * float(np.abs(w).max()))
