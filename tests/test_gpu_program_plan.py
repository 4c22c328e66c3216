"""Whole programs on the device: every recorded plan of
tests/golden/program_plans.json (the reference's acceptance programs and a
few more, planned from its front end's HIR) runs through
remora_b200.program_plan.execute_plan, one stream and one synchronisation
per program, and must give the reference's result."""

from __future__ import annotations

import numpy as np
import pytest

from remora_b200.program_plan import Plan, execute_plan
from test_program_plan import close, expected, programs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rec", programs(), ids=lambda r: r["name"])
def test_program_on_device(cuda, rec):
    close(execute_plan(Plan.from_record(rec["plan"])), expected(rec["name"]))


@pytest.mark.parametrize("rec", programs()[::4], ids=lambda r: r["name"])
def test_plan_runner_graph_replays_match_the_eager_run(cuda, rec):
    """A PlanRunner with graph=True runs eagerly once, records the steps as a
    CUDA graph, and replays it: every replay gives the eager result bit for
    bit (the kernels are deterministic) and the reference's value."""
    from remora_b200.program_plan import PlanRunner

    plan = Plan.from_record(rec["plan"])
    eager = execute_plan(plan)
    runner = PlanRunner(plan, graph=True)
    first = runner.run()[0]
    assert (runner.graph is not None) == bool(plan.steps) and runner.launches_per_run >= len(plan.steps)
    for _ in range(3):
        again = runner.run()[0]
        np.testing.assert_array_equal(again, eager)
    np.testing.assert_array_equal(first, eager)
    close(again, expected(rec["name"]))


@pytest.mark.parametrize("rec", __import__("test_program_plan").function_records(), ids=lambda r: r["name"])
def test_function_plan_on_device(cuda, rec):
    """Functions with array and scalar parameters as device plans, against
    the reference interpreter's outputs on the recorded inputs."""
    from test_program_plan import close_for, function_io

    ins, want = function_io(rec)
    close_for(rec, execute_plan(Plan.from_record(rec["plan"]), ins), want)
