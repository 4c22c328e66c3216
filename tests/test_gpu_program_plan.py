"""Whole programs on the device: every recorded plan of
tests/golden/program_plans.json (the reference's acceptance programs and a
few more, planned from its front end's HIR) runs through
remora_b200.program_plan.execute_plan, one stream and one synchronisation
per program, and must give the reference's result."""

from __future__ import annotations

import pytest

from remora_b200.program_plan import Plan, execute_plan
from test_program_plan import close, expected, programs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rec", programs(), ids=lambda r: r["name"])
def test_program_on_device(cuda, rec):
    close(execute_plan(Plan.from_record(rec["plan"])), expected(rec["name"]))
