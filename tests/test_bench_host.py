"""Host side of bench.py, on the CPU: the reference arm's JSON line (the
line the round-end comparison reads) and the nvidia-smi clock sampler that
every timed line carries, driven by a stand-in nvidia-smi on PATH."""

from __future__ import annotations

import json
import os
import subprocess
import sys
import time
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _run_bench(*args: str, env: dict | None = None) -> subprocess.CompletedProcess:
    e = dict(os.environ)
    e.update(env or {})
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True, text=True,
                          timeout=600, env=e, cwd=ROOT)


def test_reference_arm_prints_one_json_line():
    r = _run_bench("--impl", "reference", "--steps", "2", "--warmup", "3", env={"RANK": "0", "WORLD_SIZE": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == "CNN train samples/s" and d["unit"] == "samples/s"
    assert d["value"] > 0 and d["steps"] == 2 and d["warmup"] == 3 and d["n_gpus"] == 1
    assert d["higher_is_better"] is True
    assert d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["kind"] in ("port", "reference")
    assert d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert "workload" in d["config"]


def test_reference_arm_runs_on_rank_zero_only():
    r = _run_bench("--impl", "reference", "--steps", "2", "--warmup", "3", env={"RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [ln for ln in r.stdout.splitlines() if ln.startswith("{")]


def test_reference_arm_warmup_is_at_least_three():
    r = _run_bench("--impl", "reference", "--steps", "1", "--warmup", "1", env={"RANK": "0", "WORLD_SIZE": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    d = json.loads([ln for ln in r.stdout.splitlines() if ln.startswith("{")][0])
    assert d["warmup"] == 3


# ------------------------------------------------------------ clock sampler
ROW_BUSY = "0, 1965, 1965, 612.5, 97, 0x0000000000000004, Not Active, Not Active, Not Active, Active"
ROW_IDLE = "0, 345, 1965, 98.0, 0, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active"


def _fake_smi(tmp_path: Path, loop_rows: list[str], once_rows: list[str]) -> Path:
    """An nvidia-smi stand-in: with -lms it prints loop_rows then waits to be
    terminated; without it, once_rows."""
    d = tmp_path / "bin"
    d.mkdir()
    loop = "\n".join(f"echo '{r}'" for r in loop_rows)
    once = "\n".join(f"echo '{r}'" for r in once_rows)
    script = f"""#!/bin/sh
case "$*" in
  *-lms*)
{loop}
    exec sleep 30 ;;
  *)
{once} ;;
esac
"""
    p = d / "nvidia-smi"
    p.write_text(script)
    p.chmod(0o755)
    return d


@pytest.fixture()
def bench_mod():
    sys.path.insert(0, str(ROOT))
    import bench

    return bench


def test_clock_sampler_summarises_busy_rows(tmp_path, monkeypatch, bench_mod):
    d = _fake_smi(tmp_path, [ROW_IDLE, ROW_BUSY, ROW_BUSY, ROW_BUSY], [])
    monkeypatch.setenv("PATH", f"{d}{os.pathsep}{os.environ['PATH']}")
    s = bench_mod.ClockSampler(0)
    s.start()
    time.sleep(0.3)
    c = s.stop()
    # the idle row (0 % utilisation) is left out; sw_power_cap is reported
    assert c == {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"], "samples": 3}


def test_clock_sampler_falls_back_to_one_query(tmp_path, monkeypatch, bench_mod):
    # the sampling process prints nothing before it is stopped
    d = _fake_smi(tmp_path, [], [ROW_BUSY])
    monkeypatch.setenv("PATH", f"{d}{os.pathsep}{os.environ['PATH']}")
    s = bench_mod.ClockSampler(0)
    t0 = time.perf_counter()
    s.start()
    c = s.stop()
    assert time.perf_counter() - t0 < 20.0
    assert c is not None and c["sm_mhz"] == 1965.0 and c["samples"] == 1


def test_clock_sampler_without_nvidia_smi(tmp_path, monkeypatch, bench_mod):
    empty = tmp_path / "empty"
    empty.mkdir()
    monkeypatch.setenv("PATH", str(empty))
    s = bench_mod.ClockSampler(0)
    s.start()
    assert s.stop() is None
