"""Host checks of bench.py's JSON contract (no GPU, no timing): both arms
describe each workload with the same config, and the reference arm runs and
reports the requested warm-up and timed steps."""
import contextlib
import io
import json
import os
import statistics
import sys

import pytest

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402


def _args(workload, steps, warmup):
    sys_argv = sys.argv
    try:
        sys.argv = ["bench.py", "--impl", "reference", "--workload", workload, "--steps", str(steps),
                    "--warmup", str(warmup)]
        return bench.parse()
    finally:
        sys.argv = sys_argv


def test_every_workload_has_one_description():
    choices = {"qgemm", "qgemm_a8", "sgemm", "gpt2", "int4", "moe", "mla", "flash"}
    assert set(bench.WORKLOADS) == choices
    assert set(bench.REF) == choices


@pytest.mark.parametrize("workload,steps,warmup,want_steps,want_warmup", [
    ("qgemm", 4, 5, 4, 5),   # light samples: every requested step
    ("gpt2", 50, 5, 3, 3),   # samples of 10 s and more: at most 3 and 3
    ("mla", 2, 3, 2, 3),
    ("flash", 50, 5, 3, 3),
])
def test_reference_line(monkeypatch, workload, steps, warmup, want_steps, want_warmup):
    calls = []

    def fake_sample():
        calls.append(1)
        return {"value": 2.0 + len(calls), "cores": 4, "kind": "port", "sample": "fake"}

    fn, metric, unit, ms_of = bench.REF[workload]
    monkeypatch.setitem(bench.REF, workload, (fake_sample, metric, unit, ms_of))
    monkeypatch.delenv("RANK", raising=False)
    out = io.StringIO()
    with contextlib.redirect_stdout(out):
        bench.run_reference(_args(workload, steps, warmup))
    line = json.loads(out.getvalue().strip().splitlines()[-1])
    assert len(calls) == want_warmup + want_steps
    assert line["impl"] == "reference" and line["metric"] == metric and line["unit"] == unit
    assert line["steps"] == want_steps and line["warmup"] == want_warmup
    # the median of the timed samples only (the warm-up samples are 3 .. want_warmup + 2)
    timed = [2.0 + i for i in range(want_warmup + 1, want_warmup + want_steps + 1)]
    assert line["value"] == statistics.median(timed)
    assert line["config"]["workload"] == bench.WORKLOADS[workload]
    assert line["e2e"] == {"value": line["value"], "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert line["cpu_baseline"]["value"] == line["value"] and line["cpu_baseline"]["cores"] == 4


def test_reference_arm_silent_on_other_ranks(monkeypatch):
    monkeypatch.setenv("RANK", "1")
    out = io.StringIO()
    with contextlib.redirect_stdout(out):
        bench.run_reference(_args("qgemm", 1, 1))
    assert out.getvalue() == ""
