"""bench.py's reference arm on the CPU: one JSON line with the contract's keys (the arm runs the
reference's CPU loop only, so it needs no GPU), for the default headline (config 5b) and for config 2."""
import json
import subprocess
import sys

import pytest

from tests.conftest import REPO


@pytest.mark.parametrize("workload", [None, "c2"], ids=["default-c5b", "c2"])
def test_reference_arm_prints_the_contract_line(workload):
    cmd = [sys.executable, "bench.py", "--impl", "reference", "--steps", "2", "--warmup", "3"]
    if workload:
        cmd += ["--workload", workload]
    res = subprocess.run(cmd, cwd=REPO, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [l for l in res.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, res.stdout
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is True
    if workload == "c2":
        assert d["config"]["workload"].startswith("C2") and d["scaling"] == "weak"
    else:
        assert d["config"]["workload"].startswith("C5b") and d["scaling"] == "strong"
        assert d["config"]["sample_elements"] > 0
    assert d["cpu_baseline"]["kind"] in ("reference", "port") and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["e2e"]["value"] == d["value"]


def test_reference_arm_other_workloads_say_unavailable():
    res = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--workload", "c4", "--steps", "1"],
                         cwd=REPO, capture_output=True, text=True, timeout=120)
    assert res.returncode == 0
    d = json.loads(res.stdout.strip().splitlines()[-1])
    assert d["impl"] == "reference" and "unavailable" in d
