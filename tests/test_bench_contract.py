"""
bench.py's reference arm, run on the host: the one JSON line it prints (the
reference's own CPU path for the step, on the same metric as the product arm),
and the silent exit of every rank but 0 when it is launched under torchrun.
"""

import json
import os
import subprocess
import sys

from tests.conftest import ROOT


def _reference_arm(env_extra, *args):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                           *args], capture_output=True, text=True, env=env, cwd=ROOT, timeout=600)


def _json_lines(stdout):
    return [json.loads(l) for l in stdout.splitlines() if l.startswith("{")]


def test_reference_arm_prints_one_contract_line():
    import bench
    p = _reference_arm({}, "--steps", "2", "--warmup", "3")
    assert p.returncode == 0, p.stderr[-2000:]
    lines = _json_lines(p.stdout)
    assert len(lines) == 1
    d = lines[0]
    assert d["impl"] == "reference"
    assert d["metric"] == bench.METRIC and d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["steps"] == 2 and d["warmup"] >= 3 and d["n_gpus"] == 1
    assert d["value"] > 0 and d["ms_per_step"] > 0
    # the reference's CPU path when the reference is installed, else the numpy port
    assert d["cpu_baseline"]["kind"] in ("reference", "port")
    assert d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_without_work():
    p = _reference_arm({"RANK": "1", "WORLD_SIZE": "2"}, "--steps", "2", "--warmup", "3")
    assert p.returncode == 0, p.stderr[-2000:]
    assert _json_lines(p.stdout) == []
