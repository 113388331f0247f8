"""bench.py's reference arm keeps the driver's JSON contract (CPU only).

`bench.py --impl reference` times the compiled reference (oracle/_ref) on the host
cores; under torchrun only rank 0 runs and prints.  Skipped where the reference was
not built.
"""
import json
import os
import subprocess
import sys

import pytest

import pyoracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.skipif(pyoracle.ref_path() is None, reason="compiled reference (oracle/_ref) not built")


def _bench(*args, env=None):
    e = dict(os.environ)
    e.update(env or {})
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], capture_output=True, text=True,
                          timeout=600, env=e, cwd=ROOT)


def test_reference_arm_prints_one_contract_line():
    r = _bench("--impl", "reference", "--steps", "2", "--warmup", "3", "--cpu-seconds", "0.3")
    assert r.returncode == 0, r.stderr
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout
    line = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference"
    assert (line["steps"], line["warmup"], line["n_gpus"]) == (2, 3, 1)
    assert line["higher_is_better"] is True and line["value"] > 0
    sys.path.insert(0, ROOT)
    import bench
    assert (line["metric"], line["unit"]) == (bench.METRIC, bench.UNIT)
    cb = line["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["value"] == line["value"] and cb["cores"] >= 1 and cb["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"], "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert "workload" in line["config"]


def test_reference_arm_other_ranks_exit_quietly():
    r = _bench("--impl", "reference", "--steps", "1", "--warmup", "3", "--cpu-seconds", "0.1",
               env={"WORLD_SIZE": "2", "RANK": "1"})
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == ""
