"""The reference arm of bench.py (the `--impl reference` leg run beside the GPU arm), on the host cores here: one JSON
line with the keys read from it -- the GPU arm's metric, unit and direction, `impl`, the config-3 workload, a
`cpu_baseline` that describes the run and an `e2e` with no host<->device bytes -- and, in a multi-GPU launch, every
rank but 0 exits 0 without printing."""
import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def run_reference(env=None):
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "1"], cwd=ROOT,
                       env=dict(os.environ, **(env or {})), capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    return [line for line in r.stdout.splitlines() if line.startswith("{")]


def test_reference_arm_line():
    sys.path.insert(0, str(ROOT))
    import bench
    lines = run_reference()
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert (d["metric"], d["unit"], d["higher_is_better"]) == (bench.METRIC, "GB/s", True)
    assert d["value"] > 0 and (d["n_gpus"], d["steps"], d["warmup"]) == (1, 1, 1)
    assert d["config"]["workload"].startswith("BASELINE config 3")
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    cpu = d["cpu_baseline"]
    assert cpu["value"] == d["value"] and cpu["kind"] == "port" and cpu["cores"] >= 1 and cpu["sample"]


def test_reference_arm_other_ranks_print_nothing():
    assert run_reference({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}) == []
