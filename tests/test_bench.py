"""CPU checks of bench.py's output contract (no GPU needed).

The reference arm (`--impl reference`) runs the oracle only, so its JSON
line can be produced and checked here; the GPU arm shares the same keys and
is checked on the B200 by the round's bench runs.
"""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402

BASE_KEYS = ["metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
             "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"]


def test_config_tables_agree():
    assert set(bench.CONFIGS) == set(bench.WORKLOAD_TEXT)
    for name, (metric, n, dim, nq, k, kind) in bench.CONFIGS.items():
        assert metric in ("l2", "ip", "pq-l2"), name
        assert n > 0 and dim > 0 and nq > 0 and 0 < k <= 768, name


def test_traffic_file_entries():
    # Every committed ncu traffic line parses to a positive byte count.
    with open(os.path.join(ROOT, "profiles", "traffic.txt")) as f:
        pairs = [line.split()[:2] for line in f if line.strip() and not line.startswith("#")]
    assert pairs
    for config, kernel in pairs:
        assert config in bench.CONFIGS
        assert bench.ncu_traffic(config, kernel) > 0
    assert bench.ncu_traffic("c4k10", "no_such_kernel") is None


def test_reference_arm_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--config", "c1",
                        "--steps", "1", "--warmup", "1"],
                       cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    for key in BASE_KEYS:
        assert key in line, key
    assert line["impl"] == "reference"
    assert line["value"] > 0 and line["unit"] == "queries/s" and line["higher_is_better"] is True
    cpu = line["cpu_baseline"]
    assert cpu["kind"] == "port" and cpu["cores"] >= 1 and cpu["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "queries/s",
                           "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert line["config"]["workload"] == bench.WORKLOAD_TEXT["c1"]
