"""bench.py's reference arm and CPU-baseline helper, on the host (no GPU needed).

The reference arm times the CPU restatement of sampler.rs on the benchmark's workload
and must print one JSON line with the keys the benchmark contract asks for.
"""
import json
import os
import subprocess
import sys

import numpy as np

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_contract_line():
    sys.path.insert(0, REPO)
    out = subprocess.run(
        [sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--steps", "2", "--warmup", "1",
         "--ref-rows", "8"],
        cwd=REPO, capture_output=True, text=True, timeout=600, check=True).stdout
    lines = [ln for ln in out.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["unit"] == "rows/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 2 and d["warmup"] == 1
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["rows_per_gpu"] == 8
    # the same config object as the GPU arm's line (same workload, same rows per step)
    import bench
    assert d["config"] == bench.headline_config(8, d["config"]["vocab"], d["config"]["window"], 1)


def test_cpu_sample_repeats_until_the_time_bound():
    sys.path.insert(0, REPO)
    sys.path.insert(0, os.path.join(REPO, "llama.rs_b200"))
    import bench
    from lrs import workloads as W
    w = W.headline(row_ids=range(4))
    rate, secs, passes = bench.cpu_sample(w, 4, 2, 0.0)
    assert passes == 1 and rate > 0 and secs > 0
    rate, secs, passes = bench.cpu_sample(w, 4, 2, 3 * secs)
    assert passes >= 2 and secs >= 0.0 and np.isfinite(rate)
