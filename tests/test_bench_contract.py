"""bench.py's reference arm on CPU: one JSON line with the contract's keys and
the GPU arm's own config object (no GPU needed: the arm runs the reference's
CPU path, or the port of it when the reference package is absent)."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(REPO))


def test_reference_arm_line():
    env = dict(os.environ, OMP_NUM_THREADS=os.environ.get("OMP_NUM_THREADS", "8"))
    proc = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference",
                           "--steps", "1", "--warmup", "3"], cwd=REPO, env=env,
                          capture_output=True, text=True, timeout=900)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [ln for ln in proc.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, proc.stdout[-2000:]
    line = json.loads(lines[0])
    import bench

    assert line["impl"] == "reference"
    assert line["metric"] == bench.METRIC and line["unit"] == "layer-steps/s"
    assert line["higher_is_better"] is True and line["value"] > 0
    assert line["steps"] == 1 and line["warmup"] == 3 and line["n_gpus"] == 1
    # the same config object the GPU arm prints at its defaults
    assert line["config"] == bench.cfg2_config(1, cycle=12)
    cpu = line["cpu_baseline"]
    assert cpu["kind"] in ("reference", "port") and cpu["cores"] >= 1
    assert cpu["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "layer-steps/s",
                           "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
