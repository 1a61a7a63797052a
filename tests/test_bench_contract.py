"""CPU: the benchmark's reference arm prints one JSON line with the fields
the bench contract requires (the B200 arm needs a GPU)."""

from __future__ import annotations

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(*extra):
    cmd = [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "1",
           "--parents", "8", "--cpu-sample-parents", "1", "--no-reference-cuda", *extra]
    out = subprocess.run(cmd, capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    return json.loads(lines[0])


def test_reference_arm_line():
    """The reference arm runs the reference's own ActorInferenceServer from
    its unmodified install under baseline/_ref (or reports it unavailable)."""
    d = _run()
    assert d["impl"] == "reference"
    if not os.path.isdir(os.path.join(ROOT, "baseline", "_ref", "imba_chess")):
        assert "unavailable" in d
        return
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["value"] > 0 and d["unit"] == "positions/s"
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["cpu_model"] and cb["torch"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    # the same config dict as the B200 arm's line
    assert {"workload", "rows_per_step", "parallelism"} <= set(d["config"])


def test_reference_arm_unavailable_for_search_workloads():
    d = _run("--workload", "halving")
    assert d["impl"] == "reference" and "unavailable" in d
