"""The bench.py contract on the CPU: the reference arm (`--impl reference`,
the CPU restatement of the tower on this host's cores) prints one JSON line
with every key the round-end driver reads, and `--gpus N` under several
ranks is left to the GPU runs."""
import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def _last_json(stdout: str) -> dict:
    lines = [l for l in stdout.splitlines() if l.startswith("{")]
    assert lines, stdout[-2000:]
    return json.loads(lines[-1])


@pytest.mark.timeout(600)
def test_reference_arm_line():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "1"],
                       cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    line = _last_json(r.stdout)
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference"
    assert line["unit"] == "images/s" and line["value"] > 0 and line["higher_is_better"] is True
    assert line["steps"] == 1 and line["warmup"] == 1 and line["n_gpus"] == 1
    assert line["ms_per_step"] > 0
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert "workload" in line["config"]
