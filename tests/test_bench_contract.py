"""The bench's reference arm keeps the driver's JSON-line contract.

`bench.py --impl reference` times the reference's own CPU engine (or the
oracle's restatement when the reference library is not built) on the
Qwen2.5-0.5B-shape Q8_0 decode workload.  This test runs it with a short time
budget on the CPU and checks the one JSON line it prints.
"""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.timeout(600)
def test_reference_arm_json_line(tmp_path):
    env = dict(os.environ)
    env["B2_BENCH_DIR"] = str(tmp_path)
    env["B2_REF_SECONDS"] = "5"
    env.pop("RANK", None)
    env.pop("WORLD_SIZE", None)
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                          "--steps", "2", "--warmup", "3"],
                         cwd=ROOT, env=env, capture_output=True, text=True, timeout=580)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.strip().startswith("{")]
    assert len(lines) == 1, out.stdout
    rec = json.loads(lines[0])
    assert rec["impl"] == "reference"
    assert rec["unit"] == "tok/s" and rec["value"] > 0
    for key in ("metric", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "config", "cpu_baseline", "e2e"):
        assert key in rec, key
    assert rec["higher_is_better"] is True
    assert rec["warmup"] == 3 and 1 <= rec["steps"] <= 2
    cb = rec["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1
    assert cb["value"] == rec["value"]
    e2e = rec["e2e"]
    assert e2e["value"] == rec["value"] and e2e["unit"] == rec["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
