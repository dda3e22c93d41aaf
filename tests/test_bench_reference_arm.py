"""bench.py's reference arm on the host (no GPU needed: it times the CPU
implementation of the path and prepares its data with torch on the host when
no GPU is present): one JSON line with the keys the benchmark contract asks
for, on the small IVFFlat, flat, IVFPQ and binary configurations."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _line(*args):
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "3", *args],
                         capture_output=True, text=True, timeout=300, cwd=ROOT, env=env)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout
    return json.loads(lines[0])


@pytest.mark.parametrize("config,extra", [("ivf32k", ["--cpu-sample", "16"]),
                                          ("flat32k", []),
                                          ("ivfpq32k", ["--pq-cpu-sample", "16"]),
                                          ("binary32k", [])])
def test_reference_arm_line(config, extra):
    d = _line("--config", config, *extra)
    assert d["impl"] == "reference"
    assert d["value"] > 0 and d["unit"] == "queries/s" and d["higher_is_better"] is True
    assert d["steps"] == 1 and d["warmup"] == 3 and d["n_gpus"] == 1
    assert d["config"]["workload"].startswith(config)
    base = d["cpu_baseline"]
    assert base["value"] == d["value"] and base["cores"] >= 1 and base["kind"] in ("port", "reference")
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
