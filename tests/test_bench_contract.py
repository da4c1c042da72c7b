"""bench.py's output contract, on CPU: the reference arm (the reference's
algorithm on the host cores) prints exactly one JSON line with the keys the
driver reads, for the default config and for config 3."""
import json
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

BASE_KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
             "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config"}


def _run(*args):
    env = dict(os.environ)
    env.pop("RANK", None)
    env.pop("WORLD_SIZE", None)
    p = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), *args],
                       cwd=REPO, env=env, capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.strip().startswith("{")]
    assert len(lines) == 1, p.stdout[-2000:]
    return json.loads(lines[0])


def _check_reference_line(d, unit):
    assert BASE_KEYS <= set(d), BASE_KEYS - set(d)
    assert d["impl"] == "reference"
    assert d["unit"] == unit and d["value"] > 0 and d["ms_per_step"] > 0
    assert d["higher_is_better"] is True
    assert d["warmup"] >= 3 and d["steps"] >= 1 and d["n_gpus"] >= 1
    assert "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert {"value", "unit", "cores", "kind", "sample"} <= set(cb)
    assert cb["value"] == d["value"] and cb["unit"] == unit and cb["cores"] >= 1
    assert cb["kind"] in ("port", "reference")
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == unit
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_default_config_line():
    d = _run("--impl", "reference", "--steps", "1", "--warmup", "1")
    _check_reference_line(d, "GB/s")
    assert d["metric"] == "paged_decode_attention_hbm_bandwidth"


@pytest.mark.timeout(600)
def test_reference_arm_config3_line():
    d = _run("--impl", "reference", "--config", "c3", "--steps", "1", "--warmup", "1")
    _check_reference_line(d, "TFLOP/s")
