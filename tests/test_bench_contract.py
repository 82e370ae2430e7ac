"""bench.py's reference arm on the CPU: one JSON line with the driver's keys (metric, value, unit, cpu_baseline, e2e,
...), and under torchrun every rank but 0 exits 0 without work or output."""
import json
import os
import subprocess
import sys

import pytest

from conftest import REPO

KEYS = {"impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
        "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"}


def _bench(args, env=None, timeout=600):
    e = dict(os.environ)
    e.update(env or {})
    return subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), *args], cwd=REPO, env=e,
                          capture_output=True, text=True, timeout=timeout)


@pytest.mark.slow
def test_reference_arm_line():
    p = _bench(["--impl", "reference", "--steps", "1", "--warmup", "3", "--cpu-rows", "2"])
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [l for l in p.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert KEYS <= set(d), KEYS - set(d)
    assert d["impl"] == "reference" and d["metric"] == "tick frames/s" and d["unit"] == "frames/s"
    assert d["value"] > 0 and d["higher_is_better"] is True and d["scaling"] == "weak"
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert "workload" in d["config"]


def test_reference_arm_other_ranks_idle():
    p = _bench(["--impl", "reference", "--steps", "1"], env={"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"},
               timeout=120)
    assert p.returncode == 0 and not p.stdout.strip()
