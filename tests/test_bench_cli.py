"""bench.py's reference arm on the CPU: the JSON line the driver reads
(metric, value, unit, the e2e object with no host<->device bytes, the
cpu_baseline object), for the default workload and the media workload, and
the silence of the ranks other than 0."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(*args, env_extra=None):
    env = dict(os.environ)
    env.update(env_extra or {})
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "3",
                          "--warmup", "3", "--cpu-seconds", "0.3", *args], capture_output=True, text=True, env=env,
                         timeout=300, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    return out.stdout.strip()


def _check_line(line):
    d = json.loads(line)
    assert d["impl"] == "reference"
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "dtype", "data", "config", "e2e", "cpu_baseline"):
        assert k in d, k
    assert d["value"] > 0 and d["e2e"]["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["sample"] and cb["value"] == d["value"]
    return d


def test_reference_arm_default_workload():
    d = _check_line(_run())
    assert d["unit"] == "plans/s" and "512 candidates x 15 steps" in d["metric"]


def test_reference_arm_media_workload():
    d = _check_line(_run("--workload", "media"))
    assert d["unit"] == "frames/s" and d["dtype"] == "u8->f32"


@pytest.mark.parametrize("workload", ["skyjepa", "media"])
def test_reference_arm_other_ranks_print_nothing(workload):
    assert _run("--workload", workload, env_extra={"RANK": "1", "WORLD_SIZE": "2"}) == ""
