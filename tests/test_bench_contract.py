"""bench.py's reference arm on CPU: the JSON line the benchmark driver parses
(keys, units, the cpu_baseline and e2e blocks), the warm-up floor, and the
other ranks of a multi-process launch exiting quietly."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

REQUIRED = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
            "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config", "impl",
            "cpu_baseline", "e2e"}


def _run(args, env=None):
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py")] + args,
                          capture_output=True, text=True, timeout=600, cwd=ROOT,
                          env={**os.environ, **(env or {})})


def test_reference_arm_json_line():
    res = _run(["--impl", "reference", "--steps", "1", "--warmup", "1"])
    assert res.returncode == 0, res.stderr[-2000:]
    line = json.loads(res.stdout.strip().splitlines()[-1])
    assert REQUIRED <= set(line), REQUIRED - set(line)
    assert line["impl"] == "reference" and line["unit"] == "corr/s"
    assert line["warmup"] >= 3  # the floor applies even when fewer are asked
    assert line["steps"] == 1 and line["n_gpus"] == 1 and line["higher_is_better"] is True
    assert line["value"] > 0
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["cores"] >= 1 and cb["kind"] in ("port", "reference")
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"],
                           "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert "workload" in line["config"]


def test_reference_arm_other_ranks_exit_quietly():
    res = _run(["--impl", "reference", "--steps", "1", "--warmup", "3"],
               env={"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert res.returncode == 0, res.stderr[-2000:]
    assert res.stdout.strip() == ""
