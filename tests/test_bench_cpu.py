"""CPU tests of bench.py's reference arm: the JSON line the driver parses, and the
non-zero ranks of a torchrun launch exiting without work. The arm times the reference's
own CPU code (oracle/_ref, or the C restatement where that was not built)."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench(*args, env=None):
    e = dict(os.environ)
    e.update(env or {})
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT, env=e,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    return r.stdout


def test_reference_arm_prints_one_contract_line():
    out = _bench("--impl", "reference", "--workload", "c1", "--steps", "3", "--warmup", "3")
    lines = [l for l in out.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out
    line = json.loads(lines[0])
    assert line["impl"] == "reference"
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in line, k
    assert line["steps"] == 3 and line["warmup"] == 3 and line["n_gpus"] == 1
    assert line["unit"] == "TFLOP/s" and line["higher_is_better"] is True
    assert line["value"] > 0 and line["ms_per_step"] > 0
    cb = line["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert "workload" in line["config"]


def test_reference_arm_other_ranks_exit_without_work():
    out = _bench("--impl", "reference", "--workload", "c1", "--steps", "3", "--warmup", "3", "--gpus", "2",
                 env={"RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"})
    assert not [l for l in out.splitlines() if l.startswith("{")], out
