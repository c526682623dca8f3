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


def _bench_module():
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def test_parity_check_passes_on_oracle_outputs_and_catches_a_planted_error():
    # The bench's output check, run on CPU tensors that stand in for the device outputs.
    import numpy as np
    import torch
    import oracle
    bench = _bench_module()
    wl = bench.C1(gpu=False)
    wl.C = torch.from_numpy(oracle.Port().matmul(wl.A_h, wl.B_h))
    par = wl.parity("tf32x3", 2)
    assert par["ok"] and par["outputs"]["C"]["rel_err"] == 0.0
    wl.C[37, 411] += 1.0           # one wrong element: 1/128 of |A|.|B| there, far above 1e-5 sqrt(512)
    par = wl.parity("tf32x3", 2)
    assert not par["ok"] and par["worst_err_over_tol"] > 1.0
    assert par["ok"] is False and np.isfinite(par["outputs"]["C"]["rel_err"])


def test_parity_check_of_the_broadcast_bmm_sample():
    import numpy as np
    import torch
    import oracle
    bench = _bench_module()
    wl = bench.C3(gpu=False)
    C = oracle.Port().bmm(wl.A_h, np.broadcast_to(wl.B0_h, (64, 64, 512)))
    wl.C = torch.from_numpy(C)
    assert wl.parity("tf32", 2)["ok"]
    wl.C[63, 511, 0] = float("nan")
    assert not wl.parity("tf32", 2)["ok"]
