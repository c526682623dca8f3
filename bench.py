"""Benchmark: fp32-input GEMM TFLOP/s on B200 (config 5: 8192 x 8192 x 8192).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--mode tf32x3|tf32|strict]
    python bench.py --impl reference ...     # the reference's CPU matmul on the host cores

One step = one C = A.B over the whole 8192^3 problem (inputs resident in HBM; 512 MB of
operands, larger than the 126 MB L2, so no flush is needed between steps). With N > 1
GPUs (torchrun, one process per GPU, NCCL) the N columns of C are sharded over the ranks
and every rank ends with the full C (strong scaling). Prints ONE JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

N_DIM = 8192
FLOP = 2.0 * N_DIM ** 3
METRIC = "fp32-input GEMM TFLOP/s (TF32 & 3xTF32) at 1/2/4/8 B200, % of roofline"
WORKLOAD = "config5: C[8192,8192] = A[8192,8192] . B[8192,8192], A,B ~ U[-1,1] seed 1"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="mt", choices=["mt", "reference"])
    ap.add_argument("--mode", default="tf32x3", choices=["tf32x3", "tf32", "strict"])
    ap.add_argument("--no-extras", action="store_true", help="skip the other modes, e2e and CPU legs")
    ap.add_argument("--size", type=int, default=8192,
                    help="square problem size; 8192 is the benchmark, smaller sizes are profiling cases")
    return ap.parse_args()


def peaks():
    """Denominators: MEASURED_PEAKS.json (driver-measured on this pool), else the fallback."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), \
            float(p["hbm_gbs"]), "measured"
    except Exception:
        return 1590.0, 1400.0, 6650.0, "fallback"


# ------------------------------------------------------------------ clocks ----------
class ClockSampler:
    """NVML samples of SM clock and clock-event reasons while the timed region runs."""
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, device_index: int, period: float = 0.02):
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self.period = period
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                bits = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for b, name in self.REASONS.items():
                    if bits & b:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.nv is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ------------------------------------------------------------------ CPU legs ---------
def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def reference_sample(A, B, rows: int, threads: int):
    """The reference's own matmul_cpu (oracle/_ref) over C rows [0, rows) with `threads`
    host threads; falls back to the C restatement when the reference build is absent."""
    import oracle
    if oracle.have_ref():
        impl, kind = oracle.Ref(), "reference"
    else:
        impl, kind = oracle.Port(), "port"
    _, dt = impl.matmul_rows(A, B, 0, rows, threads, timing=True)
    return 2.0 * rows * A.shape[1] * B.shape[1] / dt / 1e12, dt, kind


def run_reference(args, rank):
    """--impl reference: rank 0 times the reference CPU path; other ranks exit."""
    if rank != 0:
        return
    from minitensor_b200 import inputs
    A, B = inputs.config5(N_DIM)
    threads = cpu_threads()
    rows = threads
    vals = []
    kind = "reference"
    for i in range(args.warmup + args.steps):
        v, dt, kind = reference_sample(A, B, rows, threads)
        if i >= args.warmup:
            vals.append((v, dt))
    tflops = statistics.mean(v for v, _ in vals)
    ms = statistics.mean(dt for _, dt in vals) * 1e3
    line = {
        "impl": "reference", "metric": METRIC, "value": tflops, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "sample": f"C rows 0..{rows - 1} per step ({rows} x 8192 x 8192)",
                   "threads": threads},
        "cpu_baseline": {"value": tflops, "unit": "TFLOP/s", "cores": threads, "kind": kind,
                         "sample": f"{rows} rows of C per step, reference matmul_cpu on row slices"},
        "e2e": {"value": tflops, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU arm ----------
def time_steps(fn, steps, stream):
    import torch
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(steps):
        fn()
    end.record(stream)
    torch.cuda.synchronize()
    return start.elapsed_time(end) / 1e3


def run_gpu(args, rank, world, local_rank):
    import torch
    from minitensor_b200 import engine, inputs

    global N_DIM, FLOP, WORKLOAD
    if args.size != N_DIM:
        N_DIM = args.size
        FLOP = 2.0 * N_DIM ** 3
        WORKLOAD = f"profiling case: config5 generator at {N_DIM}^3 (not the benchmark shape)"

    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    engine.lib()
    stream = torch.cuda.current_stream()
    A_h, B_h = inputs.config5(N_DIM)

    if world == 1:
        A = torch.from_numpy(A_h).cuda()
        B = torch.from_numpy(B_h).cuda()
        C = torch.empty(N_DIM, N_DIM, device="cuda")

        def step(mode=args.mode):
            engine.gemm(A, B, C, mode=mode)
    else:
        from minitensor_b200 import sharded
        plan = sharded.ShardedGemm(N_DIM, N_DIM, N_DIM, rank, world)
        A = torch.from_numpy(A_h).cuda()
        B = torch.from_numpy(np.ascontiguousarray(B_h[:, plan.n0:plan.n1])).cuda()
        C = torch.empty(N_DIM, N_DIM, device="cuda")

        def step(mode=args.mode):
            plan.run(A, B, C, mode=mode)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    n0 = engine.launch_count()
    with ClockSampler(local_rank) as clk:
        t = time_steps(step, args.steps, stream)
    launches = engine.launch_count() - n0
    if dist:
        tt = torch.tensor([t], device="cuda", dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t = float(tt.item())
    path = engine.last_path()
    tflops = FLOP * args.steps / t / 1e12
    ms = t / args.steps * 1e3

    extras = {}
    if not args.no_extras:
        # The other precisions, same workload (a few steps each).
        for m in ("tf32", "tf32x3", "strict"):
            if m == args.mode:
                continue
            s = 3 if m == "strict" else max(5, args.steps // 2)
            step(m)
            torch.cuda.synchronize()
            if dist:
                dist.barrier()
            tm = time_steps(lambda: step(m), s, stream)
            if dist:
                tt = torch.tensor([tm], device="cuda", dtype=torch.float64)
                dist.all_reduce(tt, op=dist.ReduceOp.MAX)
                tm = float(tt.item())
            extras[m] = {"value": FLOP * s / tm / 1e12, "ms_per_step": tm / s * 1e3}

    # End to end through the public API from pinned host buffers: H2D of this rank's
    # inputs, the GEMM (and the all-gather for N > 1), D2H of the full C.
    e2e = None
    if not args.no_extras:
        Ap = torch.from_numpy(A_h).pin_memory()
        Bp = torch.from_numpy(B_h if world == 1 else np.ascontiguousarray(B_h[:, plan.n0:plan.n1])).pin_memory()
        Cp = torch.empty(N_DIM, N_DIM).pin_memory()

        def e2e_step():
            A.copy_(Ap, non_blocking=True)
            B.copy_(Bp, non_blocking=True)
            step()
            Cp.copy_(C, non_blocking=True)
        e2e_step()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        s = max(3, min(args.steps, 10))
        te = time_steps(e2e_step, s, stream)
        if dist:
            tt = torch.tensor([te], device="cuda", dtype=torch.float64)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            te = float(tt.item())
        e2e = {"value": FLOP * s / te / 1e12, "unit": "TFLOP/s", "ms_per_step": te / s * 1e3,
               "h2d_bytes_per_step": int(Ap.numel() * 4 + Bp.numel() * 4), "d2h_bytes_per_step": int(Cp.numel() * 4)}

    cpu = None
    if rank == 0 and world == 1 and not args.no_extras:
        threads = cpu_threads()
        v, dt, kind = reference_sample(A_h, B_h, threads, threads)
        cpu = {"value": v, "unit": "TFLOP/s", "cores": threads, "kind": kind,
               "sample": f"C rows 0..{threads - 1} of config5 ({threads} x 8192 x 8192, {dt:.1f} s)"}

    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    bf16_burst, bf16_sust, hbm, src = peaks()
    tf32_peak = bf16_burst / 2.0   # tcgen05 kind::tf32 runs at half the bf16 rate
    per_gpu = tflops / world
    roofline = {"bound": "tensor", "achieved": per_gpu, "peak": tf32_peak, "unit": "TFLOP/s",
                "frac": per_gpu / tf32_peak, "traffic": traffic_for(args.mode),
                "peak_source": f"{src}: dense bf16 burst {bf16_burst} / 2 (tf32)",
                "kernel": path}
    if args.mode == "tf32x3":
        roofline["frac_vs_tf32_over_3"] = per_gpu / (tf32_peak / 3.0)
    line = {
        "metric": METRIC, "value": tflops, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": {"tf32x3": "fp32 (3xTF32 split, fp32-accurate)", "tf32": "tf32",
                                       "strict": "fp32"}[args.mode],
        "data": "synthetic (seeded U[-1,1], no dataset)",
        "config": {"workload": WORKLOAD, "mode": args.mode, "parallelism": f"N-column shards x{world}"
                   if world > 1 else "single GPU", "l2": "inputs 512 MB > 126 MB L2, no flush needed"},
        "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "modes": extras,
        "clocks": clk.summary(), "gpu_launches": launches,
    }
    print(json.dumps(line), flush=True)


def traffic_for(mode):
    """Per-launch DRAM bytes of the GEMM kernel from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(f"config5_{mode}")
    except Exception:
        return None


def main():
    args = parse()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", args.gpus))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    run_gpu(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
