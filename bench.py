#!/usr/bin/env python
"""Benchmark of the Lanczos hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (configuration 1): kNN graph Laplacian, n = 1,000,000 points uniform
in [0,1]^2 (seed 1), k = 10 neighbours, union-symmetrised, Gaussian weights
with h = median 10th-neighbour distance, L = D - W (fp64 CSR).
eigsh k=20 which='LA' ncv=60 tol=1e-10 from a fixed v0 (seed 0).

One bench step = one complete eigsh solve (time to converge) with the matrix,
v0 and the eigenvector output resident on the device.  The metric is Lanczos
steps per second over the timed solves; `ms_per_step` is the time to converge.
The Krylov basis (n x 61 fp64 = 488 MB) is larger than L2, so no L2 flush is
needed between steps.

With N GPUs (torchrun), every rank solves its own copy (replicas, weak
scaling); value = all ranks' Lanczos steps / max-over-ranks time.

--impl reference times the reference's algorithm on the host cores: the CPU
oracle (C restatement of the reference IRLM, OpenMP over all cores) running
the initial 60-step Lanczos factorisation of the same matrix per step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "lanczos-gpu_b200"))

import numpy as np  # noqa: E402

N_POINTS = 1_000_000
K_EIG, NCV, TOL = 20, 60, 1e-10
WORKLOAD = (f"eigsh k={K_EIG} which=LA ncv={NCV} tol={TOL:g} on the n=1e6 kNN graph Laplacian "
            "(2-D uniform points seed 1, k=10, union-symmetrised, exp(-d^2/2h^2)), fp64 CSR")


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []
        self._t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self._t = threading.Thread(target=self._read, daemon=True)
        self._t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self._t:
            self._t.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def build_workload():
    from gpu_eigsh import synthetic as syn

    t0 = time.time()
    L, info = syn.knn_laplacian(N_POINTS, k=10, seed=1)
    v0 = np.random.default_rng(0).standard_normal(L.shape[0])
    info["build_s"] = round(time.time() - t0, 2)
    return L, v0, info


def cpu_baseline(L, v0, budget_s=20.0):
    """The oracle (reference algorithm, C, all host cores) on a bounded sample:
    repeated 60-step Lanczos factorisations of the same matrix."""
    from oracle.irlm import num_threads, oracle_lanczos_steps

    oracle_lanczos_steps(L, 4, v0, cgs2=False)  # warm (page in, thread pool)
    steps, t0 = 0, time.perf_counter()
    while True:
        oracle_lanczos_steps(L, NCV, v0, cgs2=False)
        steps += NCV
        el = time.perf_counter() - t0
        if el > budget_s or steps >= 10 * NCV:
            break
    return {"value": steps / el, "unit": "steps/s", "cores": num_threads(), "kind": "port",
            "sample": f"{steps} Lanczos steps (repeated {NCV}-step factorisations with CGS + conditional DGKS "
                      f"as the reference, n=1e6 config-1 matrix) in {el:.1f} s"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    L, v0, winfo = build_workload()
    from oracle.irlm import num_threads, oracle_lanczos_steps

    for _ in range(args.warmup):
        oracle_lanczos_steps(L, 8, v0, cgs2=False)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        oracle_lanczos_steps(L, NCV, v0, cgs2=False)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = NCV * args.steps / total
    cores = num_threads()
    line = {
        "impl": "reference", "metric": "lanczos_steps_per_sec", "value": value, "unit": "steps/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * total / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": WORKLOAD, "n": L.shape[0], "nnz": int(L.nnz),
                   "sample_per_step": f"{NCV}-step Lanczos factorisation (CGS + conditional DGKS)"},
        "cpu_baseline": {"value": value, "unit": "steps/s", "cores": cores, "kind": "port",
                         "sample": f"{args.steps} x {NCV} Lanczos steps of the config-1 matrix on {cores} threads"},
        "e2e": {"value": value, "unit": "steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=__import__("datetime").timedelta(seconds=600))

    import gpu_eigsh

    L, v0, winfo = build_workload()
    n = L.shape[0]
    dev = torch.device("cuda", local)
    rp = torch.from_numpy(L.indptr.astype(np.int32)).to(dev)
    ci = torch.from_numpy(L.indices.astype(np.int32)).to(dev)
    va = torch.from_numpy(L.data.astype(np.float64)).to(dev)
    v0d = torch.from_numpy(v0).to(dev)
    Y = torch.empty((n, K_EIG), dtype=torch.float64, device=dev)
    torch.cuda.synchronize()
    plan = gpu_eigsh.EigshPlan(None, max_ncv=NCV, mixed=args.mixed,
                               device_csr=(n, L.nnz, rp.data_ptr(), ci.data_ptr(), va.data_ptr()))

    def solve(profile=False):
        w, _ = plan.solve(k=K_EIG, which="LA", ncv=NCV, tol=TOL, v0_device=v0d.data_ptr(), evecs_out=Y.data_ptr(),
                          profile=profile)
        return w, dict(plan.last_info)

    for _ in range(args.warmup):
        solve()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    infos = []
    for _ in range(args.steps):
        w, info = solve(profile=True)
        infos.append(info)
    ev1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    steps_total = sum(i["steps"] for i in infos)
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        s = torch.tensor([float(steps_total)], device=dev, dtype=torch.float64)
        dist.all_reduce(s, op=dist.ReduceOp.SUM)
        steps_total = int(s.item())
    value = steps_total / (ms / 1000.0)

    # roofline of the dominant kernel class, from the live per-kernel events
    classes = infos[0]["kernel_ms"].keys()
    kms = {c: sum(i["kernel_ms"][c] for i in infos) for c in classes}
    kcalls = {c: sum(i["kernel_calls"][c] for i in infos) for c in classes}
    kbytes = {c: sum(i["kernel_bytes"][c] for i in infos) for c in classes}
    dom = max(kms, key=lambda c: kms[c])
    peak, peak_kind = measured_peaks()
    ach = kbytes[dom] / (kms[dom] / 1000.0) / 1e9 if kms[dom] > 0 else None
    step_cls = ["spmv", "gs_project", "gs_correct_project", "gs_correct"]
    step_ms = sum(kms[c] for c in step_cls)
    step_bytes = sum(kbytes[c] for c in step_cls)
    step_ach = step_bytes / (step_ms / 1000.0) / 1e9 if step_ms > 0 else None
    launches = sum(i["launches"] for i in infos)

    line = {
        "metric": "lanczos_steps_per_sec", "value": value, "unit": "steps/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": WORKLOAD + (" (fp32 values, fp64 accumulation)" if args.mixed else ""),
                   "n": n, "nnz": int(L.nnz), "edges": winfo["edges"], "parallelism": f"replicas{world}",
                   "l2": "inputs larger than L2 (basis 488 MB), no flush"},
        "time_to_converge_s": ms / args.steps / 1000.0,
        "lanczos_steps_per_solve": infos[0]["steps"], "restarts_per_solve": infos[0]["restarts"],
        "nconv": infos[0]["nconv"],
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": ach, "peak": peak, "unit": "GB/s",
                     "frac": (ach / peak) if ach else None, "peak_source": peak_kind,
                     "traffic": None, "avg_launch_us": 1000.0 * kms[dom] / max(1, kcalls[dom]),
                     "algorithmic_bytes_per_launch": kbytes[dom] / max(1, kcalls[dom])},
        "step_roofline": {"kernels": step_cls, "achieved": step_ach, "peak": peak, "unit": "GB/s",
                          "frac": (step_ach / peak) if step_ach else None},
        "kernel_ms_per_solve": {c: kms[c] / args.steps for c in classes},
        "gpu_launches": launches,
        "clocks": clk,
    }

    if rank == 0 and not args.no_e2e:
        # end to end through the public API with host buffers: CSR upload,
        # allocation, solve, eigenvectors back to the host
        gpu_eigsh.gpu_eigsh(L, k=K_EIG, which="LA", ncv=NCV, tol=TOL, v0=v0)  # warm
        e_steps, t0 = 0, time.perf_counter()
        reps = max(1, min(args.steps, 2))
        for _ in range(reps):
            (we, Ve), inf = gpu_eigsh.gpu_eigsh(L, k=K_EIG, which="LA", ncv=NCV, tol=TOL, v0=v0, return_info=True)
            e_steps += inf["steps"]
        el = time.perf_counter() - t0
        h2d = 4 * (n + 1) + 12 * L.nnz + 8 * n
        d2h = 8 * n * K_EIG + 8 * K_EIG
        line["e2e"] = {"value": e_steps / el, "unit": "steps/s", "h2d_bytes_per_step": h2d,
                       "d2h_bytes_per_step": d2h, "ms_per_solve": 1000.0 * el / reps}
        from scipy.sparse.linalg import norm as spnorm  # noqa: F401

        res = np.linalg.norm(L @ Ve - Ve * we, axis=0).max()
        line["max_residual_over_normA"] = float(res / abs(L).sum(axis=1).max())
    if rank == 0 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(L, v0)
    plan.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--mixed", action="store_true", help="fp32 matrix values, fp64 accumulation")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
