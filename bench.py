#!/usr/bin/env python
"""Benchmark of the Lanczos hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (configuration 1): kNN graph Laplacian, n = 1,000,000 points uniform
in [0,1]^2 (seed 1), k = 10 neighbours, union-symmetrised, Gaussian weights
with h = median 10th-neighbour distance, L = D - W (fp64 CSR).
eigsh k=20 which='LA' ncv=60 tol=1e-10 from a fixed v0 (seed 0).

One bench step = one complete eigsh solve (time to converge) with the matrix,
v0 and the eigenvector output resident on the device; the plan renumbers the
rows in Cuthill-McKee order when it is created (outside the timed solves; v0
and the eigenvectors stay in the caller's numbering; --no-reorder keeps the
generator's order).  The metric is Lanczos steps per second over the timed
solves; `ms_per_step` is the time to converge.
The Krylov basis (n x 61 fp64 = 488 MB) is larger than L2, so no L2 flush is
needed between steps.

With N GPUs (torchrun), the same solve runs with the rows of the matrix
split over the ranks (Cuthill-McKee order, then N row blocks; halo exchange
before each sparse product, one reduction of the Gram-Schmidt sums per pass):
strong scaling, value = the solve's Lanczos steps / max-over-ranks time.
A "mixed" object times the same solve in the mixed mode (fp32 matrix values,
fp64 accumulation and basis), and a "summary" object at the end of the line
repeats every leg's headline number.

The same line carries an "slq" object for the second half of the metric,
"SLQ logdet+grad sec" (configuration 3): slq_logdet of the IMGP precision
operator (nu = 2, theta = kappa = 1) on the undirected edges of the same kNN
graph, fp32, 64 Rademacher probes (seed 0), lanczos_m = 30, forward plus the
Kraemer backward for d/dtheta and d/dkappa.  One SLQ step = one log-det and
its gradient through the public API (operator built once, probes resident,
as in a training loop); the probe blocks (n x 64 fp32 = 256 MB) exceed L2.

Two more objects time complete solves of the other eigsh configurations:
"rmat" (configuration 4: R-MAT scale 24, k=32 LA ncv=96 tol=1e-8, fp32
values; rows partitioned over the ranks at N > 1) and "sinv" (configuration
2: shift-invert about 0 on the 128^3 Dirichlet grid, k=16 ncv=48 tol=1e-10,
inner CG to 1e-12; one GPU, N = 1 only).

--impl reference times the reference's algorithm on the host cores: the CPU
oracle (C restatement of the reference IRLM, OpenMP over every core the
process may use, whatever OMP_NUM_THREADS a launcher set) running the initial
60-step Lanczos factorisation of the same matrix per step, and the
reference's torch SLQ algorithm (oracle/slq.py) on a bounded sample.  It
builds its matrix with the seeded generators loaded by file path and never
loads the CUDA library.
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
MAXITER = 300   # implicit restarts allowed per solve (configuration 1 needs 7, R-MAT 11): a bound, not a target
WORKLOAD = (f"eigsh k={K_EIG} which=LA ncv={NCV} tol={TOL:g} on the n=1e6 kNN graph Laplacian "
            "(2-D uniform points seed 1, k=10, union-symmetrised, exp(-d^2/2h^2)), fp64 CSR")


# DRAM bytes (ncu dram__bytes_read.sum + dram__bytes_write.sum) over the
# algorithmic bytes of the same launch, per kernel class of the headline plan
# (lag steps: the SpMV without the column write, the lag projection and
# correction, the extension-end passes) and of the SLQ phases, from the
# committed ncu summaries (configuration-1 / reduced configuration-3
# captures); `traffic` = ratio x the bench's algorithmic bytes per launch.
TRAFFIC_RATIO = {"spmv": 0.975, "gs_project": 1.008, "gs_correct_project": 1.03, "gs_correct": 1.049,
                 "basis": 1.035, "slq_forward": 0.955, "slq_backward": 0.96}


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
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self._t = threading.Thread(target=self._read, daemon=True)
        self._t.start()
        # nvidia-smi takes a moment to print its first sample; a timed region
        # of a few solves can be shorter than that.  Wait for it (up to 5 s)
        # and keep only the samples taken from here on.
        t0 = time.perf_counter()
        while not self.lines and time.perf_counter() - t0 < 5.0 and self.proc.poll() is None:
            time.sleep(0.01)
        self.lines = []

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


def _synthetic():
    """gpu_eigsh/synthetic.py (numpy / scipy generators only), loaded by file
    path: importing it through the package would map the CUDA library, which
    the reference arm must not load."""
    import importlib.util

    name = "lg_synthetic_bench"
    if name not in sys.modules:
        spec = importlib.util.spec_from_file_location(name, ROOT / "lanczos-gpu_b200" / "gpu_eigsh" / "synthetic.py")
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        sys.modules[name] = mod
    return sys.modules[name]


def host_cores() -> int:
    """Cores this process may run on.  torchrun exports OMP_NUM_THREADS=1 to
    every rank; the CPU legs set their thread counts from this instead."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def build_workload():
    syn = _synthetic()

    t0 = time.time()
    L, info = syn.knn_laplacian(N_POINTS, k=10, seed=1)
    v0 = np.random.default_rng(0).standard_normal(L.shape[0])
    info["build_s"] = round(time.time() - t0, 2)
    return L, v0, info


def cpu_baseline(L, v0, budget_s=20.0):
    """The oracle (reference algorithm, C, all host cores) on a bounded sample:
    repeated 60-step Lanczos factorisations of the same matrix."""
    from oracle.irlm import num_threads, oracle_lanczos_steps, set_num_threads

    set_num_threads(host_cores())
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


SLQ_PROBES, SLQ_M, SLQ_NU = 64, 30, 2
SLQ_WORKLOAD = (f"slq_logdet of P = (2nu/theta^2 I + L_sym(kappa))^nu, nu={SLQ_NU}, theta=kappa=1, on the undirected "
                f"edges of the n=1e6 config-1 kNN graph, fp32, m_probes={SLQ_PROBES} (seed 0), lanczos_m={SLQ_M}, "
                "forward + Kraemer backward for d/dtheta, d/dkappa")


def slq_bytes(n, nnz, B, nu, m, es):
    """Algorithmic DRAM bytes of one fused SLQ forward and backward (blocks of
    n x ld, each row read or written once; CSR once per sparse product)."""
    ld = (B + 3) // 4 * 4 if es == 4 else B + (B & 1)
    blk = n * ld * es
    csr = 8 * nnz + 8 * n                      # col + value per entry, rowptr + diag per row
    dcsr = 12 * nnz + 12 * n                   # with the d/dkappa values
    if nu == 1:
        fwd_step = (3 * blk + csr) + 4 * blk
    else:
        fwd_step = (3 * blk + csr) + (nu - 2) * (2 * blk + csr) + (4 * blk + csr)
    fwd = m * fwd_step + 2 * blk                # + ||z|| pass and the final normalisation
    bwd_step = 4 * blk + (nu - 1) * (3 * blk + dcsr) + (7 * blk + dcsr)
    return fwd, m * bwd_step


def slq_edges(n=N_POINTS):
    return _synthetic().knn_edge_list(n, k=10, seed=1)


def slq_cpu_baseline(idx, d2, n=N_POINTS, m_full=SLQ_M):
    """The oracle (the reference's torch algorithm on the host cores) on a
    bounded sample: the full workload (all probes, same graph) at Lanczos depth
    1 and 2; the cost is affine in the depth (no re-orthogonalisation), so the
    two timings extrapolate to depth SLQ_M."""
    import torch
    from oracle import slq as oslq

    torch.set_num_threads(host_cores())
    it, dt = torch.from_numpy(idx), torch.from_numpy(d2).to(torch.float32)
    t = []
    for m in (1, 2):
        mv = oslq.make_precision_matvec(dt, it, n, SLQ_NU)
        e = torch.tensor(1.0, dtype=torch.float32, requires_grad=True)
        k = torch.tensor(1.0, dtype=torch.float32, requires_grad=True)
        t0 = time.perf_counter()
        ld = oslq.slq_logdet(mv, n, (e, k), m_probes=SLQ_PROBES, lanczos_m=m, seed=0, dtype=torch.float32)
        ld.backward()
        t.append(time.perf_counter() - t0)
    per_step = t[1] - t[0]
    est = t[0] + (m_full - 1) * per_step
    return {"value": est, "unit": "s/logdet+grad", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"oracle (reference torch algorithm) forward+backward, all {SLQ_PROBES} probes on the same "
                      f"graph at lanczos_m=1 ({t[0]:.1f} s) and 2 ({t[1]:.1f} s), extrapolated linearly to "
                      f"lanczos_m={m_full}"}


def run_slq(args, dev, with_e2e, with_cpu, world=1, rank=0):
    """The SLQ leg.  With N ranks the 64 probes are split across the GPUs
    (gpu_eigsh.distributed: one all-reduce of the quadrature sums, one of the
    parameter gradients), so the total work is fixed (strong scaling) and the
    time is the max over ranks."""
    import torch

    from gpu_eigsh import _slq
    from gpu_eigsh.funm_torch import slq_logdet
    from gpu_eigsh.imgp import make_imgp_precision_matvec

    n, M = args.slq_n, args.slq_m
    idx, d2 = slq_edges(n)
    mv = make_imgp_precision_matvec(x_edge_dists=torch.from_numpy(d2).to(dev, torch.float32),
                                    idx=torch.from_numpy(idx).to(dev), operator_dim=n, nu=SLQ_NU)
    ell = torch.tensor(1.0, dtype=torch.float32, device=dev, requires_grad=True)
    kap = torch.tensor(1.0, dtype=torch.float32, device=dev, requires_grad=True)
    if world > 1:
        import torch.distributed as dist

        from gpu_eigsh.distributed import probe_range, slq_logdet_sharded

    def step(e, k, device):
        e.grad = None
        k.grad = None
        if world > 1:
            ld = slq_logdet_sharded(mv, n, (e, k), m_probes=SLQ_PROBES, lanczos_m=M, seed=0, dtype=torch.float32)
        else:
            ld = slq_logdet(mv, n, (e, k), m_probes=SLQ_PROBES, lanczos_m=M, seed=0, dtype=torch.float32,
                            device=device)
        ld.backward()
        return ld

    for _ in range(args.warmup):
        step(ell, kap, dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("slq_timed")     # selects the timed steps in profiler launch lists
    ev0.record()
    for _ in range(args.steps):
        ld = step(ell, kap, dev)
    ev1.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    sec = ms / 1000.0 / args.steps
    full = (n, M) == (N_POINTS, SLQ_M)
    out = {"workload": SLQ_WORKLOAD if full else f"reduced: n={n}, lanczos_m={M}", "metric": "slq_logdet_grad_sec",
           "value": sec, "unit": "s/logdet+grad", "higher_is_better": False,
           "scaling": "strong" if world > 1 else None,
           "parallelism": f"probes sharded over {world} GPUs" if world > 1 else "1 GPU",
           "n": n, "edges": int(idx.shape[1]), "csr_nnz": mv.nnz,
           "logdet": float(ld.detach()), "grad_theta": float(ell.grad), "grad_kappa": float(kap.grad)}
    B = SLQ_PROBES
    if world > 1:
        c0, c1 = probe_range(SLQ_PROBES, rank, world)
        B = c1 - c0

    # roofline: the fused forward (nu sparse products per step, recurrence
    # folded in) and backward, timed alone with events on the launch stream
    op = mv.operator(1.0, 1.0)
    from gpu_eigsh.funm_torch import _probes

    Z = _probes(n, SLQ_PROBES, 0, torch.float32, dev)[:, :B].contiguous()
    fwd_b, bwd_b = slq_bytes(n, mv.nnz, B, SLQ_NU, M, 4)
    tf, tb = [], []
    for r in range(3):
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record()
        V, Y, al, be, zn = op.forward(Z, B, _slq.ld_for(B, torch.float32), M)
        e1.record()
        q, ga, gb, _ = _slq.small_side(al, be, zn, "log", 0, g_scale=1.0 / B)
        e2b = torch.cuda.Event(enable_timing=True)
        e2b.record()
        op.backward(V, Y, al, be, ga, gb, None, B, _slq.ld_for(B, torch.float32), M)
        e2.record()
        torch.cuda.synchronize()
        if r:
            tf.append(e0.elapsed_time(e1))
            tb.append(e2b.elapsed_time(e2))
        del V, Y
    peak, peak_kind = measured_peaks()
    f_ms, b_ms = statistics.median(tf), statistics.median(tb)
    fa, ba = fwd_b / (f_ms / 1000) / 1e9, bwd_b / (b_ms / 1000) / 1e9
    dom = ("slq_backward", ba, b_ms, bwd_b) if b_ms >= f_ms else ("slq_forward", fa, f_ms, fwd_b)
    out["roofline"] = {"bound": "hbm", "kernel": dom[0], "achieved": dom[1], "peak": peak, "unit": "GB/s",
                       "frac": dom[1] / peak, "peak_source": peak_kind,
                       "traffic": TRAFFIC_RATIO[dom[0]] * dom[3], "traffic_unit": "bytes per phase (all steps)",
                       "traffic_source": "ncu DRAM/algorithmic ratio of the phase (committed ncu summary) x algorithmic bytes",
                       "algorithmic_bytes_per_launch": dom[3], "avg_launch_ms": dom[2]}
    out["phases"] = {"forward_ms": f_ms, "forward_GBs": fa, "forward_frac": fa / peak, "forward_bytes": fwd_b,
                     "backward_ms": b_ms, "backward_GBs": ba, "backward_frac": ba / peak, "backward_bytes": bwd_b}
    nu = SLQ_NU
    out["gpu_launches_per_step"] = (1 + M * nu + 1) + 1 + (M * (1 + nu) + 1)

    if with_e2e:
        # through the public API with host parameters: lengthscale and bandwidth
        # live on the host, the log-det and both gradients come back to it
        e_h = torch.tensor(1.0, dtype=torch.float32, requires_grad=True)
        k_h = torch.tensor(1.0, dtype=torch.float32, requires_grad=True)
        step(e_h, k_h, "cpu")
        t0 = time.perf_counter()
        for _ in range(args.steps):
            step(e_h, k_h, "cpu")
        el = (time.perf_counter() - t0) / args.steps
        out["e2e"] = {"value": el, "unit": "s/logdet+grad", "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 12,
                      "note": "operator and probes stay resident across steps (built once, as in a training loop)"}
    if with_cpu:
        out["cpu_baseline"] = slq_cpu_baseline(idx, d2, n, M)
    return out


RMAT_SCALE, RMAT_K, RMAT_NCV, RMAT_TOL, RMAT_RELABEL_SEED = 24, 32, 96, 1e-8, 3
RMAT_WORKLOAD = (f"eigsh k={RMAT_K} which=LA ncv={RMAT_NCV} tol={RMAT_TOL:g} on the normalised Laplacian of an R-MAT "
                 f"graph, scale {RMAT_SCALE} (n=16,777,216), edge factor 16, (a,b,c,d)=(.57,.19,.19,.05), seed 2 "
                 "(torch CUDA generator), symmetrised, no duplicates or self-loops, vertices renumbered by a seeded "
                 "random permutation; fp32 CSR values, fp64 accumulation and basis; rows renumbered by descending "
                 "degree at plan creation (outside the timed solves; on several GPUs the sorted rows are dealt "
                 "round-robin to the row blocks)")


def run_rmat(args, dev, world=1, rank=0):
    """Configuration 4 on one GPU: generate the graph on the device, then time
    complete eigsh solves (mixed precision) with the matrix resident."""
    import torch

    import gpu_eigsh
    from gpu_eigsh import synthetic as syn

    scale = args.rmat_scale
    t0 = time.time()
    # vertices renumbered by a seeded random permutation (the same graph) so
    # that equal row blocks carry equal shares of the nonzeros; the same matrix
    # and v0 at every GPU count
    n, rp, col, val, info = syn.rmat_laplacian_device(scale, device=dev, relabel_seed=RMAT_RELABEL_SEED)
    torch.cuda.synchronize()
    gen_s = time.time() - t0
    nnz = int(col.numel())
    v0_full = np.random.default_rng(0).standard_normal(n)
    info.pop("perm", None)
    comm = None
    if world > 1:
        # rows split over the ranks (every rank generated the same graph):
        # sorted by descending degree and dealt round-robin to the row
        # blocks, so every rank holds the same share of hubs and nonzeros
        import torch.distributed as dist

        from gpu_eigsh.distributed import Communicator, partition_rows
        from gpu_eigsh.ordering import degree_order, permute_symmetric

        perm = degree_order(rp, world)
        rp, col, val, _ = permute_symmetric(rp, col, val, perm)
        v0_full = v0_full[perm.cpu().numpy()]
        del perm
        torch.cuda.empty_cache()
        comm = Communicator()
        r0, r1 = partition_rows(n, world, rank)
        a, b = int(rp[r0]), int(rp[r1])
        rp = (rp[r0:r1 + 1] - a).contiguous()
        col = col[a:b].contiguous()
        val = val[a:b].contiguous()
        plan = gpu_eigsh.EigshPlan(None, max_ncv=RMAT_NCV, mixed=True, comm=comm, n_global=n,
                                   device_csr=(r1 - r0, int(col.numel()), rp.data_ptr(), col.data_ptr(),
                                               val.data_ptr()))
    else:
        r0, r1 = 0, n
        plan = gpu_eigsh.EigshPlan(None, max_ncv=RMAT_NCV, mixed=True, reorder="degree",
                                   device_csr=(n, nnz, rp.data_ptr(), col.data_ptr(), val.data_ptr()))
    del val
    v0 = torch.from_numpy(v0_full[r0:r1].copy()).to(dev)
    Y = torch.empty((r1 - r0, RMAT_K), dtype=torch.float64, device=dev)

    def solve(profile=False):
        w, _ = plan.solve(k=RMAT_K, which="LA", ncv=RMAT_NCV, tol=RMAT_TOL, maxiter=MAXITER, v0_device=v0.data_ptr(),
                          evecs_out=Y.data_ptr(), profile=profile)
        return w, dict(plan.last_info)

    solve()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    steps = max(1, min(args.steps, 2))
    torch.cuda.nvtx.range_push("rmat_timed")
    ev0.record()
    infos = [solve(profile=True)[1] for _ in range(steps)]
    ev1.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / steps
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    w, _ = solve()
    peak, peak_kind = measured_peaks()
    classes = infos[0]["kernel_ms"].keys()
    kms = {c: sum(i["kernel_ms"][c] for i in infos) for c in classes}
    kbytes = {c: sum(i["kernel_bytes"][c] for i in infos) for c in classes}
    step_cls = ["spmv", "gs_project", "gs_correct_project", "gs_correct"]
    sms, sbytes = sum(kms[c] for c in step_cls), sum(kbytes[c] for c in step_cls)
    out = {"workload": RMAT_WORKLOAD if scale == RMAT_SCALE else f"reduced: R-MAT scale {scale}",
           "metric": "time_to_converge_s", "value": ms / 1000.0, "unit": "s", "higher_is_better": False,
           "n": n, "nnz": nnz, "edges": info["edges"], "max_degree": info["max_degree"],
           "isolated": info["isolated"], "generate_s": round(gen_s, 2),
           "lanczos_steps_per_solve": infos[0]["steps"], "restarts_per_solve": infos[0]["restarts"],
           "nconv": infos[0]["nconv"], "steps_per_sec": infos[0]["steps"] / (ms / 1000.0),
           "top_eigenvalues": [float(x) for x in w[-4:]],
           "kernel_ms_per_solve": {c: kms[c] / steps for c in classes},
           "step_roofline": {"kernels": step_cls, "achieved": sbytes / (sms / 1000) / 1e9 if sms else None,
                             "peak": peak, "unit": "GB/s", "peak_source": peak_kind,
                             "frac": (sbytes / (sms / 1000) / 1e9 / peak) if sms else None},
           "gpu_launches_per_solve": infos[0]["launches"],
           "parallelism": f"rows partitioned over {world} GPUs ({transport_name(plan)} transport)" if world > 1
           else "1 GPU",
           "scaling": "strong" if world > 1 else None}
    plan.close()
    if comm is not None:
        comm.close()
    return out


SINV_N, SINV_K, SINV_NCV, SINV_TOL, SINV_CG_TOL = 128, 16, 48, 1e-10, 1e-12
SINV_WORKLOAD = (f"eigsh sigma=0 k={SINV_K} ncv={SINV_NCV} tol={SINV_TOL:g} (shift-invert, inner CG to "
                 f"{SINV_CG_TOL:g}) on the 7-point Dirichlet Laplacian of a {SINV_N}^3 grid (n=2,097,152, "
                 "nnz=14,581,760), fp64")


def run_sinv(args, dev):
    """Configuration 2 on one GPU: the shift-invert path (Lanczos on
    (A - sigma I)^-1, every operator application one CG solve on the device),
    matrix assembled on the GPU, complete solves timed with CUDA events."""
    import torch

    import gpu_eigsh
    from gpu_eigsh import synthetic as syn

    N = args.sinv_n
    n, rp, col, val = syn.grid3d_dirichlet_device(N, device=dev)
    nnz = int(col.numel())
    plan = gpu_eigsh.EigshPlan(None, max_ncv=SINV_NCV, device_csr=(n, nnz, rp.data_ptr(), col.data_ptr(),
                                                                    val.data_ptr()))
    v0 = torch.from_numpy(np.random.default_rng(0).standard_normal(n)).to(dev)
    Y = torch.empty((n, SINV_K), dtype=torch.float64, device=dev)

    def solve(profile=False):
        w, _ = plan.solve(k=SINV_K, sigma=0.0, ncv=SINV_NCV, tol=SINV_TOL, cg_tol=SINV_CG_TOL,
                          v0_device=v0.data_ptr(), evecs_out=Y.data_ptr(), profile=profile)
        return w, dict(plan.last_info)

    solve()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("sinv_timed")
    ev0.record()
    w, info = solve(profile=True)
    ev1.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    peak, peak_kind = measured_peaks()
    cg_ms, cg_b, cg_calls = info["kernel_ms"]["cg"], info["kernel_bytes"]["cg"], info["kernel_calls"]["cg"]
    exact = syn.grid_eigenvalues(N, 3)[:400]
    near = exact[np.abs(exact[None, :] - w[:, None]).argmin(1)]
    out = {"workload": SINV_WORKLOAD if N == SINV_N else f"reduced: {N}^3 grid",
           "metric": "time_to_converge_s", "value": ms / 1000.0, "unit": "s", "higher_is_better": False,
           "n": n, "nnz": nnz, "lanczos_steps_per_solve": info["steps"], "restarts_per_solve": info["restarts"],
           "cg_iterations_per_solve": info["cg_iters"],
           "cg_iterations_per_operator_application": info["cg_iters"] / max(1, info["steps"]),
           "nconv": info["nconv"], "max_rel_err_vs_analytic": float(np.max(np.abs(w - near) / near)),
           "eigenvalues": [float(x) for x in w[:4]],
           "kernel_ms_per_solve": dict(info["kernel_ms"]),
           "roofline": {"bound": "hbm", "kernel": "cg (cg_k1 + cg_k2, one CG iteration)",
                        "achieved": cg_b / (cg_ms / 1000.0) / 1e9 if cg_ms else None, "peak": peak, "unit": "GB/s",
                        "frac": (cg_b / (cg_ms / 1000.0) / 1e9 / peak) if cg_ms else None, "peak_source": peak_kind,
                        "avg_iteration_us": 1000.0 * cg_ms / max(1, cg_calls),
                        "algorithmic_bytes_per_iteration": cg_b / max(1, cg_calls)},
           "gpu_launches_per_solve": info["launches"], "parallelism": "1 GPU"}
    plan.close()
    return out


GRAPH_N, GRAPH_DIM, GRAPH_K, GRAPH_BW, GRAPH_SEED = 100_000, 10, 15, 0.3, 123
GRAPH_WORKLOAD = (f"kNN graph Laplacian of benchmark/generate_large_laplacian.py's defaults: n={GRAPH_N:,} points "
                  f"RandomState({GRAPH_SEED}).random((n, {GRAPH_DIM})), k={GRAPH_K}, weights exp(-d^2/(4 bw^2)) "
                  f"bw={GRAPH_BW}, A.maximum(A.T), L = D - A (exact neighbours, fp64)")


def run_graph(args, dev, with_cpu):
    """Graph construction on one GPU: lg_knn (all-pairs tiles at dim 10) and
    the Laplacian assembly, points resident (value) and from host points to a
    host CSR (e2e); the reference generator's cKDTree path timed on the host
    as the CPU baseline (oracle/graph.py restates it)."""
    import torch

    from gpu_eigsh import graph as G

    pts = G.generate_points(GRAPH_N, GRAPH_DIM, GRAPH_SEED)
    P = torch.from_numpy(pts).to(dev)

    def build():
        idx, d2 = G.knn(P, GRAPH_K)
        return G.laplacian_from_knn(idx, d2, GRAPH_BW)

    for _ in range(2):
        build()
    torch.cuda.synchronize()
    e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    reps, t_knn, t_all = 3, [], []
    for _ in range(reps):
        e[0].record()
        idx, d2 = G.knn(P, GRAPH_K)
        e[1].record()
        rp, col, val = G.laplacian_from_knn(idx, d2, GRAPH_BW)
        e[2].record()
        torch.cuda.synchronize()
        t_knn.append(e[0].elapsed_time(e[1]))
        t_all.append(e[0].elapsed_time(e[2]))
    nnz = int(rp[-1])
    # end to end: host points in, host scipy CSR out
    t0 = time.perf_counter()
    L = G.generate_knn_laplacian(GRAPH_N, GRAPH_DIM, GRAPH_K, GRAPH_BW, GRAPH_SEED)
    e2e_s = time.perf_counter() - t0
    knn_ms = min(t_knn)
    pairs = float(GRAPH_N) * (GRAPH_N - 1)
    out = {"workload": GRAPH_WORKLOAD, "metric": "graph_build_s", "value": min(t_all) / 1000.0, "unit": "s",
           "higher_is_better": False, "n": GRAPH_N, "nnz": nnz, "knn_ms": knn_ms,
           "laplacian_ms": min(t_all) - knn_ms,
           "knn_search": "all-pairs tiles (dim > 3), fp64, contraction-free distance sums",
           "distance_pairs_per_s": pairs / (knn_ms / 1000.0),
           "fp64_ops_per_s": pairs * GRAPH_DIM * 3 / (knn_ms / 1000.0),
           "e2e": {"value": e2e_s, "unit": "s", "h2d_bytes": pts.nbytes, "d2h_bytes": int(L.data.nbytes +
                                                                                            L.indices.nbytes +
                                                                                            L.indptr.nbytes)},
           "parallelism": "1 GPU"}
    if with_cpu:
        from oracle import graph as OG

        t0 = time.perf_counter()
        OG.generator_laplacian(GRAPH_N, GRAPH_DIM, GRAPH_K, GRAPH_BW, GRAPH_SEED)
        out["cpu_baseline"] = {"value": time.perf_counter() - t0, "unit": "s", "cores": 1, "kind": "port",
                               "sample": "the full workload: the generator's cKDTree build and query (one thread, as "
                                         "the script calls it) and its scipy assembly"}
    return out


class HeadlineSolver:
    """The configuration-1 solve of the headline.

    One GPU: an EigshPlan on the device CSR that renumbers the rows in
    Cuthill-McKee order inside the plan (LG_PLAN_REORDER_BFS).  N GPUs: the
    same Cuthill-McKee order applied before the split (gpu_eigsh.ordering),
    rows in N blocks (gpu_eigsh.distributed.PartitionedEigsh), the halo of
    boundary rows exchanged before each sparse product, one solve shared by
    all ranks (strong scaling).  solve(profile) -> (eigenvalues, info)."""

    def __init__(self, L, v0, dev, world, rank, mixed=False, reorder=True):
        import torch

        import gpu_eigsh

        self.world, self.n = world, L.shape[0]
        n = self.n
        rp = torch.from_numpy(L.indptr.astype(np.int32)).to(dev)
        ci = torch.from_numpy(L.indices.astype(np.int32)).to(dev)
        va = torch.from_numpy(L.data.astype(np.float64)).to(dev)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        if world == 1:
            self.comm = None
            self.plan = gpu_eigsh.EigshPlan(None, max_ncv=NCV, mixed=mixed, reorder=reorder,
                                            device_csr=(n, L.nnz, rp.data_ptr(), ci.data_ptr(), va.data_ptr()))
            self.v0 = torch.from_numpy(v0).to(dev)
            self.Y = torch.empty((n, K_EIG), dtype=torch.float64, device=dev)
            self.exchange = None
        else:
            from gpu_eigsh.distributed import Communicator, PartitionedEigsh, partition_rows
            from gpu_eigsh.ordering import cm_order, permute_symmetric

            perm = cm_order(rp, ci)
            self.perm = perm.cpu().numpy()
            rp, ci, va, _ = permute_symmetric(rp, ci, va, perm)
            r0, r1 = partition_rows(n, world, rank)
            a, b = int(rp[r0]), int(rp[r1])
            lrp = (rp[r0:r1 + 1] - a).contiguous()
            lci, lva = ci[a:b].contiguous(), va[a:b].contiguous()
            self.v0 = torch.from_numpy(v0).to(dev)[perm][r0:r1].contiguous()
            self.comm = Communicator()
            self.pe = PartitionedEigsh(self.comm, n, lrp, lci, lva, max_ncv=NCV, mixed=mixed)
            self.plan = self.pe.plan
            self.Y = torch.empty((r1 - r0, K_EIG), dtype=torch.float64, device=dev)
            self.exchange = self.pe.exchange_info
            self.rows = (r0, r1)
        torch.cuda.synchronize()
        self.plan_s = time.perf_counter() - t0

    def solve(self, profile=False):
        w, _ = self.plan.solve(k=K_EIG, which="LA", ncv=NCV, tol=TOL, maxiter=MAXITER, v0_device=self.v0.data_ptr(),
                               evecs_out=self.Y.data_ptr(), profile=profile)
        return w, dict(self.plan.last_info)

    def close(self):
        self.plan.close()
        if self.comm is not None:
            self.comm.close()


def transport_name(plan):
    """'peer' (reductions and exchanges as kernels over NVLink peer memory) or
    'nccl', as the partitioned plan chose."""
    import ctypes as C

    from gpu_eigsh import _native

    m = C.c_int(0)
    _native.check(_native.lib.lg_eigsh_plan_transport(plan._plan, C.byref(m)))
    return {v: k for k, v in _native.TRANSPORT.items()}[m.value]


def max_over_ranks(x, dev, world):
    import torch
    import torch.distributed as dist

    if world == 1:
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def e2e_partitioned(args, L, v0, dev, world, rank):
    """End to end at N GPUs through the public API: each rank copies its
    slice of the (already renumbered) host CSR and v0 from pinned host memory,
    builds the partitioned plan (a collective: halo lists), solves, and
    copies its rows of the eigenvectors back to the host.  Wall time per
    call, max over ranks."""
    import torch
    import torch.distributed as dist

    from gpu_eigsh.distributed import Communicator, PartitionedEigsh, partition_rows

    n = L.shape[0]
    rp = torch.from_numpy(L.indptr.astype(np.int32))
    ci = torch.from_numpy(L.indices.astype(np.int32))
    r0, r1 = partition_rows(n, world, rank)
    a, b = int(rp[r0]), int(rp[r1])
    h_rp = (rp[r0:r1 + 1] - a).pin_memory()
    h_ci = ci[a:b].pin_memory()
    h_va = torch.from_numpy(L.data[a:b].astype(np.float64)).pin_memory()
    h_v0 = torch.from_numpy(v0[r0:r1].copy()).pin_memory()
    comm = Communicator()

    phases = {}
    # the eigenvector rows come back into pinned host memory (allocated once,
    # like the pinned input slices above)
    Yh = torch.empty((r1 - r0, K_EIG), dtype=torch.float64).pin_memory()

    def call():
        t0 = time.perf_counter()
        d_rp, d_ci = h_rp.to(dev, non_blocking=True), h_ci.to(dev, non_blocking=True)
        d_va, d_v0 = h_va.to(dev, non_blocking=True), h_v0.to(dev, non_blocking=True)
        pe = PartitionedEigsh(comm, n, d_rp, d_ci, d_va, max_ncv=NCV)
        t1 = time.perf_counter()
        w, Y = pe.solve(K_EIG, d_v0, which="LA", ncv=NCV, tol=TOL, maxiter=MAXITER)
        t2 = time.perf_counter()
        Yh.copy_(Y)
        t3 = time.perf_counter()
        steps = pe.last_info["steps"]
        pe.close()
        t4 = time.perf_counter()
        phases.update(upload_and_plan=1e3 * (t1 - t0), solve=1e3 * (t2 - t1), evecs_d2h=1e3 * (t3 - t2),
                      close=1e3 * (t4 - t3))
        return w, Yh, steps

    call()
    reps = max(1, min(args.steps, 2))
    dist.barrier()
    t0 = time.perf_counter()
    steps = 0
    for _ in range(reps):
        _, _, st = call()
        steps += st
    dist.barrier()
    el = max_over_ranks(time.perf_counter() - t0, dev, world)
    comm.close()
    h2d = int(h_rp.numel() * 4 + h_ci.numel() * 4 + h_va.numel() * 8 + h_v0.numel() * 8)
    d2h = int((r1 - r0) * K_EIG * 8)
    return {"value": steps / el, "unit": "steps/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_solve": 1000.0 * el / reps,
            "host_ms_last_call": {k: round(v, 2) for k, v in phases.items()},
            "note": "rank 0's bytes and phases; every rank copies its own CSR slice and eigenvector rows"}


ADJ_K = 20
ADJ_WORKLOAD = (f"differentiable_eigsh backward (implicit differentiation, k={ADJ_K} smallest pairs, reference "
                "defaults ncv=3k maxiter=3000 tol=1e-12, cg_max_iters=500 cg_tol=1e-10) on the n=1e6 kNN graph "
                "Laplacian, random upstream gradients on all eigenvalues and eigenvectors (seed 0)")


def adj_bytes_per_iteration(n, nnz, k):
    """Algorithmic DRAM bytes of one block-CG iteration of lg_eigsh_adjoint
    (blocks n x ld doubles, ld = k rounded up to 8): the sparse product reads
    the CSR and P and writes AP; the update reads P, AP, Xi, R and writes Xi,
    R; the Gram reads X and R; the deflation reads X, R, P and writes R, P."""
    blk = 8 * n * ((k + 7) // 8 * 8)
    return (12 * nnz + 4 * (n + 1) + 2 * blk) + 6 * blk + 2 * blk + 5 * blk


def run_adjoint(args, L, dev, with_cpu):
    """The differentiable eigsh backward on configuration 1: eigenpairs from
    the forward (outside the timed region), then loss.backward() timed with
    CUDA events on the stream the adjoint runs on."""
    import torch

    from gpu_eigsh import differentiable_eigsh

    n = L.shape[0]
    crow = torch.from_numpy(L.indptr.astype(np.int64)).to(dev)
    col = torch.from_numpy(L.indices.astype(np.int64)).to(dev)
    rng = np.random.default_rng(0)
    ge = torch.from_numpy(rng.standard_normal(ADJ_K)).to(dev)
    gv = torch.from_numpy(rng.standard_normal((n, ADJ_K))).to(dev)
    times, info = [], None
    for rep in range(2):
        vals = torch.from_numpy(L.data.astype(np.float64)).to(dev).requires_grad_(True)
        A = torch.sparse_csr_tensor(crow, col, vals, L.shape, check_invariants=False)
        t0 = time.perf_counter()
        w, V = differentiable_eigsh(A, k=ADJ_K)
        fwd_s = time.perf_counter() - t0
        loss = (w * ge).sum() + (V * gv).sum()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        loss.backward()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
        if rep == 0:
            # the iteration counts of the pairs, from the autograd node
            node = w.grad_fn
            info = {"cg_iters": list(getattr(node, "cg_iters", [])), "forward_s": fwd_s,
                    "eigenvalues": [float(x) for x in w.detach().cpu()[:4]]}
    ms = times[-1]
    iters = max(abs(i) for i in info["cg_iters"]) if info["cg_iters"] else 0
    peak, peak_kind = measured_peaks()
    bpi = adj_bytes_per_iteration(n, L.nnz, ADJ_K)
    ach = bpi * iters / (ms / 1000.0) / 1e9 if iters else None
    out = {"workload": ADJ_WORKLOAD, "metric": "adjoint_backward_s", "value": ms / 1000.0, "unit": "s",
           "higher_is_better": False, "k": ADJ_K, "block_cg_iterations": iters,
           "cg_iterations_per_pair": info["cg_iters"], "forward_s": round(info["forward_s"], 3),
           "roofline": {"bound": "hbm", "kernel": "block CG iteration (adj_spmm, adj_update, adj_gram, adj_deflate)",
                        "achieved": ach, "peak": peak, "unit": "GB/s", "frac": (ach / peak) if ach else None,
                        "peak_source": peak_kind, "algorithmic_bytes_per_iteration": bpi,
                        "note": "whole backward time (incl. setup and the gradient SDDMM) / iterations"},
           "parallelism": "1 GPU"}
    if with_cpu:
        out["cpu_baseline"] = adjoint_cpu_baseline(L, w.detach().cpu().numpy(), V.detach().cpu().numpy(),
                                                    gv[:, 0].cpu().numpy(), max(iters, 1))
    return out


def adjoint_cpu_baseline(L, w, X, g0, iters_gpu, sample_iters=30):
    """The oracle (the reference's per-pair deflated CG, numpy/scipy on the host)
    on a bounded sample: one pair, `sample_iters` CG iterations, scaled to k
    pairs x the GPU's iteration count."""
    from oracle import adjoint as OA

    rhs = OA.deflate(g0.copy(), X)
    OA.cg_deflated(L, float(w[0]), rhs, X, tol=0.0, max_iters=2)   # warm
    t0 = time.perf_counter()
    OA.cg_deflated(L, float(w[0]), rhs, X, tol=0.0, max_iters=sample_iters)
    el = time.perf_counter() - t0
    per_it = el / sample_iters
    return {"value": per_it * iters_gpu * ADJ_K, "unit": "s", "cores": host_cores(), "kind": "port",
            "sample": f"{sample_iters} deflated-CG iterations of one pair in {el:.2f} s, scaled to {ADJ_K} pairs x "
                      f"{iters_gpu} iterations (scipy sparse matvec + numpy deflation, host BLAS threads)"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    L, v0, winfo = build_workload()
    from oracle.irlm import num_threads, oracle_lanczos_steps, set_num_threads

    set_num_threads(host_cores())
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
    if not args.no_slq:
        del L
        idx, d2 = slq_edges()
        cb = slq_cpu_baseline(idx, d2)
        line["slq"] = {"workload": SLQ_WORKLOAD, "metric": "slq_logdet_grad_sec", "value": cb["value"],
                       "unit": cb["unit"], "higher_is_better": False, "cpu_baseline": cb,
                       "e2e": {"value": cb["value"], "unit": cb["unit"], "h2d_bytes_per_step": 0,
                               "d2h_bytes_per_step": 0}}
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
                                timeout=__import__("datetime").timedelta(seconds=180))

    import gpu_eigsh

    if args.only_rmat:
        out = run_rmat(args, torch.device("cuda", local), world=world, rank=rank)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps(out), flush=True)
        return 0
    if args.only_adjoint:
        L, _, _ = build_workload()
        out = run_adjoint(args, L, torch.device("cuda", local), with_cpu=not args.no_cpu_baseline) if rank == 0 \
            else None
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps(out), flush=True)
        return 0
    if args.only_graph:
        out = run_graph(args, torch.device("cuda", local), with_cpu=not args.no_cpu_baseline) if rank == 0 else None
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps(out), flush=True)
        return 0
    if args.only_sinv:
        out = run_sinv(args, torch.device("cuda", local)) if rank == 0 else None
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps(out), flush=True)
        return 0
    if args.only_slq:
        out = run_slq(args, torch.device("cuda", local), with_e2e=False, with_cpu=False, world=world, rank=rank)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps(out), flush=True)
        return 0
    L, v0, winfo = build_workload()
    n = L.shape[0]
    dev = torch.device("cuda", local)
    hs = HeadlineSolver(L, v0, dev, world, rank, mixed=args.mixed, reorder=args.reorder)

    for _ in range(args.warmup):
        hs.solve()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("eigsh_timed")   # selects the timed solves in profiler launch lists
    ev0.record()
    timed_infos = []
    for _ in range(args.steps):
        w, info = hs.solve()
        timed_infos.append(info)
    ev1.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = max_over_ranks(ev0.elapsed_time(ev1), dev, world)
    # one solve shared by all ranks: its Lanczos steps (the same on every rank)
    steps_total = sum(i["steps"] for i in timed_infos)
    value = steps_total / (ms / 1000.0)
    # the same solves again with a CUDA event pair around every launch (the
    # per-kernel times of the roofline); recording ~1800 events adds ~15 % to
    # a solve, so the timed solves above run without them
    infos = [hs.solve(profile=True)[1] for _ in range(args.steps)]

    # roofline of the dominant kernel class, from the live per-kernel events
    # (rank 0's rows at N > 1)
    classes = infos[0]["kernel_ms"].keys()
    kms = {c: sum(i["kernel_ms"][c] for i in infos) for c in classes}
    kcalls = {c: sum(i["kernel_calls"][c] for i in infos) for c in classes}
    kbytes = {c: sum(i["kernel_bytes"][c] for i in infos) for c in classes}
    # the dominant kernel class among those that move data (not the comm waits)
    dom = max((c for c in kms if kbytes[c] > 0), key=lambda c: kms[c])
    peak, peak_kind = measured_peaks()
    ach = kbytes[dom] / (kms[dom] / 1000.0) / 1e9 if kms[dom] > 0 else None
    step_cls = ["spmv", "gs_project", "gs_correct_project", "gs_correct"]
    step_ms = sum(kms[c] for c in step_cls)
    step_bytes = sum(kbytes[c] for c in step_cls)
    step_ach = step_bytes / (step_ms / 1000.0) / 1e9 if step_ms > 0 else None
    # The events of the profile pass also cost the step kernels their
    # programmatic overlap.  In the timed solves (no events) the step kernels
    # run for the solve time less the other kernels (restart, V*Q, peer waits,
    # as the profile pass timed them): the same bytes over that time.
    # (one GPU only: the profile pass's peer waits are longer than the timed
    # solve's, so at N > 1 this would credit the step kernels with wait time)
    other_ms = sum(kms[c] for c in classes if c not in step_cls) / args.steps
    step_timed_ms = ms / args.steps - other_ms
    step_timed_ach = ((step_bytes / args.steps) / (step_timed_ms / 1000.0) / 1e9
                      if step_timed_ms > 0 and world == 1 else None)
    launches = sum(i["launches"] for i in timed_infos)
    if world > 1:
        par = (f"rows partitioned over {world} GPUs (Cuthill-McKee order, {hs.exchange[0]} exchange, "
               f"{transport_name(hs.plan)} transport)")
    else:
        par = "1 GPU"

    line = {
        "metric": "lanczos_steps_per_sec", "value": value, "unit": "steps/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": WORKLOAD + (" (fp32 values, fp64 accumulation)" if args.mixed else "")
                   + ("; rows renumbered in Cuthill-McKee order at plan creation (outside the timed solves; v0 "
                      "and eigenvectors in the caller's numbering)" if args.reorder or world > 1 else ""),
                   "n": n, "nnz": int(L.nnz), "edges": winfo["edges"], "parallelism": par,
                   "l2": "inputs larger than L2 (basis 488 MB), no flush"},
        "time_to_converge_s": ms / args.steps / 1000.0, "plan_create_s": hs.plan_s,
        "lanczos_steps_per_solve": timed_infos[0]["steps"], "restarts_per_solve": timed_infos[0]["restarts"],
        "nconv": timed_infos[0]["nconv"], "top_eigenvalues": [float(x) for x in w[-4:]],
        "kernel_times": "per-kernel CUDA events in a second pass of the same solves (profile mode)",
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": ach, "peak": peak, "unit": "GB/s",
                     "frac": (ach / peak) if ach else None, "peak_source": peak_kind,
                     "traffic": (TRAFFIC_RATIO[dom] * kbytes[dom] / max(1, kcalls[dom])) if dom in TRAFFIC_RATIO
                     else None,
                     "traffic_source": "ncu DRAM/algorithmic ratio of this kernel (committed ncu summary) x algorithmic bytes",
                     "avg_launch_us": 1000.0 * kms[dom] / max(1, kcalls[dom]),
                     "algorithmic_bytes_per_launch": kbytes[dom] / max(1, kcalls[dom])},
        "step_roofline": {"kernels": step_cls, "achieved": step_ach, "peak": peak, "unit": "GB/s",
                          "frac": (step_ach / peak) if step_ach else None,
                          "timed_solve": {"achieved": step_timed_ach,
                                          "frac": (step_timed_ach / peak) if step_timed_ach else None,
                                          "ms_per_solve": step_timed_ms if world == 1 else None,
                                          "definition": "step-kernel bytes per solve / (timed solve time - "
                                                        "profile-pass time of the other kernel classes)"}},
        "kernel_ms_per_solve": {c: kms[c] / args.steps for c in classes},
        "gpu_launches": launches,
        "clocks": clk,
    }
    if world > 1:
        line["exchange"] = {"mode": hs.exchange[0], "halo_rows_received_rank0": hs.exchange[1],
                            "halo_rows_sent_rank0": hs.exchange[2], "rows_rank0": list(hs.rows)}
    perm = getattr(hs, "perm", None)
    hs.close()

    if not args.no_e2e:
        if world == 1:
            # end to end through the public API with host buffers: CSR upload,
            # allocation, solve, eigenvectors back to the host
            gpu_eigsh.gpu_eigsh(L, k=K_EIG, which="LA", ncv=NCV, tol=TOL, maxiter=MAXITER, v0=v0)  # warm
            e_steps, t0 = 0, time.perf_counter()
            reps = max(1, min(args.steps, 2))
            phases = []
            for _ in range(reps):
                (we, Ve), inf = gpu_eigsh.gpu_eigsh(L, k=K_EIG, which="LA", ncv=NCV, tol=TOL, maxiter=MAXITER,
                                                   v0=v0, return_info=True)
                e_steps += inf["steps"]
                phases.append(inf["host_ms"])
            el = time.perf_counter() - t0
            h2d = 4 * (n + 1) + 12 * L.nnz + 8 * n
            d2h = 8 * n * K_EIG + 8 * K_EIG
            line["e2e"] = {"value": e_steps / el, "unit": "steps/s", "h2d_bytes_per_step": h2d,
                           "d2h_bytes_per_step": d2h, "ms_per_solve": 1000.0 * el / reps,
                           "host_ms_last_call": {k: round(v, 2) for k, v in phases[-1].items()}}
            res = np.linalg.norm(L @ Ve - Ve * we, axis=0).max()
            line["max_residual_over_normA"] = float(res / abs(L).sum(axis=1).max())
        else:
            Lp = L[perm][:, perm].tocsr()
            Lp.sort_indices()
            line["e2e"] = e2e_partitioned(args, Lp, v0[perm], dev, world, rank)
            del Lp
    if rank == 0 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(L, v0)
    if world == 1 and not args.no_mixed:
        line["mixed"] = run_mixed(args, L, v0, dev)
    if world == 1 and not args.no_adjoint:
        line["adjoint"] = run_adjoint(args, L, dev, with_cpu=not args.no_cpu_baseline)
    del L
    if not args.no_slq:
        # with N > 1 every rank takes part in the sharded e2e steps (collectives)
        line["slq"] = run_slq(args, dev, with_e2e=(not args.no_e2e) and (world > 1 or rank == 0),
                              with_cpu=(rank == 0 and not args.no_cpu_baseline), world=world, rank=rank)
        line["gpu_launches"] += line["slq"]["gpu_launches_per_step"] * args.steps
    if not args.no_rmat:
        line["rmat"] = run_rmat(args, dev, world=world, rank=rank)
    if not args.no_sinv and world == 1:
        # the shift-invert path is single-GPU (every rank would repeat it)
        line["sinv"] = run_sinv(args, dev)
    if not args.no_graph and world == 1:
        line["graph"] = run_graph(args, dev, with_cpu=not args.no_cpu_baseline)
    line["summary"] = summary(line)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def run_mixed(args, L, v0, dev):
    """Configuration 1 in the mixed mode (fp32 matrix values, fp64
    accumulation and basis), one GPU: complete solves timed with CUDA events."""
    import torch

    hs = HeadlineSolver(L, v0, dev, 1, 0, mixed=True, reorder=args.reorder)
    hs.solve()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = max(1, min(args.steps, 5))
    ev0.record()
    infos = [hs.solve() for _ in range(reps)]
    ev1.record()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / reps
    w, info = infos[-1]
    prof = hs.solve(profile=True)[1]
    hs.close()
    return {"workload": WORKLOAD + " (fp32 values, fp64 accumulation and basis)", "metric": "lanczos_steps_per_sec",
            "value": info["steps"] / (ms / 1000.0), "unit": "steps/s", "time_to_converge_s": ms / 1000.0,
            "lanczos_steps_per_solve": info["steps"], "restarts_per_solve": info["restarts"],
            "nconv": info["nconv"], "top_eigenvalues": [float(x) for x in w[-4:]],
            "kernel_ms_per_solve": dict(prof["kernel_ms"]), "parallelism": "1 GPU"}


def summary(line):
    """The headline figures of every leg in a few keys, last on the line."""
    def g(obj, *keys):
        for k in keys:
            if not isinstance(obj, dict) or k not in obj:
                return None
            obj = obj[k]
        return obj

    out = {"eigsh_steps_per_s": line["value"], "eigsh_s": line["time_to_converge_s"],
           "eigsh_e2e_steps_per_s": g(line, "e2e", "value"), "eigsh_step_frac": g(line, "step_roofline", "frac"),
           "eigsh_step_frac_timed": g(line, "step_roofline", "timed_solve", "frac"),
           "eigsh_cpu_steps_per_s": g(line, "cpu_baseline", "value"),
           "mixed_s": g(line, "mixed", "time_to_converge_s"),
           "slq_s": g(line, "slq", "value"), "slq_e2e_s": g(line, "slq", "e2e", "value"),
           "slq_cpu_s": g(line, "slq", "cpu_baseline", "value"),
           "rmat_s": g(line, "rmat", "value"), "sinv_s": g(line, "sinv", "value"),
           "adjoint_s": g(line, "adjoint", "value"), "graph_s": g(line, "graph", "value")}
    return {k: (round(v, 6) if isinstance(v, float) else v) for k, v in out.items() if v is not None}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--mixed", action="store_true", help="fp32 matrix values, fp64 accumulation")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-slq", action="store_true", help="skip the SLQ log-det + gradient leg")
    ap.add_argument("--only-slq", action="store_true", help="run the SLQ leg alone (no eigsh)")
    ap.add_argument("--only-rmat", action="store_true", help="run the configuration-4 (R-MAT) eigsh leg alone")
    ap.add_argument("--no-rmat", action="store_true", help="skip the configuration-4 (R-MAT) eigsh leg")
    ap.add_argument("--rmat-scale", type=int, default=RMAT_SCALE, help="R-MAT scale (reduced cases for profiling)")
    ap.add_argument("--no-reorder", dest="reorder", action="store_false",
                    help="keep the generator's row numbering inside the headline plan (default: Cuthill-McKee "
                         "renumbering inside the plan, LG_PLAN_REORDER_BFS, done at plan creation)")
    ap.add_argument("--no-adjoint", action="store_true", help="skip the differentiable-eigsh backward leg")
    ap.add_argument("--only-adjoint", action="store_true", help="run the differentiable-eigsh backward leg alone")
    ap.add_argument("--no-mixed", action="store_true", help="skip the configuration-1 mixed-precision leg")
    ap.add_argument("--only-sinv", action="store_true", help="run the configuration-2 (shift-invert) leg alone")
    ap.add_argument("--no-sinv", action="store_true", help="skip the configuration-2 (shift-invert) leg")
    ap.add_argument("--sinv-n", type=int, default=SINV_N, help="grid side of the shift-invert leg (reduced cases)")
    ap.add_argument("--only-graph", action="store_true", help="run the graph-construction leg alone")
    ap.add_argument("--no-graph", action="store_true", help="skip the graph-construction leg")
    ap.add_argument("--slq-n", type=int, default=N_POINTS, help="SLQ graph size (reduced cases for profiling)")
    ap.add_argument("--slq-m", type=int, default=SLQ_M, help="SLQ Lanczos depth (reduced cases for profiling)")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
