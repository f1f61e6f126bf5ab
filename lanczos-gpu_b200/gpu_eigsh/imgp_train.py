"""Marginal-likelihood training loops for the precision-parameterised graph
GP (the reference's python/gpu_eigsh/imgp_train.py), on this package's fused
operator and SLQ.

Three variants share the data, the initialisation and the optimiser (Adam on
lengthscale and graphbandwidth, both clamped to >= 1e-3 after each step) and
differ only in log det P:

  imgp_train_ours           fused stochastic Lanczos quadrature with the
                            Kraemer backward (gpu_eigsh.funm_torch.slq_logdet)
  imgp_train_dense          slogdet of the materialised n x n operator (small n)
  imgp_train_naive_lanczos  one unrolled three-term Lanczos per probe with
                            autograd through the iteration (the biased baseline
                            the reference documents)

Each returns a TrainResult with the per-iteration trajectory.  Loss = the
per-point negative log marginal likelihood 0.5 (y^T P y - log det P +
n log 2 pi) / n; a non-finite or exploding loss or gradient ends the run as
"diverged", as in the reference.
"""
from __future__ import annotations

import math
import time
from dataclasses import dataclass, field
from typing import Callable, Optional

import torch

from .funm_torch import slq_logdet
from .imgp import make_imgp_precision_matvec

__all__ = ["TrainResult", "imgp_train_ours", "imgp_train_dense", "imgp_train_naive_lanczos"]


@dataclass
class TrainResult:
    method: str
    final_loss: float
    final_lengthscale: float
    final_graphbandwidth: float
    iter_losses: list = field(default_factory=list)
    iter_lengthscales: list = field(default_factory=list)
    iter_graphbandwidths: list = field(default_factory=list)
    iter_wall_seconds: list = field(default_factory=list)
    peak_memory_bytes: int = 0
    diverged: bool = False
    diverged_at_iter: Optional[int] = None

    def summary_line(self) -> str:
        """One line: method, final loss and parameters, and whether training
        stopped early."""
        state = f"stopped at step {self.diverged_at_iter}" if self.diverged else "completed"
        return (f"{self.method}: final loss {self.final_loss:.4f}, lengthscale {self.final_lengthscale:.4f}, "
                f"graphbandwidth {self.final_graphbandwidth:.4f} ({state}, {len(self.iter_losses)} steps)")


def _inv_quad(matvec, y, lengthscale, graphbandwidth):
    """y^T P y, exact."""
    return torch.dot(y, matvec(y, lengthscale, graphbandwidth).to(y.dtype))


def _unrolled_lanczos_logdet(matvec, n, lengthscale, graphbandwidth, m_probes, lanczos_m, seed):
    """log det P by one three-term Lanczos (no re-orthogonalisation) per
    Rademacher probe, differentiated by autograd through the iteration; Ritz
    values clamped at 1e-30 before the log, as the reference does."""
    dtype, device = lengthscale.dtype, lengthscale.device
    gen = torch.Generator(device="cpu").manual_seed(seed)
    total = torch.zeros((), dtype=dtype, device=device)
    for _ in range(m_probes):
        z = (torch.randint(0, 2, (n,), generator=gen, dtype=dtype) * 2.0 - 1.0).to(device)
        znorm = torch.linalg.norm(z)
        v_prev = torch.zeros_like(z)
        v = z / znorm
        alphas, betas = [], []
        beta = torch.zeros((), dtype=dtype, device=device)
        for j in range(lanczos_m):
            w = matvec(v, lengthscale, graphbandwidth).to(dtype)
            a = torch.dot(v, w)
            w = w - a * v - beta * v_prev
            alphas.append(a)
            if j + 1 < lanczos_m:
                beta = torch.linalg.norm(w)
                betas.append(beta)
                v_prev, v = v, w / beta
        T = torch.diag(torch.stack(alphas))
        if betas:
            b = torch.stack(betas)
            T = T + torch.diag(b, 1) + torch.diag(b, -1)
        theta, S = torch.linalg.eigh(T)
        total = total + znorm * znorm * (S[0, :] ** 2 * torch.log(theta.clamp_min(1e-30))).sum()
    return total / m_probes


def _train(method: str, logdet_fn: Callable, matvec, y: torch.Tensor, lengthscale_init: float,
           graphbandwidth_init: float, n: int, max_iter: int, lr: float, verbose: bool,
           divergence_loss_threshold: float = 1e6) -> TrainResult:
    dtype, device = y.dtype, y.device
    theta = torch.tensor(lengthscale_init, dtype=dtype, device=device, requires_grad=True)
    kappa = torch.tensor(graphbandwidth_init, dtype=dtype, device=device, requires_grad=True)
    opt = torch.optim.Adam([theta, kappa], lr=lr)
    log_2pi = math.log(2.0 * math.pi)
    res = TrainResult(method=method, final_loss=float("nan"), final_lengthscale=lengthscale_init,
                      final_graphbandwidth=graphbandwidth_init)
    if device.type == "cuda":
        torch.cuda.reset_peak_memory_stats(device)
    t0 = time.perf_counter()
    for it in range(max_iter):
        opt.zero_grad()
        try:
            loss = 0.5 * (_inv_quad(matvec, y, theta, kappa) - logdet_fn(theta, kappa) + n * log_2pi) / n
        except RuntimeError as e:
            res.diverged, res.diverged_at_iter = True, it
            if verbose:
                print(f"  {method}: step {it}: the loss could not be evaluated ({e}); stopping")
            break
        lv = float(loss.detach())
        if not math.isfinite(lv) or abs(lv) > divergence_loss_threshold:
            res.diverged, res.diverged_at_iter = True, it
            if verbose:
                print(f"  {method}: step {it}: loss {lv} is non-finite or beyond the divergence bound; stopping")
            break
        loss.backward()
        if not all(bool(torch.isfinite(p.grad).all()) for p in (theta, kappa) if p.grad is not None):
            res.diverged, res.diverged_at_iter = True, it
            if verbose:
                print(f"  {method}: step {it}: a gradient is non-finite; stopping")
            break
        opt.step()
        with torch.no_grad():
            theta.clamp_(min=1e-3)
            kappa.clamp_(min=1e-3)
        res.iter_losses.append(lv)
        res.iter_lengthscales.append(float(theta.detach()))
        res.iter_graphbandwidths.append(float(kappa.detach()))
        res.iter_wall_seconds.append(time.perf_counter() - t0)
        if verbose and (it % 5 == 0 or it == max_iter - 1):
            print(f"  [{method}] it {it:>3d}  loss={lv:>8.3f}  theta={float(theta):>6.3f}  kappa={float(kappa):>6.3f}")
    if not res.diverged and res.iter_losses:
        res.final_loss = res.iter_losses[-1]
        res.final_lengthscale = res.iter_lengthscales[-1]
        res.final_graphbandwidth = res.iter_graphbandwidths[-1]
    if device.type == "cuda":
        res.peak_memory_bytes = int(torch.cuda.max_memory_allocated(device))
    return res


def imgp_train_ours(*, train_targets, x_edge_dists, idx, n, nu=2, lengthscale_init=1.0, graphbandwidth_init=1.0,
                    max_iter=50, lr=0.05, m_probes=50, lanczos_m=20, seed=0, verbose=False) -> TrainResult:
    """Adam on the marginal likelihood with the fused SLQ log-det."""
    matvec = make_imgp_precision_matvec(x_edge_dists=x_edge_dists, idx=idx, operator_dim=n, nu=nu)

    def logdet_fn(theta, kappa):
        return slq_logdet(matvec, n, (theta, kappa), m_probes=m_probes, lanczos_m=lanczos_m, seed=seed,
                          dtype=theta.dtype, device=theta.device)

    return _train("imgp-ours", logdet_fn, matvec, train_targets, lengthscale_init, graphbandwidth_init, n, max_iter,
                  lr, verbose)


def imgp_train_dense(*, train_targets, x_edge_dists, idx, n, nu=2, lengthscale_init=1.0, graphbandwidth_init=1.0,
                     max_iter=50, lr=0.05, verbose=False) -> TrainResult:
    """Adam with slogdet of the materialised operator (n columns of P; small n)."""
    matvec = make_imgp_precision_matvec(x_edge_dists=x_edge_dists, idx=idx, operator_dim=n, nu=nu)

    def logdet_fn(theta, kappa):
        I = torch.eye(n, dtype=theta.dtype, device=theta.device)
        P = matvec(I, theta, kappa).to(theta.dtype)   # P I = P, one block product
        return torch.linalg.slogdet(P)[1]

    return _train("imgp-full", logdet_fn, matvec, train_targets, lengthscale_init, graphbandwidth_init, n, max_iter,
                  lr, verbose)


def imgp_train_naive_lanczos(*, train_targets, x_edge_dists, idx, n, nu=2, lengthscale_init=1.0,
                             graphbandwidth_init=1.0, max_iter=50, lr=0.05, m_probes=10, lanczos_m=30, seed=0,
                             verbose=False) -> TrainResult:
    """Adam with the unrolled-autograd Lanczos log-det (the biased baseline)."""
    matvec = make_imgp_precision_matvec(x_edge_dists=x_edge_dists, idx=idx, operator_dim=n, nu=nu)

    def logdet_fn(theta, kappa):
        return _unrolled_lanczos_logdet(matvec, n, theta, kappa, m_probes, lanczos_m, seed)

    return _train("imgp-naive", logdet_fn, matvec, train_targets, lengthscale_init, graphbandwidth_init, n, max_iter,
                  lr, verbose)
