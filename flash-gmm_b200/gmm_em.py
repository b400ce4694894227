"""EM fitting on top of the B200 E-step: the caller the reference documents
in its README (README.md:41-61 and 81-103) and its full-covariance docstring
(flash_gmm_full_h100.py:257-260), as a library function.

    params = fit(X, K=1024, covariance_type="iso", n_iter=50)

One iteration = one E-step through the C ABI (or a sharded / streamed
E-step) + the M-step below on the O(K D) statistics, on the device, with no
host synchronisation except the convergence test on sum(logZ).

M-step (`m_step`), from the E-step statistics computed at the current means
mu_old:
  pi_k  = Nk_k / N
  mu_k  = mu_acc_k / Nk_k
  iso:  sigma_k^2 = (sig_k - Nk_k |mu_k - mu_old_k|^2) / (D Nk_k)
  diag: sigma_kd^2 = (sig_kd - Nk_k (mu_kd - mu_old_kd)^2) / Nk_k
  full: Sigma_k = sig_outer_k / Nk_k - mu_k mu_k^T  (flash_gmm_full_h100.py:259),
        prec_chol_k = cholesky(Sigma_k^-1)  (lower, prec_chol prec_chol^T = Sigma^-1)
The iso/diag variance subtracts the shift of the mean: sig is centred on
mu_old, and sum_n r (x - mu)^2 = sig - Nk (mu - mu_old)^2 exactly, which keeps
EM's log-likelihood monotone.  variance="readme" uses sig / (D Nk) as written
in the reference's README (the old-mean shortcut).  reg_covar is added to
every variance (diagonal of Sigma) and components with Nk below
min_count keep their previous parameters.
"""

from __future__ import annotations

import math
from typing import Callable, Iterable, Optional

import torch

import _fgmm_lib as L
import gmm_stream as GS

_VARIANT = {"iso": L.FGMM_VARIANT_ISO, "diag": L.FGMM_VARIANT_DIAG, "full": L.FGMM_VARIANT_FULL}


def init_params(X: torch.Tensor, K: int, covariance_type: str = "iso", seed: int = 0):
    """Means = K distinct rows of X (the benchmark recipe), unit variances,
    uniform weights.  Returns (mu, cov, log_pi) in the E-step's input form."""
    N, D = X.shape
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    idx = torch.randperm(N, generator=g)[:K].to(X.device)
    mu = X[idx].float().clone()
    dev = X.device
    if covariance_type == "iso":
        cov = torch.zeros(K, device=dev)
    elif covariance_type == "diag":
        cov = torch.zeros(K, D, device=dev)
    elif covariance_type == "full":
        cov = torch.eye(D, device=dev).expand(K, D, D).contiguous()
    else:
        raise ValueError(f"unknown covariance_type {covariance_type!r}")
    log_pi = torch.full((K,), -math.log(K), device=dev)
    return mu, cov, log_pi


def m_step(covariance_type: str, N: int, Nk: torch.Tensor, mu_acc: torch.Tensor,
           sig: torch.Tensor, mu_old: torch.Tensor, cov_old: torch.Tensor,
           reg_covar: float = 1e-6, min_count: float = 1e-3, variance: str = "exact"):
    """New (mu, cov, log_pi) from one E-step's statistics (module docstring)."""
    if variance not in ("exact", "readme"):
        raise ValueError("variance must be 'exact' or 'readme'")
    K, D = mu_acc.shape
    alive = Nk > min_count
    nk = torch.where(alive, Nk, torch.ones_like(Nk)).double()
    mu = mu_acc.double() / nk[:, None]
    shift2 = (mu - mu_old.double()) ** 2 if variance == "exact" else torch.zeros_like(mu)
    if covariance_type == "iso":
        var = (sig.double() - nk * shift2.sum(1)) / (D * nk)
        cov = torch.log(var.clamp_min(0.0) + reg_covar).float()
    elif covariance_type == "diag":
        var = (sig.double() - nk[:, None] * shift2) / nk[:, None]
        cov = torch.log(var.clamp_min(0.0) + reg_covar).float()
    elif covariance_type == "full":
        Sigma = sig.double() / nk[:, None, None] - mu[:, :, None] * mu[:, None, :]
        Sigma = 0.5 * (Sigma + Sigma.transpose(1, 2))
        Sigma = Sigma + reg_covar * torch.eye(D, device=Sigma.device, dtype=Sigma.dtype)
        cov = torch.linalg.cholesky(torch.linalg.inv(Sigma)).float()
    else:
        raise ValueError(f"unknown covariance_type {covariance_type!r}")
    mu = mu.float()
    keep = ~alive
    mu = torch.where(keep[:, None], mu_old.float(), mu)
    if covariance_type == "full":
        cov = torch.where(keep[:, None, None], cov_old.float(), cov)
    elif covariance_type == "diag":
        cov = torch.where(keep[:, None], cov_old.float(), cov)
    else:
        cov = torch.where(keep, cov_old.float(), cov)
    log_pi = torch.log(Nk.double().clamp_min(1e-30) / N).float()
    log_pi = log_pi - torch.logsumexp(log_pi, 0)
    return mu, cov, log_pi


def _library_estep(covariance_type: str):
    variant = _VARIANT[covariance_type]

    def run(X, mu, cov, log_pi):
        logZ, Nk, mu_acc, sig = L.estep(variant, X, mu, cov, log_pi)
        return logZ.sum(), Nk, mu_acc, sig
    return run


def fit(X, K: Optional[int] = None, covariance_type: str = "iso", n_iter: int = 100,
        tol: float = 1e-5, init=None, seed: int = 0, reg_covar: float = 1e-6,
        variance: str = "exact", estep_fn: Optional[Callable] = None,
        n_rows: Optional[int] = None):
    """EM iterations until the mean log-likelihood changes by less than tol.

    X: (N, D) float32 CUDA tensor (or anything estep_fn accepts).
    init: optional (mu, cov, log_pi); else `init_params(X, K)`.
    estep_fn(X, mu, cov, log_pi) -> (sum logZ, Nk, mu_acc, sig): defaults to
      the library E-step; pass a sharded or streamed E-step for multi-GPU
      (`sharded_estep`) or host-resident data (`streamed_estep`).
    n_rows: total rows N when X is not a tensor (streaming).
    Returns dict(mu, cov, log_pi, log_likelihood=[mean logZ per iteration],
                 n_iter, converged).
    """
    if covariance_type not in _VARIANT:
        raise ValueError(f"unknown covariance_type {covariance_type!r}")
    if init is None:
        if K is None:
            raise ValueError("fit needs K or init")
        mu, cov, log_pi = init_params(X, K, covariance_type, seed)
    else:
        mu, cov, log_pi = (t.float() for t in init)
    N = n_rows if n_rows is not None else X.shape[0]
    step = estep_fn or _library_estep(covariance_type)
    history = []
    converged = False
    it = 0
    for it in range(1, n_iter + 1):
        sum_logZ, Nk, mu_acc, sig = step(X, mu, cov, log_pi)
        ll = float(sum_logZ) / N  # the one host synchronisation per iteration
        history.append(ll)
        mu, cov, log_pi = m_step(covariance_type, N, Nk, mu_acc, sig, mu, cov,
                                 reg_covar=reg_covar, variance=variance)
        if len(history) >= 2 and abs(history[-1] - history[-2]) < tol * max(1.0, abs(ll)):
            converged = True
            break
    return {"mu": mu, "cov": cov, "log_pi": log_pi, "log_likelihood": history,
            "n_iter": it, "converged": converged}


def sharded_estep(covariance_type: str, group=None, local_estep: Optional[Callable] = None):
    """E-step over the rows each rank holds (torch.distributed, NCCL): the
    statistics and sum(logZ) are summed over ranks (gmm_stream.ShardedEStep
    plus one scalar all-reduce).  local_estep(X, mu, cov, log_pi, out) is
    the per-rank E-step (default: the library)."""
    import torch.distributed as dist
    sharded = GS.ShardedEStep(covariance_type, group=group, estep_fn=local_estep)

    def run(X_local, mu, cov, log_pi):
        logZ, Nk, mu_acc, sig = sharded(X_local, mu, cov, log_pi)
        s = logZ.sum().reshape(1)
        if dist.is_available() and dist.is_initialized():
            dist.all_reduce(s, group=group)
        return s[0], Nk, mu_acc, sig
    return run


def streamed_estep(covariance_type: str, device=None):
    """E-step over host chunks (an iterable factory: X is a callable returning
    a fresh iterable of (n_i, D) pinned CPU tensors each iteration), using the
    double-buffered copy stream of gmm_stream.stream_estep."""
    def run(chunks: Callable[[], Iterable[torch.Tensor]], mu, cov, log_pi):
        logZ, Nk, mu_acc, sig = GS.stream_estep(chunks(), mu, cov, log_pi,
                                                variant=covariance_type, device=device,
                                                keep_logZ=True)
        return logZ.sum(), Nk, mu_acc, sig
    return run
