"""CPU oracle for the Gaussian-mixture E-step -- TEST INFRASTRUCTURE ONLY.

This module restates, in plain numpy (float64 by default), the arithmetic of
the four reference Flash-GMM entry points.  It is the checker the parity tests,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg compare the
CUDA path against.  Nothing in the product package imports it; the product path
fails loudly when its CUDA library is missing instead of falling back here.

Pinning: the isotropic fp32 restatement is pinned against golden vectors that
``tests/golden/make_golden.py`` produced by running the reference's own Triton
kernels (flash_gmm.py:50-103, 110-166) under ``TRITON_INTERPRET=1``; the
diagonal and full-covariance restatements are pinned against fp32-substituted
runs of the reference kernels (flash_gmm_diag_h100.py:63-130, 159-282 and
flash_gmm_full_h100.py:71-139, 146-228) made by the same script.  The
reference ships no golden vectors or tests of its own.

All functions return ``(logZ, Nk, mu_acc, sig)`` with the reference's shapes
and natural-log ``logZ`` (flash_gmm_h100.py:326, diag:382, full:335).
"""

from __future__ import annotations

import math

import numpy as np

LOG_2PI = math.log(2.0 * math.pi)   # flash_gmm.py:91 (1.8378770664093453)
LOG2_E = 1.0 / math.log(2.0)        # flash_gmm_h100.py:251


def _lse_rows(ll: np.ndarray) -> np.ndarray:
    """Row-wise log-sum-exp with the max shift (flash_gmm.py:95-102)."""
    m = np.max(ll, axis=1)
    m_safe = np.where(np.isfinite(m), m, 0.0)
    s = np.sum(np.exp(ll - m_safe[:, None]), axis=1)
    with np.errstate(divide="ignore"):
        return m_safe + np.log(s)


def _responsibilities(ll: np.ndarray):
    logZ = _lse_rows(ll)
    r = np.exp(ll - logZ[:, None])           # flash_gmm.py:151
    r = np.where(np.isfinite(ll), r, 0.0)   # flash_gmm.py:152 masks to 0
    return logZ, r


def loglik_iso(X, mu, log_sigma_sq, log_pi):
    """ll[n,k] and sq[n,k] of the isotropic model (flash_gmm.py:84-93).

    ll = log_pi_k - 0.5*||x_n - mu_k||^2 * exp(-lss_k) - 0.5*D*(log 2pi + lss_k).
    ``sq`` is formed as x_sq - 2 x.mu + mu_sq exactly as the reference
    expands it (flash_gmm.py:85-88); in float64 the expansion is exact enough.
    """
    X = np.asarray(X, dtype=np.float64)
    mu = np.asarray(mu, dtype=np.float64)
    lss = np.asarray(log_sigma_sq, dtype=np.float64)
    lpi = np.asarray(log_pi, dtype=np.float64)
    D = X.shape[1]
    x_sq = np.sum(X * X, axis=1)
    mu_sq = np.sum(mu * mu, axis=1)
    sq = x_sq[:, None] - 2.0 * (X @ mu.T) + mu_sq[None, :]
    ll = lpi[None, :] - 0.5 * sq * np.exp(-lss)[None, :] \
        - 0.5 * D * (LOG_2PI + lss[None, :])
    return ll, sq


def estep_iso(X, mu, log_sigma_sq, log_pi, chunk: int = 65536):
    """Isotropic E-step (flash_gmm.py:173-217; same maths as
    flash_gmm_h100.py:254-328, whose log2-space folding at 286-291 and
    137-138 is an algebraic rewrite of the same ll).

    Returns logZ (N,), Nk (K,), mu_acc (K,D) = R^T X (flash_gmm.py:161),
    sig_acc (K,) = sum_n r_nk ||x_n - mu_k||^2 (flash_gmm.py:156).
    """
    X = np.asarray(X, dtype=np.float64)
    N, D = X.shape
    K = np.asarray(mu).shape[0]
    logZ = np.empty(N)
    Nk = np.zeros(K)
    mu_acc = np.zeros((K, D))
    sig = np.zeros(K)
    for s in range(0, N, chunk):
        xs = X[s:s + chunk]
        ll, sq = loglik_iso(xs, mu, log_sigma_sq, log_pi)
        lz, r = _responsibilities(ll)
        logZ[s:s + chunk] = lz
        Nk += r.sum(axis=0)
        mu_acc += r.T @ xs
        sig += (r * sq).sum(axis=0)
    return logZ, Nk, mu_acc, sig


def loglik_diag(X, mu, log_sigma_sq, log_pi):
    """ll[n,k] of the diagonal model, restating flash_gmm_diag_h100.py:332-339
    (c0 with the log-det and mu^2/sigma^2 terms) and 116-119
    (ll2 = c0 - x^2 . inv^T + 2 x . (mu*inv)^T), converted back to natural-log
    units: ll = log_pi - 0.5*(D log 2pi + sum_d lss) - 0.5 sum_d (x-mu)^2 e^-lss.
    """
    X = np.asarray(X, dtype=np.float64)
    mu = np.asarray(mu, dtype=np.float64)
    lss = np.asarray(log_sigma_sq, dtype=np.float64)
    lpi = np.asarray(log_pi, dtype=np.float64)
    D = X.shape[1]
    inv = np.exp(-lss)                                          # (K, D)
    quad = (X * X) @ inv.T - 2.0 * X @ (mu * inv).T \
        + np.sum(mu * mu * inv, axis=1)[None, :]
    ll = (lpi - 0.5 * (D * LOG_2PI + lss.sum(axis=1)))[None, :] - 0.5 * quad
    return ll


def estep_diag(X, mu, log_sigma_sq, log_pi, chunk: int = 65536):
    """Diagonal-covariance E-step (flash_gmm_diag_h100.py:305-384).

    sig_acc (K,D) is the centred, unweighted per-dimension second moment
    sum_n r_nk (x_nd - mu_kd)^2, which the reference rebuilds from raw moments
    at diag:258-260.  The reference's pass-2 slab-overlap defect
    (diag:220-236 over-counts rows when ceil(N/N_SPLIT) % BLOCK_N != 0) is NOT
    reproduced: this is the intended maths.
    """
    X = np.asarray(X, dtype=np.float64)
    mu = np.asarray(mu, dtype=np.float64)
    N, D = X.shape
    K = mu.shape[0]
    logZ = np.empty(N)
    Nk = np.zeros(K)
    mu_acc = np.zeros((K, D))
    rx2 = np.zeros((K, D))
    for s in range(0, N, chunk):
        xs = X[s:s + chunk]
        ll = loglik_diag(xs, mu, log_sigma_sq, log_pi)
        lz, r = _responsibilities(ll)
        logZ[s:s + chunk] = lz
        Nk += r.sum(axis=0)
        mu_acc += r.T @ xs
        rx2 += r.T @ (xs * xs)
    sig = rx2 - 2.0 * mu * mu_acc + mu * mu * Nk[:, None]
    return logZ, Nk, mu_acc, sig


def loglik_full(X, mu, prec_chol, log_pi):
    """ll[n,k] of the full-covariance model (flash_gmm_full_h100.py:288-296,
    124-129): maha = ||L_k^T (x - mu_k)||^2 with prec_chol[k] = L_k,
    ll = log_pi + sum_d log(|L_kdd| + 1e-30) - 0.5 D log 2pi - 0.5 maha.
    """
    X = np.asarray(X, dtype=np.float64)
    mu = np.asarray(mu, dtype=np.float64)
    L = np.asarray(prec_chol, dtype=np.float64)
    lpi = np.asarray(log_pi, dtype=np.float64)
    D = X.shape[1]
    K = mu.shape[0]
    log_diag = np.log(np.abs(np.diagonal(L, axis1=1, axis2=2)) + 1e-30).sum(axis=1)
    c = lpi + log_diag - 0.5 * D * LOG_2PI
    ll = np.empty((X.shape[0], K))
    for k in range(K):
        v = (X - mu[k][None, :]) @ L[k]       # rows of (L_k^T (x - mu_k))^T
        ll[:, k] = c[k] - 0.5 * np.sum(v * v, axis=1)
    return ll


def estep_full(X, mu, prec_chol, log_pi, chunk: int = 16384):
    """Full-covariance E-step (flash_gmm_full_h100.py:235-336).

    sig_outer (K,D,D) = sum_n r_nk x_n x_n^T, the UNcentred second moment the
    reference accumulates at full:213-228 (M-step recovery at full:257-260).
    """
    X = np.asarray(X, dtype=np.float64)
    N, D = X.shape
    K = np.asarray(mu).shape[0]
    logZ = np.empty(N)
    Nk = np.zeros(K)
    mu_acc = np.zeros((K, D))
    sig = np.zeros((K, D, D))
    for s in range(0, N, chunk):
        xs = X[s:s + chunk]
        ll = loglik_full(xs, mu, prec_chol, log_pi)
        lz, r = _responsibilities(ll)
        logZ[s:s + chunk] = lz
        Nk += r.sum(axis=0)
        mu_acc += r.T @ xs
        # sum_n r_nk x_ni x_nj as one (K x n) @ (n x D^2) product
        xx = (xs[:, :, None] * xs[:, None, :]).reshape(len(xs), D * D)
        sig += (r.T @ xx).reshape(K, D, D)
    return logZ, Nk, mu_acc, sig


# ---------------------------------------------------------------------------
# Timed CPU baseline: the same isotropic formulas, dense fp32 on torch-CPU,
# chunked over N (multithreaded over the host cores).  Used only by bench.py's
# cpu_baseline / --impl reference legs.
# ---------------------------------------------------------------------------

def estep_iso_cpu_fp32(X, mu, log_sigma_sq, log_pi, chunk: int = 65536):
    """fp32 torch-CPU restatement of flash_gmm.py:84-101 and 151-166.

    ll = c_k + x . (mu_k e^{-lss_k}) - 0.5 |x|^2 e^{-lss_k} with
    c_k = log pi_k - D/2 (log 2pi + lss_k) - 0.5 |mu_k|^2 e^{-lss_k} (the
    expanded distance of flash_gmm.py:84-93, one matmul and one in-place
    update per chunk), and sig_k = sum_n r_nk |x_n - mu_k|^2 from the raw
    moments sum r |x|^2 - 2 mu_k . mu_acc_k + Nk |mu_k|^2, so no N x K
    matrix other than ll/r is formed."""
    import torch
    N, D = X.shape
    K = mu.shape[0]
    mu = mu.float()
    lss = log_sigma_sq.float()
    inv_s = torch.exp(-lss)
    mu_sq = (mu * mu).sum(1)
    c = log_pi.float() - 0.5 * D * (LOG_2PI + lss) - 0.5 * mu_sq * inv_s
    w = mu * inv_s[:, None]
    logZ = torch.empty(N)
    Nk = torch.zeros(K)
    mu_acc = torch.zeros(K, D)
    rxsq = torch.zeros(K)
    for s in range(0, N, chunk):
        xs = X[s:s + chunk].float()
        x_sq = (xs * xs).sum(1)
        ll = torch.addmm(c[None, :], xs, w.T)
        ll.addcmul_(x_sq[:, None], inv_s[None, :], value=-0.5)
        lz = torch.logsumexp(ll, dim=1)
        r = ll.sub_(lz[:, None]).exp_()          # in place: ll is not needed again
        logZ[s:s + chunk] = lz
        Nk += r.sum(0)
        mu_acc += r.T @ xs
        rxsq += r.T @ x_sq
    sig = rxsq - 2.0 * (mu_acc * mu).sum(1) + Nk * mu_sq
    return logZ, Nk, mu_acc, sig


def estep_diag_cpu_fp32(X, mu, log_sigma_sq, log_pi, chunk: int = 65536):
    """fp32 torch-CPU restatement of flash_gmm_diag_h100.py:332-339, 116-119
    (ll2 = c0 - x^2 . inv^T + 2 x . (mu*inv)^T) and 258-260 (sig from raw
    moments)."""
    import torch
    N, D = X.shape
    K = mu.shape[0]
    mu = mu.float()
    lss = log_sigma_sq.float()
    inv = torch.exp(-lss)
    const = log_pi.float() - 0.5 * (D * LOG_2PI + lss.sum(1)) - 0.5 * (mu * mu * inv).sum(1)
    w = mu * inv
    logZ = torch.empty(N)
    Nk = torch.zeros(K)
    mu_acc = torch.zeros(K, D)
    rx2 = torch.zeros(K, D)
    for s in range(0, N, chunk):
        xs = X[s:s + chunk].float()
        x2 = xs * xs
        ll = torch.addmm(const[None, :], xs, w.T)
        ll.addmm_(x2, inv.T, alpha=-0.5)
        lz = torch.logsumexp(ll, dim=1)
        r = ll.sub_(lz[:, None]).exp_()          # in place: ll is not needed again
        logZ[s:s + chunk] = lz
        Nk += r.sum(0)
        mu_acc += r.T @ xs
        rx2 += r.T @ x2
    sig = rx2 - 2.0 * mu * mu_acc + mu * mu * Nk[:, None]
    return logZ, Nk, mu_acc, sig


def estep_full_cpu_fp32(X, mu, prec_chol, log_pi, chunk: int = 16384):
    """fp32 torch-CPU restatement of flash_gmm_full_h100.py:288-296, 124-129
    (maha = ||L_k^T (x - mu_k)||^2) and 213-228 (sig_outer = sum r x x^T)."""
    import torch
    N, D = X.shape
    K = mu.shape[0]
    mu = mu.float()
    L = prec_chol.float()
    log_diag = torch.log(torch.diagonal(L, dim1=1, dim2=2).abs() + 1e-30).sum(1)
    c = log_pi.float() + log_diag - 0.5 * D * LOG_2PI
    b = torch.einsum("kd,kde->ke", mu, L)          # (L_k^T mu_k)^T
    logZ = torch.empty(N)
    Nk = torch.zeros(K)
    mu_acc = torch.zeros(K, D)
    sig = torch.zeros(K, D, D)
    for s in range(0, N, chunk):
        xs = X[s:s + chunk].float()
        v = torch.einsum("nd,kde->nke", xs, L) - b[None]   # (n, K, D)
        ll = c[None, :] - 0.5 * (v * v).sum(2)
        lz = torch.logsumexp(ll, dim=1)
        r = ll.sub_(lz[:, None]).exp_()
        logZ[s:s + chunk] = lz
        Nk += r.sum(0)
        mu_acc += r.T @ xs
        # sum_n r_nk x_ni x_nj as one (K x n) @ (n x D^2) product (the
        # three-operand einsum ran ~14x slower on the host BLAS)
        sig += (r.T @ (xs[:, :, None] * xs[:, None, :]).reshape(len(xs), D * D)).view(K, D, D)
    return logZ, Nk, mu_acc, sig
