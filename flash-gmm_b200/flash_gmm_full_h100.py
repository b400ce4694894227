"""Drop-in for the reference's ``flash_gmm_full_h100`` module.

``flash_gmm_estep_full(X, mu, prec_chol, log_pi) -> (logZ, Nk, mu_acc,
sig_outer)`` with prec_chol (K, D, D) the lower-triangular Cholesky factor of
each precision matrix (prec_chol[k] @ prec_chol[k].T = Sigma_k^-1) and
sig_outer (K, D, D) = sum_n r_nk x_n x_n^T, uncentred
(flash_gmm_full_h100.py:235-336).

M-step recovery (flash_gmm_full_h100.py:257-260):
    pi_k = Nk[k] / N;  mu_k = mu_acc[k] / Nk[k];
    Sigma_k = sig_outer[k] / Nk[k] - mu_k mu_k^T
"""

from __future__ import annotations

import torch

import _fgmm_lib


def flash_gmm_estep_full(
    X: torch.Tensor,
    mu: torch.Tensor,
    prec_chol: torch.Tensor,    # (K, D, D) -- lower-triangular Cholesky factor of Sigma^-1
    log_pi: torch.Tensor,        # (K,)
):
    """Flash-GMM E-step with full covariance; see the module docstring."""
    N, D = X.shape
    K = mu.shape[0]
    assert prec_chol.shape == (K, D, D), \
        f"prec_chol must be (K, D, D)=({K}, {D}, {D}), got {tuple(prec_chol.shape)}"
    assert X.is_cuda and mu.is_cuda
    return _fgmm_lib.estep(_fgmm_lib.FGMM_VARIANT_FULL, X, mu, prec_chol, log_pi)
