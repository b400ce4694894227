"""Drop-in for the reference's ``flash_gmm_diag_h100`` module.

``flash_gmm_estep_diag(X, mu, log_sigma_sq, log_pi) -> (logZ, Nk, mu_acc,
sig_acc)`` with log_sigma_sq of shape (K, D) and sig_acc (K, D) the centred
per-dimension second moment sum_n r_nk (x_nd - mu_kd)^2
(flash_gmm_diag_h100.py:305-384, 258-260).  Unlike the reference's split-K
pass 2 (diag:220-236), every row is counted exactly once for any N.
"""

from __future__ import annotations

import torch

import _fgmm_lib


def flash_gmm_estep_diag(
    X: torch.Tensor,
    mu: torch.Tensor,
    log_sigma_sq: torch.Tensor,
    log_pi: torch.Tensor,
):
    N, D = X.shape
    K = mu.shape[0]
    assert log_sigma_sq.shape == (K, D), \
        f"log_sigma_sq must be (K, D)=({K}, {D}), got {tuple(log_sigma_sq.shape)}"
    assert X.is_cuda and mu.is_cuda
    return _fgmm_lib.estep(_fgmm_lib.FGMM_VARIANT_DIAG, X, mu, log_sigma_sq, log_pi)
