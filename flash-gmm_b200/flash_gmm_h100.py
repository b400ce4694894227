"""Drop-in for the reference's ``flash_gmm_h100`` module (flash_gmm_h100.py).

Same entry point and return convention as flash_gmm_h100.py:254-328
(``flash_gmm_estep(X, mu, log_sigma_sq, log_pi) -> (logZ, Nk, mu_acc,
sig_acc)``, logZ in natural-log units).  The reference trades accuracy for
speed here (bf16 X and mu, ~5e-3); on B200 the same tcgen05 kernels as
``flash_gmm`` run with fp32-level accuracy, so both modules return the same
results.
"""

from __future__ import annotations

import torch

import _fgmm_lib


def flash_gmm_estep(
    X: torch.Tensor,
    mu: torch.Tensor,
    log_sigma_sq: torch.Tensor,
    log_pi: torch.Tensor,
):
    """Compute the GMM E-step sufficient statistics on GPU.

    Returns (logZ, Nk, mu_acc, sig_acc).
    """
    assert X.is_cuda and mu.is_cuda
    return _fgmm_lib.estep(_fgmm_lib.FGMM_VARIANT_ISO, X, mu, log_sigma_sq, log_pi)
