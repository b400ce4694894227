"""Drop-in for the reference's portable ``flash_gmm`` module (flash_gmm.py).

``flash_gmm_estep`` keeps the reference signature, assertions and return
convention (flash_gmm.py:173-217) and runs the isotropic E-step through
libflashgmm_sm100.so: tcgen05 tensor-core kernels on sm_100a, with fp32-level
accuracy (the reference's fp32 ``tl.dot`` runs as TF32 on a GPU).

    logZ, Nk, mu_acc, sig_acc = flash_gmm_estep(X, mu, log_sigma_sq, log_pi)

M-step (flash_gmm.py:34-37): pi = Nk / N, mu = mu_acc / Nk[:, None],
sigma^2 = sig_acc / (D * Nk).
"""

from __future__ import annotations

import torch

import _fgmm_lib


def flash_gmm_estep(
    X: torch.Tensor,              # (N, D) float32, GPU
    mu: torch.Tensor,             # (K, D) float32, GPU
    log_sigma_sq: torch.Tensor,   # (K,)   float32, GPU
    log_pi: torch.Tensor,         # (K,)   float32, GPU
    BLOCK_N: int = 64,
    BLOCK_K: int = 16,
    BLOCK_D: int = 128,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Isotropic GMM E-step: (logZ, Nk, mu_acc, sig_acc), fresh float32 tensors.

    ``BLOCK_N`` / ``BLOCK_K`` are accepted for compatibility; tile shapes are
    fixed per kernel.  ``BLOCK_D`` keeps its meaning as the D bound checked by
    the reference (flash_gmm.py:189).
    """
    _, D = X.shape
    assert D <= BLOCK_D, f"D={D} exceeds BLOCK_D={BLOCK_D}; increase BLOCK_D."
    assert X.is_cuda and mu.is_cuda, "Inputs must be on GPU."
    return _fgmm_lib.estep(_fgmm_lib.FGMM_VARIANT_ISO, X, mu, log_sigma_sq, log_pi)
