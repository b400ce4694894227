"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations the E-step is measured on.

The reference tunes on public datasets (Deep10M, SIFT1M, GloVe -- named in
flash_gmm_diag_h100.py:298-301) that are not available here; these seeded
mixtures stand in for them with the paper's shapes (K=1024, D=96-128).

    C1  isotropic  N=10,000     K=64    D=32   (the reference's CPU-runnable case)
    C2  isotropic  N=1,000,000  K=1024  D=128  (the headline configuration)
    C3  diagonal   N=1,000,000  K=1024  D=96
    C4  full       N=250,000    K=256   D=64
    C5  isotropic  N=100,000,000 K=1024 D=128, generated on the device by
        row-keyed counter RNG (see ``gmm_stream``), sharded across GPUs.

Every generator takes a torch.Generator seed and a device; the same seed and
device give the same tensors.
"""

from __future__ import annotations

import math

import torch

CONFIGS = {
    "c1": dict(kind="iso", N=10_000, K=64, D=32),
    "c2": dict(kind="iso", N=1_000_000, K=1024, D=128),
    "c3": dict(kind="diag", N=1_000_000, K=1024, D=96),
    "c4": dict(kind="full", N=250_000, K=256, D=64),
    "c5": dict(kind="iso", N=100_000_000, K=1024, D=128),
}


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def config_c1(device="cpu", seed: int = 0):
    """X ~ N(0,1) then mu ~ N(0,1) from the same generator, lss = 0,
    log_pi = -log 64 (the reference's own smoke-test recipe,
    flash_gmm.py:229-234, at the C1 shape)."""
    N, K, D = 10_000, 64, 32
    g = _gen(seed, device)
    X = torch.randn(N, D, generator=g, device=device)
    mu = torch.randn(K, D, generator=g, device=device)
    lss = torch.zeros(K, device=device)
    lpi = torch.full((K,), -math.log(K), device=device)
    return X, mu, lss, lpi


def iso_mixture(N: int, K: int, D: int, seed: int = 1234, device="cpu"):
    """C2 recipe: K true centres ~ N(0, 4I); each sample is a uniformly chosen
    centre plus N(0, I) noise; mu = K random rows of X; log_sigma_sq = 0;
    log_pi = -log K."""
    g = _gen(seed, device)
    centres = 2.0 * torch.randn(K, D, generator=g, device=device)
    lab = torch.randint(0, K, (N,), generator=g, device=device)
    X = centres[lab]
    X.add_(torch.randn(N, D, generator=g, device=device))
    idx = torch.randperm(N, generator=g, device=device)[:K]
    mu = X[idx].clone()
    lss = torch.zeros(K, device=device)
    lpi = torch.full((K,), -math.log(K), device=device)
    return X, mu, lss, lpi


def diag_mixture(N: int, K: int, D: int, seed: int = 2345, device="cpu"):
    """C3 recipe: K centres ~ N(0, 4I); per-dimension noise std
    exp(U(-1/2, 1/2)) drawn once per dimension; mu = random rows of X;
    log_sigma_sq ~ U(-1, 1) per (k, d); log_pi = log_softmax(N(0, 1))."""
    g = _gen(seed, device)
    centres = 2.0 * torch.randn(K, D, generator=g, device=device)
    std = torch.exp(torch.rand(D, generator=g, device=device) - 0.5)
    lab = torch.randint(0, K, (N,), generator=g, device=device)
    X = centres[lab]
    X.add_(torch.randn(N, D, generator=g, device=device) * std[None, :])
    idx = torch.randperm(N, generator=g, device=device)[:K]
    mu = X[idx].clone()
    lss = 2.0 * torch.rand(K, D, generator=g, device=device) - 1.0
    lpi = torch.log_softmax(torch.randn(K, generator=g, device=device), dim=0)
    return X, mu, lss, lpi


def full_mixture(N: int, K: int, D: int, seed: int = 3456, device="cpu"):
    """C4 recipe: K centres ~ N(0, 4I) with correlated noise z C,
    C = I + 0.1 tril(N(0,1), -1); prec_chol[k] lower-triangular with diagonal
    exp(U(-1/2, 1/2)) and off-diagonal N(0, 0.1^2); mu = random rows of X;
    log_pi = log_softmax(N(0, 1))."""
    g = _gen(seed, device)
    centres = 2.0 * torch.randn(K, D, generator=g, device=device)
    C = torch.eye(D, device=device) + 0.1 * torch.tril(
        torch.randn(D, D, generator=g, device=device), diagonal=-1)
    lab = torch.randint(0, K, (N,), generator=g, device=device)
    X = centres[lab]
    X.add_(torch.randn(N, D, generator=g, device=device) @ C)
    idx = torch.randperm(N, generator=g, device=device)[:K]
    mu = X[idx].clone()
    off = 0.1 * torch.tril(torch.randn(K, D, D, generator=g, device=device), diagonal=-1)
    diag = torch.exp(torch.rand(K, D, generator=g, device=device) - 0.5)
    L = off + torch.diag_embed(diag)
    lpi = torch.log_softmax(torch.randn(K, generator=g, device=device), dim=0)
    return X, mu, L, lpi


def make_config(name: str, device="cpu", N: int | None = None):
    """Inputs for a named configuration, optionally with fewer rows."""
    c = CONFIGS[name]
    n = c["N"] if N is None else N
    if name == "c1":
        return config_c1(device)
    if c["kind"] == "iso":
        return iso_mixture(n, c["K"], c["D"], device=device)
    if c["kind"] == "diag":
        return diag_mixture(n, c["K"], c["D"], device=device)
    return full_mixture(n, c["K"], c["D"], device=device)
