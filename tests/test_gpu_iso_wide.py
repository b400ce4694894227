"""Isotropic tensor-core path for 128 < D <= 256 (64-row tiles, W_hi in
TMEM, W_lo in shared memory) against the fp64 oracle and the general
CUDA-core kernels.

Tolerances: logZ elementwise rel 1e-5, statistics normwise rel 1e-4
(tests/parity.py)."""

import math

import numpy as np
import pytest
import torch

import _fgmm_lib as L
import flash_gmm_h100
import gmm_data
from oracle import gmm_oracle as O
from parity import assert_parity

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _np(out):
    torch.cuda.synchronize()
    return tuple(t.detach().cpu().numpy() for t in out)


def _case(N, K, D, seed, offset=0.0):
    """C2 recipe (gmm_data) with means moved off the data rows, varied
    variances and weights, shifted by ``offset``."""
    X, mu, _, _ = gmm_data.iso_mixture(N, K, D, seed=seed)
    g = torch.Generator().manual_seed(seed + 1)
    X = X + offset
    mu = mu[:K] + offset + 0.3 * torch.randn(min(K, mu.shape[0]), D, generator=g)
    if mu.shape[0] < K:
        mu = torch.cat([mu, X[:K - mu.shape[0]] + 0.3])
    lss = 0.4 * torch.rand(K, generator=g) - 0.2
    lpi = torch.log_softmax(torch.randn(K, generator=g), 0)
    return X, mu, lss, lpi


SHAPES = [(1, 1, 129), (257, 3, 144), (5000, 100, 160), (6000, 300, 200), (4000, 1024, 256),
          (3000, 700, 250)]


@pytest.mark.parametrize("N,K,D", SHAPES)
def test_wide_iso_vs_oracle_and_general(N, K, D):
    X, mu, lss, lpi = _case(N, K, D, seed=N + K + D)
    ref = O.estep_iso(X.numpy(), mu.numpy(), lss.numpy(), lpi.numpy())
    Xd, mud, lssd, lpid = (t.to(DEV) for t in (X, mu, lss, lpi))
    tc = _np(flash_gmm_h100.flash_gmm_estep(Xd, mud, lssd, lpid))
    gen = _np(L.estep(L.FGMM_VARIANT_ISO, Xd, mud, lssd, lpid, force_general=True))
    assert_parity(tc, ref, what=f"wide iso {N}x{K}x{D} vs oracle")
    assert_parity(tc, gen, what=f"wide iso {N}x{K}x{D} vs general")


def test_wide_iso_offset_strided_neg_inf_and_accumulate():
    """Features near +40, X column-major, mu with a row stride, two -inf
    log-weights, and a second call adding into the first's statistics."""
    N, K, D = 6000, 200, 192
    X, mu, lss, lpi = _case(N, K, D, seed=3, offset=40.0)
    lpi[[7, 150]] = -math.inf
    ref = O.estep_iso(X.numpy(), mu.numpy(), lss.numpy(), lpi.numpy())
    Xt = X.t().contiguous().to(DEV).t()
    mu_big = torch.zeros(K, 2 * D)
    mu_big[:, :D] = mu
    mud = mu_big.to(DEV)[:, :D]
    lssd, lpid = lss.to(DEV), lpi.to(DEV)
    out = _np(L.estep(L.FGMM_VARIANT_ISO, Xt, mud, lssd, lpid))
    assert_parity(out, ref, what="wide iso offset, strided, -inf weights")
    assert out[1][7] == 0.0 and out[1][150] == 0.0
    first = L.estep(L.FGMM_VARIANT_ISO, Xt[:2500], mud, lssd, lpid)
    second = (torch.empty(N - 2500, device=DEV),) + tuple(t.clone() for t in first[1:])
    L.estep(L.FGMM_VARIANT_ISO, Xt[2500:], mud, lssd, lpid, out=second, accumulate=True)
    acc = (np.concatenate([_np(first)[0], _np(second)[0]]),) + _np(second)[1:]
    assert_parity(acc, ref, what="wide iso accumulated over two calls")


def test_wide_iso_more_than_1024_components_and_repeat():
    N, K, D = 3000, 1500, 136
    X, mu, lss, lpi = _case(N, K, D, seed=11)
    ref = O.estep_iso(X.numpy(), mu.numpy(), lss.numpy(), lpi.numpy())
    args = tuple(t.to(DEV) for t in (X, mu, lss, lpi))
    tc = _np(L.estep(L.FGMM_VARIANT_ISO, *args))
    assert_parity(tc, ref, what=f"wide iso K={K}")
    again = _np(L.estep(L.FGMM_VARIANT_ISO, *args))
    for a, b in zip(tc, again):
        np.testing.assert_array_equal(a, b)


def test_wide_iso_many_tiles_invariants():
    """N = 400K rows (chunked call, every stage buffer reused many times):
    sum_k Nk = N, sum_k mu_acc = sum_n x_n, and agreement with the general
    kernels."""
    X, mu, lss, lpi = gmm_data.iso_mixture(400_000, 1024, 256, seed=5, device=DEV)
    tc = _np(L.estep(L.FGMM_VARIANT_ISO, X, mu, lss, lpi))
    gen = _np(L.estep(L.FGMM_VARIANT_ISO, X, mu, lss, lpi, force_general=True))
    assert abs(tc[1].astype(np.float64).sum() - X.shape[0]) <= 1e-5 * X.shape[0]
    xs = X.double().sum(0).cpu().numpy()
    np.testing.assert_allclose(tc[2].astype(np.float64).sum(0), xs,
                               atol=1e-4 * np.abs(tc[2]).max() * 4)
    assert_parity(tc, gen, what="wide iso N=400K vs general")
