"""Diagonal-covariance tensor-core path (features [(x-c)^2, (x-c)]) against
the fp64 oracle and the general CUDA-core kernels.

Tolerances: logZ elementwise rel 1e-5, statistics normwise rel 1e-4
(tests/parity.py)."""

import math

import numpy as np
import pytest
import torch

import _fgmm_lib as L
import flash_gmm_diag_h100
import gmm_data
from oracle import gmm_oracle as O
from parity import assert_parity

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _np(out):
    torch.cuda.synchronize()
    return tuple(t.detach().cpu().numpy() for t in out)


def _case(N, K, D, seed, offset=0.0, spread=2.0):
    g = torch.Generator().manual_seed(seed)
    centres = spread * torch.randn(K, D, generator=g) + offset
    lab = torch.randint(0, K, (N,), generator=g)
    std = torch.exp(torch.rand(D, generator=g) - 0.5)
    X = centres[lab] + torch.randn(N, D, generator=g) * std
    # means near data rows (not equal to them: sig = 0 exactly would make the
    # normwise relative comparison ill-posed)
    mu = X[torch.randperm(N, generator=g)[:K]] + 0.3 * torch.randn(K, D, generator=g)
    lss = 2.0 * torch.rand(K, D, generator=g) - 1.0
    lpi = torch.log_softmax(torch.randn(K, generator=g), 0)
    return X, mu, lss, lpi


SHAPES = [(1, 1, 1), (257, 3, 5), (3000, 129, 17), (5000, 200, 64), (4000, 1000, 96),
          (2500, 1024, 80)]


@pytest.mark.parametrize("N,K,D", SHAPES)
def test_tc_diag_vs_oracle_and_general(N, K, D):
    X, mu, lss, lpi = _case(N, K, D, seed=N + K + D)
    ref = O.estep_diag(X.numpy(), mu.numpy(), lss.numpy(), lpi.numpy())
    Xd, mud, lssd, lpid = (t.to(DEV) for t in (X, mu, lss, lpi))
    tc = _np(flash_gmm_diag_h100.flash_gmm_estep_diag(Xd, mud, lssd, lpid))
    gen = _np(L.estep(L.FGMM_VARIANT_DIAG, Xd, mud, lssd, lpid, force_general=True))
    assert_parity(tc, ref, what=f"tc diag {N}x{K}x{D} vs oracle")
    assert_parity(tc, gen, what=f"tc diag {N}x{K}x{D} vs general")


def test_tc_diag_offset_data_and_strided_inputs():
    """Data far from the origin (all features ~ +60) exercise the centring;
    X transposed in memory and mu with a row stride exercise the strides."""
    N, K, D = 6000, 300, 48
    X, mu, lss, lpi = _case(N, K, D, seed=11, offset=60.0)
    ref = O.estep_diag(X.numpy(), mu.numpy(), lss.numpy(), lpi.numpy())
    Xt = X.t().contiguous().to(DEV).t()                     # strides (1, N)
    mu_big = torch.zeros(K, 2 * D)
    mu_big[:, :D] = mu
    mud = mu_big.to(DEV)[:, :D]                             # strides (2D, 1)
    out = _np(L.estep(L.FGMM_VARIANT_DIAG, Xt, mud, lss.to(DEV), lpi.to(DEV)))
    assert_parity(out, ref, what="offset diag, strided")


@pytest.mark.parametrize("kind,N,K,D", [("iso", 600_000, 2048, 128), ("diag", 300_000, 1500, 96)])
def test_tc_more_than_1024_components_many_tiles(kind, N, K, D):
    """K > 1024 with many row tiles per cluster, so every stage buffer is
    reused many times in both passes: against the general kernels, plus
    sum_k Nk = N and sum_k mu_acc = sum_n x_n."""
    X, mu, cov, lpi = (t.to(DEV) for t in _many_components(kind, N, K, D, 0.0))
    v = L.FGMM_VARIANT_ISO if kind == "iso" else L.FGMM_VARIANT_DIAG
    tc = _np(L.estep(v, X, mu, cov, lpi))
    gen = _np(L.estep(v, X, mu, cov, lpi, force_general=True))
    assert np.isfinite(tc[0]).all() and np.isfinite(tc[1]).all()
    assert abs(tc[1].astype(np.float64).sum() - N) <= 1e-5 * N
    xs = X.double().sum(0).cpu().numpy()
    np.testing.assert_allclose(tc[2].astype(np.float64).sum(0), xs,
                               atol=1e-4 * np.abs(tc[2]).max() * 4)
    assert_parity(tc, gen, what=f"{kind} K={K} N={N} vs general")


def test_tc_iso_offset_data():
    """Isotropic data far from the origin (every feature near +60): the
    centred features keep the expanded distance at fp32-level accuracy."""
    X, mu, lss, lpi = _many_components("iso", 8000, 700, 128, 60.0)
    ref = O.estep_iso(X.numpy(), mu.numpy(), lss.numpy(), lpi.numpy())
    out = _np(L.estep(L.FGMM_VARIANT_ISO, *(t.to(DEV) for t in (X, mu, lss, lpi))))
    assert_parity(out, ref, what="offset iso")


def test_tc_diag_neg_inf_weight():
    N, K, D = 2000, 40, 16
    X, mu, lss, lpi = _case(N, K, D, seed=3)
    lpi[5] = -math.inf
    lpi[17] = -math.inf
    ref = O.estep_diag(X.numpy(), mu.numpy(), lss.numpy(), lpi.numpy())
    out = _np(flash_gmm_diag_h100.flash_gmm_estep_diag(*(t.to(DEV) for t in (X, mu, lss, lpi))))
    assert_parity(out, ref, what="diag -inf log_pi")
    assert out[1][5] == 0.0 and out[1][17] == 0.0


def test_c3_full_size():
    """C3 at full size (N=1M, K=1024, D=96) against the fp64 oracle, plus
    sum_k Nk = N and sum_k mu_acc = sum_n x_n."""
    X, mu, lss, lpi = gmm_data.make_config("c3", device=DEV)
    out = _np(flash_gmm_diag_h100.flash_gmm_estep_diag(X, mu, lss, lpi))
    logZ, Nk, mu_acc, sig = out
    N = X.shape[0]
    assert abs(Nk.astype(np.float64).sum() - N) <= 1e-5 * N
    xs = X.double().sum(0).cpu().numpy()
    np.testing.assert_allclose(mu_acc.astype(np.float64).sum(0), xs,
                               atol=1e-4 * np.abs(mu_acc).max() * 4)
    ref = O.estep_diag(X.cpu().numpy(), mu.cpu().numpy(), lss.cpu().numpy(), lpi.cpu().numpy())
    assert_parity(out, ref, what="C3 full size")


def _many_components(kind, N, K, D, offset):
    """The C2 / C3 recipes (gmm_data) with means moved off the data rows,
    varied variances and weights, all shifted by `offset`."""
    make = gmm_data.iso_mixture if kind == "iso" else gmm_data.diag_mixture
    X, mu, cov, _ = make(N, K, D, seed=K + D)
    g = torch.Generator().manual_seed(D)
    X, mu = X + offset, mu + offset + 0.3 * torch.randn(K, D, generator=g)
    if kind == "iso":
        cov = 0.4 * torch.rand(K, generator=g) - 0.2
    lpi = torch.log_softmax(torch.randn(K, generator=g), 0)
    return X, mu, cov, lpi


@pytest.mark.parametrize("kind,N,K,D,offset", [("iso", 4000, 1500, 64, 0.0),
                                               ("iso", 3000, 2048, 128, 0.0),
                                               ("iso", 4000, 3100, 32, 0.0),
                                               ("iso", 3000, 2048, 128, 40.0),
                                               ("diag", 3000, 1500, 48, 0.0),
                                               ("diag", 2400, 2300, 96, 0.0)])
def test_tc_more_than_1024_components(kind, N, K, D, offset):
    """K > 1024: blocks of 1024 components, LSE-only pass per block, combined
    logZ, then the statistics pass per block with that logZ."""
    X, mu, cov, lpi = _many_components(kind, N, K, D, offset)
    v = L.FGMM_VARIANT_ISO if kind == "iso" else L.FGMM_VARIANT_DIAG
    ref = (O.estep_iso if kind == "iso" else O.estep_diag)(X.numpy(), mu.numpy(), cov.numpy(),
                                                            lpi.numpy())
    Xd, mud, covd, lpid = (t.to(DEV) for t in (X, mu, cov, lpi))
    tc = _np(L.estep(v, Xd, mud, covd, lpid))
    gen = _np(L.estep(v, Xd, mud, covd, lpid, force_general=True))
    assert_parity(tc, ref, what=f"{kind} K={K} vs oracle")
    assert_parity(tc, gen, what=f"{kind} K={K} vs general")
    again = _np(L.estep(v, Xd, mud, covd, lpid))
    for a, b in zip(tc, again):
        np.testing.assert_array_equal(a, b)


@pytest.mark.parametrize("kind", ["iso", "diag"])
def test_tc_more_than_1024_components_edge_cases(kind):
    """K > 1024: -inf log-weights in several blocks (their Nk stays 0), a
    ragged last block, a transposed X, a single row, and the accumulate flag
    adding a second call's statistics."""
    N, K, D = 2500, 2100, 40
    X, mu, cov, lpi = _many_components(kind, N, K, D, 0.0)
    dead = [3, 1030, 2099]
    lpi[dead] = -math.inf
    v = L.FGMM_VARIANT_ISO if kind == "iso" else L.FGMM_VARIANT_DIAG
    oracle = O.estep_iso if kind == "iso" else O.estep_diag
    ref = oracle(X.numpy(), mu.numpy(), cov.numpy(), lpi.numpy())
    Xt = X.t().contiguous().to(DEV).t()
    mud, covd, lpid = mu.to(DEV), cov.to(DEV), lpi.to(DEV)
    out = _np(L.estep(v, Xt, mud, covd, lpid))
    assert_parity(out, ref, what=f"{kind} K={K} -inf weights, transposed X")
    assert all(out[1][k] == 0.0 for k in dead)

    one = _np(L.estep(v, Xt[:1], mud, covd, lpid))
    assert_parity(one, oracle(X[:1].numpy(), mu.numpy(), cov.numpy(), lpi.numpy()),
                  what=f"{kind} K={K} one row")

    first = L.estep(v, Xt[:1200], mud, covd, lpid)
    second = (torch.empty(N - 1200, device=DEV),) + tuple(t.clone() for t in first[1:])
    L.estep(v, Xt[1200:], mud, covd, lpid, out=second, accumulate=True)
    acc = (np.concatenate([_np(first)[0], _np(second)[0]]),) + _np(second)[1:]
    assert_parity(acc, ref, what=f"{kind} K={K} accumulated over two calls")


@pytest.mark.parametrize("N,K,D", [(3000, 300, 100), (4000, 1024, 128), (257, 5, 112),
                                   (2500, 1500, 120)])
def test_tc_diag_wide_features(N, K, D):
    """96 < D <= 128: 256 features on 64-row tiles (W_lo in shared memory,
    two distance passes added in registers), incl. K > 1024."""
    X, mu, lss, lpi = _case(N, K, D, seed=N + D)
    ref = O.estep_diag(X.numpy(), mu.numpy(), lss.numpy(), lpi.numpy())
    Xd, mud, lssd, lpid = (t.to(DEV) for t in (X, mu, lss, lpi))
    tc = _np(flash_gmm_diag_h100.flash_gmm_estep_diag(Xd, mud, lssd, lpid))
    gen = _np(L.estep(L.FGMM_VARIANT_DIAG, Xd, mud, lssd, lpid, force_general=True))
    assert_parity(tc, ref, what=f"diag wide {N}x{K}x{D} vs oracle")
    assert_parity(tc, gen, what=f"diag wide {N}x{K}x{D} vs general")
