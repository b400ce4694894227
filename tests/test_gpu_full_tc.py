"""Full-covariance tensor-core path (pass 1: x~ L GEMM + per-row log-sum-exp;
pass 2: R^T [x~ x~^T, x~, 1] statistics) against the fp64 oracle and the
general CUDA-core kernels.

Tolerances: logZ elementwise rel 1e-5, statistics normwise rel 1e-4
(tests/parity.py)."""

import math

import numpy as np
import pytest
import torch

import _fgmm_lib as L
import flash_gmm_full_h100
import gmm_data
from oracle import gmm_oracle as O
from parity import assert_parity

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _np(out):
    torch.cuda.synchronize()
    return tuple(t.detach().cpu().numpy() for t in out)


def _case(N, K, D, seed, offset=0.0):
    g = torch.Generator().manual_seed(seed)
    centres = 2.0 * torch.randn(K, D, generator=g) + offset
    lab = torch.randint(0, K, (N,), generator=g)
    C = torch.eye(D) + 0.1 * torch.tril(torch.randn(D, D, generator=g), -1)
    X = centres[lab] + torch.randn(N, D, generator=g) @ C
    mu = X[torch.randperm(N, generator=g)[:K]] + 0.3 * torch.randn(K, D, generator=g)
    off = 0.1 * torch.tril(torch.randn(K, D, D, generator=g), -1)
    Lc = off + torch.diag_embed(torch.exp(torch.rand(K, D, generator=g) - 0.5))
    lpi = torch.log_softmax(torch.randn(K, generator=g), 0)
    return X, mu, Lc, lpi


SHAPES = [(1, 1, 1), (257, 3, 5), (3000, 70, 24), (5000, 256, 64), (2000, 300, 33),
          (4100, 17, 48)]


@pytest.mark.parametrize("N,K,D", SHAPES)
def test_tc_full_vs_oracle_and_general(N, K, D):
    X, mu, Lc, lpi = _case(N, K, D, seed=N + K + D)
    ref = O.estep_full(X.numpy(), mu.numpy(), Lc.numpy(), lpi.numpy())
    Xd, mud, Ld, lpid = (t.to(DEV) for t in (X, mu, Lc, lpi))
    tc = _np(flash_gmm_full_h100.flash_gmm_estep_full(Xd, mud, Ld, lpid))
    gen = _np(L.estep(L.FGMM_VARIANT_FULL, Xd, mud, Ld, lpid, force_general=True))
    assert_parity(tc, ref, what=f"tc full {N}x{K}x{D} vs oracle")
    assert_parity(tc, gen, what=f"tc full {N}x{K}x{D} vs general")


def test_tc_full_offset_data_and_strided_inputs():
    N, K, D = 3000, 40, 32
    X, mu, Lc, lpi = _case(N, K, D, seed=21, offset=40.0)
    ref = O.estep_full(X.numpy(), mu.numpy(), Lc.numpy(), lpi.numpy())
    Xt = X.t().contiguous().to(DEV).t()
    mu_big = torch.zeros(K, 2 * D)
    mu_big[:, :D] = mu
    mud = mu_big.to(DEV)[:, :D]
    out = _np(L.estep(L.FGMM_VARIANT_FULL, Xt, mud, Lc.to(DEV), lpi.to(DEV)))
    assert_parity(out, ref, what="offset full, strided")


def test_tc_full_neg_inf_weight_and_accumulate():
    N, K, D = 2500, 30, 16
    X, mu, Lc, lpi = _case(N, K, D, seed=4)
    lpi[3] = -math.inf
    ref = O.estep_full(X.numpy(), mu.numpy(), Lc.numpy(), lpi.numpy())
    Xd, mud, Ld, lpid = (t.to(DEV) for t in (X, mu, Lc, lpi))
    out = _np(flash_gmm_full_h100.flash_gmm_estep_full(Xd, mud, Ld, lpid))
    assert_parity(out, ref, what="full -inf log_pi")
    assert out[1][3] == 0.0
    again = _np(flash_gmm_full_h100.flash_gmm_estep_full(Xd, mud, Ld, lpid))
    for u, w in zip(out, again):
        np.testing.assert_array_equal(u, w)          # bitwise run-to-run
    acc = L.estep(L.FGMM_VARIANT_FULL, Xd[:1000], mud, Ld, lpid)
    acc = (torch.empty(N - 1000, device=DEV),) + acc[1:]
    L.estep(L.FGMM_VARIANT_FULL, Xd[1000:], mud, Ld, lpid, out=acc, accumulate=True)
    acc = _np(acc)
    for u, w in zip(acc[1:], out[1:]):
        assert np.max(np.abs(u - w)) <= 1e-5 * np.max(np.abs(w))


def test_c4_full_size():
    """C4 at full size (N=250K, K=256, D=64): the tensor-core path against the
    general CUDA-core kernels (themselves oracle-checked), the fp64 oracle's
    logZ on the first 20,000 rows, and the invariants sum_k Nk = N,
    sum_k mu_acc = sum_n x_n and sum_k sig_outer = sum_n x x^T."""
    X, mu, Lc, lpi = gmm_data.make_config("c4", device=DEV)
    out = _np(flash_gmm_full_h100.flash_gmm_estep_full(X, mu, Lc, lpi))
    logZ, Nk, mu_acc, sig = out
    N = X.shape[0]
    assert abs(Nk.astype(np.float64).sum() - N) <= 1e-5 * N
    Xc = X.double().cpu().numpy()
    np.testing.assert_allclose(mu_acc.astype(np.float64).sum(0), Xc.sum(0),
                               atol=1e-4 * np.abs(mu_acc).max() * 4)
    np.testing.assert_allclose(sig.astype(np.float64).sum(0), Xc.T @ Xc,
                               atol=1e-4 * np.abs(sig).max() * 4)
    gen = _np(L.estep(L.FGMM_VARIANT_FULL, X, mu, Lc, lpi, force_general=True))
    assert_parity(out, gen, what="C4 full size vs general")
    ll = O.loglik_full(Xc[:20000], mu.cpu().numpy(), Lc.cpu().numpy(), lpi.cpu().numpy())
    m = ll.max(axis=1, keepdims=True)
    lz = (m + np.log(np.exp(ll - m).sum(axis=1, keepdims=True)))[:, 0]
    err = np.max(np.abs(logZ[:20000] - lz) / np.maximum(1.0, np.abs(lz)))
    assert err <= 1e-5, f"C4 logZ rel err {err:.3e}"
