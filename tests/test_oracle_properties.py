"""Size-independent properties of the E-step, checked on the CPU oracle:
component permutation, row-split additivity (the streaming identity), shift
invariance of the centred statistics, -inf weights, and the identities that
tie the three variants together (a diagonal model with equal per-dimension
variances is the isotropic one; a full model with L_k = exp(-lss_k/2) I is
too).  The GPU parity tests apply the same identities to the CUDA path."""

import numpy as np
import pytest

from oracle import gmm_oracle as O

RTOL = 1e-10


def _iso_case(N=700, K=37, D=11, seed=0):
    rng = np.random.default_rng(seed)
    centres = 2.0 * rng.standard_normal((K, D))
    X = centres[rng.integers(0, K, N)] + rng.standard_normal((N, D))
    mu = X[rng.permutation(N)[:K]] + 0.1 * rng.standard_normal((K, D))
    lss = 0.6 * rng.random(K) - 0.3
    lpi = rng.standard_normal(K)
    lpi -= np.log(np.exp(lpi).sum())
    return X, mu, lss, lpi


def _close(a, b, rtol=RTOL):
    a, b = np.asarray(a), np.asarray(b)
    scale = max(1.0, float(np.max(np.abs(b), initial=0.0)))
    assert float(np.max(np.abs(a - b), initial=0.0)) <= rtol * scale


def _cases():
    X, mu, lss, lpi = _iso_case()
    rng = np.random.default_rng(1)
    K, D = mu.shape
    lss_d = 0.6 * rng.random((K, D)) - 0.3
    L = np.tril(0.1 * rng.standard_normal((K, D, D)), -1)
    L[:, np.arange(D), np.arange(D)] = np.exp(rng.random((K, D)) - 0.5)
    return {"iso": (O.estep_iso, X, mu, lss, lpi),
            "diag": (O.estep_diag, X, mu, lss_d, lpi),
            "full": (O.estep_full, X, mu, L, lpi)}


@pytest.mark.parametrize("kind", ["iso", "diag", "full"])
def test_component_permutation(kind):
    fn, X, mu, cov, lpi = _cases()[kind]
    perm = np.random.default_rng(2).permutation(mu.shape[0])
    a = fn(X, mu, cov, lpi)
    b = fn(X, mu[perm], cov[perm], lpi[perm])
    _close(b[0], a[0])
    for x, y in zip(b[1:], a[1:]):
        _close(x, y[perm])


@pytest.mark.parametrize("kind", ["iso", "diag", "full"])
def test_row_split_additivity(kind):
    fn, X, mu, cov, lpi = _cases()[kind]
    whole = fn(X, mu, cov, lpi)
    parts = [fn(X[s], mu, cov, lpi) for s in (slice(0, 1), slice(1, 333), slice(333, None))]
    _close(np.concatenate([p[0] for p in parts]), whole[0])
    for i in (1, 2, 3):
        _close(sum(p[i] for p in parts), whole[i])


@pytest.mark.parametrize("kind", ["iso", "diag", "full"])
def test_shift_of_data_and_means(kind):
    """x -> x + c, mu -> mu + c: logZ, Nk and the centred iso/diag statistics
    stay, mu_acc gains Nk c, and the uncentred full sig_outer gains
    c mu_acc^T + mu_acc c^T + Nk c c^T."""
    fn, X, mu, cov, lpi = _cases()[kind]
    c = np.random.default_rng(3).standard_normal(X.shape[1]) * 5.0
    a = fn(X, mu, cov, lpi)
    b = fn(X + c, mu + c, cov, lpi)
    _close(b[0], a[0], 1e-9)
    _close(b[1], a[1], 1e-9)
    _close(b[2], a[2] + a[1][:, None] * c[None, :], 1e-9)
    if kind == "full":
        extra = (np.einsum("i,kj->kij", c, a[2]) + np.einsum("ki,j->kij", a[2], c)
                 + a[1][:, None, None] * np.outer(c, c)[None])
        _close(b[3], a[3] + extra, 1e-9)
    else:
        _close(b[3], a[3], 1e-9)


@pytest.mark.parametrize("kind", ["iso", "diag", "full"])
def test_neg_inf_weight_removes_the_component(kind):
    fn, X, mu, cov, lpi = _cases()[kind]
    dead = np.array([0, 5, 20])
    lpi2 = lpi.copy()
    lpi2[dead] = -np.inf
    keep = np.setdiff1d(np.arange(mu.shape[0]), dead)
    a = fn(X, mu, cov, lpi2)
    b = fn(X, mu[keep], cov[keep], lpi2[keep])
    _close(a[0], b[0])
    assert np.all(a[1][dead] == 0.0) and np.all(a[2][dead] == 0.0) and np.all(a[3][dead] == 0.0)
    for x, y in zip(a[1:], b[1:]):
        _close(x[keep], y)


def test_diag_with_equal_variances_is_iso():
    X, mu, lss, lpi = _iso_case()
    D = X.shape[1]
    a = O.estep_iso(X, mu, lss, lpi)
    b = O.estep_diag(X, mu, np.repeat(lss[:, None], D, axis=1), lpi)
    for x, y in zip(b[:3], a[:3]):
        _close(x, y)
    _close(b[3].sum(axis=1), a[3])      # sum_d r (x_d - mu_d)^2 = r ||x - mu||^2


def test_full_with_scaled_identity_cholesky_is_iso():
    X, mu, lss, lpi = _iso_case()
    K, D = mu.shape
    L = np.exp(-0.5 * lss)[:, None, None] * np.eye(D)[None]
    a = O.estep_iso(X, mu, lss, lpi)
    b = O.estep_full(X, mu, L, lpi)
    for x, y in zip(b[:3], a[:3]):
        _close(x, y)
    # centred from the uncentred second moment: tr(S_k) - 2 mu_k.m_k + Nk |mu_k|^2
    centred = (np.trace(b[3], axis1=1, axis2=2) - 2.0 * np.sum(mu * b[2], axis=1)
               + b[1] * np.sum(mu * mu, axis=1))
    _close(centred, a[3], 1e-9)


def test_responsibilities_sum_to_one_and_logz_is_the_normaliser():
    X, mu, lss, lpi = _iso_case(N=50)
    ll, _ = O.loglik_iso(X, mu, lss, lpi)
    logZ, Nk, _, _ = O.estep_iso(X, mu, lss, lpi)
    r = np.exp(ll - logZ[:, None])
    _close(r.sum(axis=1), np.ones(50))
    _close(r.sum(axis=0), Nk)
    _close(logZ, np.log(np.exp(ll).sum(axis=1)))
