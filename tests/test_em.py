"""EM fitting (flash-gmm_b200/gmm_em.py): M-step formulas, the EM loop's
monotone log-likelihood and recovery of a separated mixture on CPU with the
oracle E-step, the sharded loop on 2 gloo ranks, and (GPU) the library
E-step against the oracle inside the same loop."""

import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import gmm_em as EM
from oracle import gmm_oracle as O

ORACLE = {"iso": O.estep_iso, "diag": O.estep_diag, "full": O.estep_full}


def oracle_estep(kind):
    def run(X, mu, cov, lpi):
        lz, nk, ma, sg = ORACLE[kind](X.cpu().numpy(), mu.cpu().numpy(), cov.cpu().numpy(),
                                      lpi.cpu().numpy())
        t = lambda a: torch.tensor(a, dtype=torch.float32)
        return torch.tensor(lz.sum(), dtype=torch.float64), t(nk), t(ma), t(sg)
    return run


def oracle_local(kind):
    def run(X, mu, cov, lpi, out):
        lz, nk, ma, sg = ORACLE[kind](X.numpy(), mu.numpy(), cov.numpy(), lpi.numpy())
        for dst, src in zip(out, (lz, nk, ma, sg)):
            dst.copy_(torch.from_numpy(np.asarray(src, dtype=np.float32)).reshape(dst.shape))
    return run


def mixture(N, K, D, seed, sep=8.0):
    g = torch.Generator().manual_seed(seed)
    centres = sep * torch.randn(K, D, generator=g)
    lab = torch.randint(0, K, (N,), generator=g)
    X = centres[lab] + torch.randn(N, D, generator=g) * (0.5 + torch.rand(K, 1, generator=g)[lab])
    return X, centres


@pytest.mark.parametrize("kind", ["iso", "diag", "full"])
def test_m_step_closed_forms(kind):
    g = torch.Generator().manual_seed(3)
    N, K, D = 1000, 5, 4
    X = torch.randn(N, D, generator=g) * 2
    r = torch.softmax(torch.randn(N, K, generator=g), 1).double()
    mu_old = torch.randn(K, D, generator=g)
    Nk = r.sum(0)
    mu_acc = r.T @ X.double()
    diff = X.double()[:, None, :] - mu_old.double()[None]
    if kind == "iso":
        sig = (r[:, :, None] * diff ** 2).sum((0, 2)); cov_old = torch.zeros(K)
    elif kind == "diag":
        sig = (r[:, :, None] * diff ** 2).sum(0); cov_old = torch.zeros(K, D)
    else:
        sig = torch.einsum("nk,ni,nj->kij", r, X.double(), X.double()); cov_old = torch.eye(D).repeat(K, 1, 1)
    mu, cov, lpi = EM.m_step(kind, N, Nk.float(), mu_acc.float(), sig.float(), mu_old, cov_old,
                             reg_covar=0.0)
    mu_ref = mu_acc / Nk[:, None]
    np.testing.assert_allclose(mu.numpy(), mu_ref.numpy(), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(lpi.exp().numpy(), (Nk / N).numpy(), rtol=1e-5)
    dn = X.double()[:, None, :] - mu_ref[None]
    if kind == "iso":
        var = (r[:, :, None] * dn ** 2).sum((0, 2)) / (D * Nk)
        np.testing.assert_allclose(cov.exp().numpy(), var.numpy(), rtol=1e-4)
    elif kind == "diag":
        var = (r[:, :, None] * dn ** 2).sum(0) / Nk[:, None]
        np.testing.assert_allclose(cov.exp().numpy(), var.numpy(), rtol=1e-4)
    else:
        S = torch.einsum("nk,nki,nkj->kij", r, dn, dn) / Nk[:, None, None]
        P = cov.double() @ cov.double().transpose(1, 2)
        np.testing.assert_allclose((P @ S).numpy(), np.broadcast_to(np.eye(D), (K, D, D)),
                                   atol=1e-3)


def test_m_step_readme_variance_and_dead_components():
    N, K, D = 100, 3, 2
    Nk = torch.tensor([50.0, 0.0, 50.0])
    mu_acc = torch.tensor([[50.0, 0.0], [0.0, 0.0], [0.0, 100.0]])
    sig = torch.tensor([100.0, 0.0, 200.0])
    mu_old = torch.tensor([[0.0, 0.0], [7.0, 7.0], [0.0, 0.0]])
    cov_old = torch.tensor([0.1, 0.2, 0.3])
    mu, cov, lpi = EM.m_step("iso", N, Nk, mu_acc, sig, mu_old, cov_old, reg_covar=0.0,
                             variance="readme")
    assert torch.allclose(cov[[0, 2]].exp(), torch.tensor([1.0, 2.0]))   # sig / (D Nk)
    assert torch.equal(mu[1], mu_old[1]) and cov[1] == cov_old[1]        # dead component kept
    assert lpi[1] < -20


@pytest.mark.parametrize("kind", ["iso", "diag", "full"])
def test_fit_with_oracle_is_monotone_and_recovers_centres(kind):
    X, centres = mixture(1500, 4, 3, seed=11)
    init = EM.init_params(X, 4, kind, seed=2)
    out = EM.fit(X, init=init, covariance_type=kind, n_iter=40, tol=1e-7,
                 estep_fn=oracle_estep(kind))
    ll = out["log_likelihood"]
    assert all(b >= a - 1e-6 * abs(a) for a, b in zip(ll, ll[1:])), ll
    # every true centre has a fitted mean next to it
    d = torch.cdist(centres, out["mu"])
    assert float(d.min(1).values.max()) < 0.5


def _sharded_fit_worker(rank, world, kind, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    X, _ = mixture(1200, 3, 2, seed=5)
    init = EM.init_params(X, 3, kind, seed=1)
    lo, hi = rank * 600, (rank + 1) * 600
    out = EM.fit(X[lo:hi], init=init, covariance_type=kind, n_iter=8, tol=0.0,
                 estep_fn=EM.sharded_estep(kind, local_estep=oracle_local(kind)), n_rows=1200)
    if rank == 0:
        q.put((out["mu"].numpy(), out["log_likelihood"]))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("kind", ["iso", "diag", "full"])
def test_sharded_fit_on_two_gloo_ranks_matches_single_process(kind):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + (os.getpid() % 300)
    procs = [ctx.Process(target=_sharded_fit_worker, args=(r, 2, kind, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    mu_sh, ll_sh = q.get(timeout=120)
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    X, _ = mixture(1200, 3, 2, seed=5)
    init = EM.init_params(X, 3, kind, seed=1)
    out = EM.fit(X, init=init, covariance_type=kind, n_iter=8, tol=0.0,
                 estep_fn=oracle_estep(kind))
    np.testing.assert_allclose(mu_sh, out["mu"].numpy(), rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(ll_sh, out["log_likelihood"], rtol=1e-5)


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["iso", "diag", "full"])
def test_fit_with_library_estep_tracks_the_oracle(kind):
    X, centres = mixture(20000, 16, 8, seed=7)
    init = EM.init_params(X, 16, kind, seed=3)
    gpu = EM.fit(X.cuda(), init=tuple(t.cuda() for t in init), covariance_type=kind, n_iter=6,
                 tol=0.0)
    cpu = EM.fit(X, init=init, covariance_type=kind, n_iter=6, tol=0.0,
                 estep_fn=oracle_estep(kind))
    np.testing.assert_allclose(gpu["log_likelihood"], cpu["log_likelihood"], rtol=1e-5)
    np.testing.assert_allclose(gpu["mu"].cpu().numpy(), cpu["mu"].numpy(), rtol=1e-3, atol=1e-3)
    np.testing.assert_allclose(gpu["log_pi"].cpu().numpy(), cpu["log_pi"].numpy(), atol=1e-3)
