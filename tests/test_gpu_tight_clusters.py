"""Inputs where the expanded distance |x|^2 - 2 x.mu + |mu|^2 cancels hard,
through the drop-in entry points (default dispatch, i.e. the tensor-core
path), against the fp64 oracle; and the full-size C4 statistics against the
oracle.

The tight-cluster recipe: cluster centres ~ N(0, 9 I) (three times the unit
noise), rows = centre + N(0, I), means within 0.01 of data rows, log
variances ~ U(-1, 1) (down to -1: sharper components weigh the distance
more), log weights = log_softmax(N(0, 1)).  Rows then sit close to a mean
while |x - c| and |mu - c| stay large, so the distance is a small difference
of large products -- the regime where an fp32 expanded form loses the most.

Tolerances: logZ elementwise rel 1e-5, statistics normwise rel 1e-4
(tests/parity.py)."""

import pytest
import torch

import flash_gmm
import flash_gmm_diag_h100
import flash_gmm_full_h100
import gmm_data
from oracle import gmm_oracle as O
from parity import assert_parity

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _np(out):
    torch.cuda.synchronize()
    return tuple(t.detach().cpu().numpy() for t in out)


def _tight(N, K, D, kind, seed, equal_var=False):
    g = torch.Generator().manual_seed(seed)
    centres = 3.0 * torch.randn(K, D, generator=g)
    lab = torch.randint(0, K, (N,), generator=g)
    X = centres[lab] + torch.randn(N, D, generator=g)
    mu = X[torch.randperm(N, generator=g)[:K]] + 0.01 * torch.randn(K, D, generator=g)
    shape = (K,) if kind == "iso" else (K, D)
    if equal_var:
        lss = torch.full(shape, -1.0)
    else:
        lss = 2.0 * torch.rand(shape, generator=g) - 1.0
    lpi = torch.log_softmax(torch.randn(K, generator=g), 0)
    return X, mu, lss, lpi


@pytest.mark.parametrize("kind,N,K,D,equal_var", [
    ("iso", 65536, 1024, 128, False),   # C2 shape, per-component variances
    ("iso", 65536, 1024, 128, True),    # C2 shape, one shared variance (e^-1)
    ("iso", 40000, 256, 64, False),
    ("diag", 65536, 1024, 96, False),   # C3 shape
    ("diag", 40000, 512, 64, False),
    ("iso", 30000, 1024, 256, False),   # wide kernel (64-row tiles, two distance chains)
    ("iso", 30000, 2048, 128, False),   # one pass on 16-CTA clusters
    ("iso", 20000, 4096, 64, False),    # blocks of 1024 components, two phases
    ("diag", 30000, 1024, 128, False),  # wide diagonal
    ("diag", 20000, 4096, 64, False),   # blocked diagonal
], ids=["iso-c2", "iso-c2-equal-var", "iso-k256", "diag-c3", "diag-k512", "iso-d256",
        "iso-k2048", "iso-k4096", "diag-d128", "diag-k4096"])
def test_tight_clusters_default_path_vs_oracle(kind, N, K, D, equal_var):
    X, mu, lss, lpi = _tight(N, K, D, kind, seed=11 + K + D, equal_var=equal_var)
    args = (X.to(DEV), mu.to(DEV), lss.to(DEV), lpi.to(DEV))
    if kind == "iso":
        out = _np(flash_gmm.flash_gmm_estep(*args, BLOCK_D=max(128, D)))
    else:
        out = _np(flash_gmm_diag_h100.flash_gmm_estep_diag(*args))
    ref = (O.estep_iso if kind == "iso" else O.estep_diag)(
        X.numpy(), mu.numpy(), lss.numpy(), lpi.numpy())
    assert_parity(out, ref, what=f"tight clusters {kind} N={N} K={K} D={D}")


def test_c4_full_size_statistics_vs_oracle():
    """All 250K rows of the C4 recipe (K = 256, D = 64): logZ, Nk, mu_acc and
    the uncentred sig_outer (flash_gmm_full_h100.py:213-228) against the fp64
    oracle."""
    X, mu, L, lpi = gmm_data.make_config("c4")
    out = _np(flash_gmm_full_h100.flash_gmm_estep_full(X.to(DEV), mu.to(DEV), L.to(DEV),
                                                       lpi.to(DEV)))
    ref = O.estep_full(X.numpy(), mu.numpy(), L.numpy(), lpi.numpy())
    assert_parity(out, ref, what="C4 full size vs oracle")
