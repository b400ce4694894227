"""X scale of the tensor-core paths: data far from the means' centre.

The split passes scale x - c by one power of two so that its fp16 hi/lo
words stay in range.  The scale comes from the largest |mu - c| and from an
evenly spaced sample of 4096 rows of X, so inputs whose means sit close
together (a single component, means near the global mean) keep the data in
range; a row far outside everything sampled sets the workspace's status word
(FGMM_STATUS_RANGE) and makes the statistics NaN, which estep(check=True)
turns into an exception.  Tolerances as in tests/parity.py."""

import pytest
import torch

import _fgmm_lib as L
import flash_gmm
import flash_gmm_diag_h100
from oracle import gmm_oracle as O
from parity import assert_parity

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _np(out):
    torch.cuda.synchronize()
    return tuple(t.detach().cpu().numpy() for t in out)


def test_diag_single_component_on_unstandardised_features():
    """K = 1 (so every mean equals the centre and max|mu - c| = 0) on features
    around 1e3 with spread 1e2: the scale must come from the data."""
    g = torch.Generator().manual_seed(3)
    N, D = 20000, 48
    X = 1000.0 + 100.0 * torch.randn(N, D, generator=g)
    mu = X.mean(0, keepdim=True) + torch.randn(1, D, generator=g)
    lss = torch.log(X.var(0, keepdim=True)) + 0.1 * torch.randn(1, D, generator=g)
    lpi = torch.zeros(1)
    out = _np(flash_gmm_diag_h100.flash_gmm_estep_diag(X.to(DEV), mu.to(DEV), lss.to(DEV),
                                                       lpi.to(DEV)))
    assert_parity(out, O.estep_diag(X.numpy(), mu.numpy(), lss.numpy(), lpi.numpy()),
                  what="diag K=1, |x| ~ 1e3")


@pytest.mark.parametrize("kind", ["iso", "diag"])
def test_means_near_the_global_mean(kind):
    """Means = global mean + 0.01 N(0, 1): max|mu - c| is tiny against the
    data's spread."""
    g = torch.Generator().manual_seed(4)
    N, K, D = 30000, 64, 32
    X = 5.0 + 2.0 * torch.randn(N, D, generator=g)
    mu = X.mean(0, keepdim=True) + 0.01 * torch.randn(K, D, generator=g)
    shape = (K,) if kind == "iso" else (K, D)
    lss = torch.log(torch.full(shape, 4.0)) + 0.05 * torch.randn(shape, generator=g)
    lpi = torch.log_softmax(torch.randn(K, generator=g), 0)
    fn = flash_gmm.flash_gmm_estep if kind == "iso" else flash_gmm_diag_h100.flash_gmm_estep_diag
    out = _np(fn(X.to(DEV), mu.to(DEV), lss.to(DEV), lpi.to(DEV)))
    ref = (O.estep_iso if kind == "iso" else O.estep_diag)(X.numpy(), mu.numpy(), lss.numpy(),
                                                            lpi.numpy())
    assert_parity(out, ref, what=f"{kind} means near the global mean")


def test_row_outside_the_range_is_reported():
    """One row 1e8 away from the centre, not among the sampled rows (rows
    i * N / 4096; row 1 is not one of them): the status word says so, the
    statistics are NaN, and check=True raises."""
    g = torch.Generator().manual_seed(5)
    N, K, D = 20000, 64, 32
    X = torch.randn(N, D, generator=g)
    X[1, 0] = 1e8
    mu = torch.randn(K, D, generator=g)
    lss = torch.zeros(K)
    lpi = torch.full((K,), -torch.log(torch.tensor(float(K))).item())
    args = [t.to(DEV) for t in (X, mu, lss, lpi)]
    with pytest.raises(L.FlashGMMError, match="fp16's range"):
        L.estep(L.FGMM_VARIANT_ISO, *args, check=True)
    out = L.estep(L.FGMM_VARIANT_ISO, *args)
    torch.cuda.synchronize()
    assert torch.isnan(out[1]).all() and torch.isnan(out[2]).all()
    # in range again: the same call on the data without the outlier is clean
    X[1, 0] = 0.5
    L.estep(L.FGMM_VARIANT_ISO, X.to(DEV), *args[1:], check=True)
