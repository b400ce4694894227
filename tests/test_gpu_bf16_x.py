"""bfloat16-stored X (fgmm_estep_x with FGMM_X_BF16): every path widens X
exactly as it reads it, so the results must equal, bit for bit, those of the
fp32 entry points on the widened values -- tensor-core (128-row, wide and
diagonal kernels, full covariance, K > 1024) and general kernels, contiguous,
transposed and 2-byte-aligned X."""

import numpy as np
import pytest
import torch

import _fgmm_lib as L
import gmm_data

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _np(out):
    torch.cuda.synchronize()
    return tuple(t.detach().cpu().numpy() for t in out)


def _inputs(kind, N, K, D, seed):
    g = torch.Generator().manual_seed(seed)
    if kind == "full":
        X, mu, cov, lpi = gmm_data.full_mixture(N, K, D, seed=seed)
    elif kind == "diag":
        X, mu, cov, lpi = gmm_data.diag_mixture(N, K, D, seed=seed)
    else:
        X, mu, cov, lpi = gmm_data.iso_mixture(N, K, D, seed=seed)
        cov = 0.4 * torch.rand(K, generator=g) - 0.2
    mu = mu + 0.2 * torch.randn(mu.shape, generator=g)
    return X, mu, cov, lpi


VARIANT = {"iso": L.FGMM_VARIANT_ISO, "diag": L.FGMM_VARIANT_DIAG, "full": L.FGMM_VARIANT_FULL}
CASES = [("iso", 5000, 300, 128), ("iso", 3000, 200, 200), ("iso", 3000, 1500, 64),
         ("diag", 4000, 300, 96), ("diag", 3000, 200, 120), ("full", 3000, 100, 48),
         ("full", 1500, 40, 80)]


@pytest.mark.parametrize("kind,N,K,D", CASES)
@pytest.mark.parametrize("general", [False, True])
def test_bf16_x_equals_fp32_on_widened_values(kind, N, K, D, general):
    X, mu, cov, lpi = _inputs(kind, N, K, D, seed=N + K + D)
    Xb = X.to(DEV).to(torch.bfloat16)
    Xw = Xb.float()
    args = tuple(t.to(DEV) for t in (mu, cov, lpi))
    v = VARIANT[kind]
    a = _np(L.estep(v, Xb, *args, force_general=general))
    b = _np(L.estep(v, Xw, *args, force_general=general))
    for x, y in zip(a, b):
        np.testing.assert_array_equal(x, y)


@pytest.mark.parametrize("kind,D", [("iso", 128), ("diag", 96), ("full", 64)])
def test_bf16_x_strided_and_unaligned(kind, D):
    """A transposed bf16 X and one starting 2 bytes past an 8-byte boundary
    (no vector loads) give the contiguous result."""
    N, K = 4000, 150
    X, mu, cov, lpi = _inputs(kind, N, K, D, seed=D)
    Xb = X.to(DEV).to(torch.bfloat16)
    args = tuple(t.to(DEV) for t in (mu, cov, lpi))
    v = VARIANT[kind]
    ref = _np(L.estep(v, Xb, *args))
    Xt = Xb.t().contiguous().t()
    buf = torch.empty(N * D + 1, dtype=torch.bfloat16, device=DEV)
    Xu = buf[1:].view(N, D)
    Xu.copy_(Xb)
    for Xs in (Xt, Xu):
        out = _np(L.estep(v, Xs, *args))
        for x, y in zip(out, ref):
            np.testing.assert_array_equal(x, y)
