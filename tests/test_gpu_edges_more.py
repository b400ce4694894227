"""Edge cases across the newer paths: K just above 1024 (a 16-CTA cluster
mostly of padding components), one row with K > 1024, the wide diagonal
kernel with -inf weights on offset data, streaming over bfloat16 chunks with
a ragged last chunk, and an EM fit on bfloat16 X.  Parity bar: tests/parity.py
(logZ elementwise 1e-5 relative, statistics normwise 1e-4)."""

import math

import numpy as np
import pytest
import torch

import _fgmm_lib as L
import gmm_data
import gmm_em
import gmm_stream as GS
from oracle import gmm_oracle as O
from parity import assert_parity

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _np(out):
    torch.cuda.synchronize()
    return tuple(t.detach().cpu().numpy() for t in out)


def _iso(N, K, D, seed):
    X, mu, _, _ = gmm_data.iso_mixture(max(N, K), K, D, seed=seed)
    g = torch.Generator().manual_seed(seed)
    X = X[:N]
    mu = mu + 0.3 * torch.randn(K, D, generator=g)
    lss = 0.4 * torch.rand(K, generator=g) - 0.2
    lpi = torch.log_softmax(torch.randn(K, generator=g), 0)
    return X, mu, lss, lpi


@pytest.mark.parametrize("N,K,D", [(3000, 1025, 64), (1, 1500, 96), (7, 2048, 33)])
def test_iso_components_just_past_1024_and_single_rows(N, K, D):
    X, mu, lss, lpi = _iso(N, K, D, seed=N + K)
    ref = O.estep_iso(X.numpy(), mu.numpy(), lss.numpy(), lpi.numpy())
    out = _np(L.estep(L.FGMM_VARIANT_ISO, *(t.to(DEV) for t in (X, mu, lss, lpi))))
    assert_parity(out, ref, what=f"iso {N}x{K}x{D}")


def test_diag_wide_neg_inf_weights_offset_data():
    N, K, D = 3000, 250, 128
    X, mu, lss, lpi = gmm_data.diag_mixture(N, K, D, seed=9)
    g = torch.Generator().manual_seed(9)
    X, mu = X + 25.0, mu + 25.0 + 0.3 * torch.randn(K, D, generator=g)
    lpi[[0, 200]] = -math.inf
    ref = O.estep_diag(X.numpy(), mu.numpy(), lss.numpy(), lpi.numpy())
    out = _np(L.estep(L.FGMM_VARIANT_DIAG, *(t.to(DEV) for t in (X, mu, lss, lpi))))
    assert_parity(out, ref, what="diag D=128 offset, -inf weights")
    assert out[1][0] == 0.0 and out[1][200] == 0.0


def test_stream_bf16_chunks_with_ragged_last_chunk():
    X, mu, lss, lpi = _iso(50_000, 300, 128, seed=4)
    Xb = X.to(torch.bfloat16)
    chunks = [Xb[i:i + 16_384].pin_memory() for i in range(0, Xb.shape[0], 16_384)]
    assert chunks[-1].shape[0] != 16_384
    args = tuple(t.to(DEV) for t in (mu, lss, lpi))
    logZ, Nk, mu_acc, sig = GS.stream_estep(chunks, *args, keep_logZ=True)
    one = L.estep(L.FGMM_VARIANT_ISO, Xb.to(DEV), *args)
    assert_parity(_np((logZ, Nk, mu_acc, sig)), _np(one), what="bf16 stream vs one call")


def test_em_fit_on_bf16_x_matches_fp32_fit_on_widened_values():
    X, _, _, _ = gmm_data.iso_mixture(20_000, 32, 16, seed=12)
    Xb = X.to(DEV).to(torch.bfloat16)
    a = gmm_em.fit(Xb, K=32, covariance_type="iso", n_iter=5, seed=1)
    b = gmm_em.fit(Xb.float(), K=32, covariance_type="iso", n_iter=5, seed=1)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(np.array(a["log_likelihood"]), np.array(b["log_likelihood"]))
    for key in ("mu", "cov", "log_pi"):
        assert torch.equal(a[key], b[key])
