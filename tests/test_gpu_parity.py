"""CUDA path vs the reference's golden outputs and the CPU oracle.

Every call goes through the drop-in entry points -> C ABI ->
libflashgmm_sm100.so.  Tolerances: logZ elementwise rel 1e-5, statistics
normwise rel 1e-4 (tests/parity.py)."""


import numpy as np
import pytest
import torch

import _fgmm_lib as L
import flash_gmm
import flash_gmm_diag_h100
import flash_gmm_full_h100
import flash_gmm_h100
import gmm_data
from oracle import gmm_oracle as O
from parity import assert_parity, golden_inputs, golden_names, load_golden, variant_of

pytestmark = pytest.mark.gpu
DEV = "cuda"
ORACLE = {"iso": O.estep_iso, "diag": O.estep_diag, "full": O.estep_full}
VARIANT = {"iso": L.FGMM_VARIANT_ISO, "diag": L.FGMM_VARIANT_DIAG, "full": L.FGMM_VARIANT_FULL}
ENTRY = {"iso": flash_gmm.flash_gmm_estep, "diag": flash_gmm_diag_h100.flash_gmm_estep_diag,
         "full": flash_gmm_full_h100.flash_gmm_estep_full}


def _np(out):
    torch.cuda.synchronize()
    return tuple(t.detach().cpu().numpy() for t in out)


def _to_dev(X, *rest):
    if X.flags.c_contiguous:
        Xt = torch.from_numpy(np.array(X)).to(DEV)
    else:   # keep the fixture's strided (transposed) layout on the device
        Xt = torch.from_numpy(np.ascontiguousarray(X.T)).to(DEV).t()
    return (Xt,) + tuple(torch.from_numpy(np.ascontiguousarray(a)).to(DEV) for a in rest)


NAMES = [n for n in golden_names() if n != "diag_slab_overlap_defect"]


@pytest.mark.parametrize("general", [False, True], ids=["auto", "general"])
@pytest.mark.parametrize("name", NAMES)
def test_golden_fixture(name, general):
    z = load_golden(name)
    v = variant_of(name)
    X, mu, cov, lpi = golden_inputs(name, z)
    Xd, mud, covd, lpid = _to_dev(X, mu, cov, lpi)
    if general:
        out = _np(L.estep(VARIANT[v], Xd, mud, covd, lpid, force_general=True))
    else:
        out = _np(ENTRY[v](Xd, mud, covd, lpid))
    ref = (z["out_logZ"], z["out_Nk"], z["out_mu_acc"], z["out_sig"])
    assert_parity(out, ref, what=f"{name} vs reference fixture")
    assert_parity(out, ORACLE[v](X, mu, cov, lpi), what=f"{name} vs oracle")


def test_h100_module_matches_portable_module():
    X, mu, lss, lpi = (t.to(DEV) for t in gmm_data.config_c1())
    a = _np(flash_gmm.flash_gmm_estep(X, mu, lss, lpi))
    b = _np(flash_gmm_h100.flash_gmm_estep(X, mu, lss, lpi))
    for u, w in zip(a, b):
        np.testing.assert_array_equal(u, w)


@pytest.mark.parametrize("cfg,n", [("c2", 40_000), ("c3", 20_000), ("c4", 4_000)])
def test_scaled_configs_vs_oracle(cfg, n):
    X, mu, cov, lpi = gmm_data.make_config(cfg, N=n)
    v = gmm_data.CONFIGS[cfg]["kind"]
    out = _np(ENTRY[v](X.to(DEV), mu.to(DEV), cov.to(DEV), lpi.to(DEV)))
    ref = ORACLE[v](X.numpy(), mu.numpy(), cov.numpy(), lpi.numpy())
    assert_parity(out, ref, what=f"{cfg}[N={n}]")


@pytest.mark.parametrize("v", ["iso", "diag", "full"])
def test_deterministic_and_accumulate(v):
    g = torch.Generator().manual_seed(5)
    N, K, D = 3000, 70, 24
    X = torch.randn(N, D, generator=g).to(DEV)
    mu = torch.randn(K, D, generator=g).to(DEV)
    cov = {"iso": 0.2 * torch.randn(K, generator=g),
           "diag": 0.2 * torch.randn(K, D, generator=g),
           "full": torch.tril(0.1 * torch.randn(K, D, D, generator=g), -1) + torch.eye(D)}[v].to(DEV)
    lpi = torch.log_softmax(torch.randn(K, generator=g), 0).to(DEV)
    a = _np(ENTRY[v](X, mu, cov, lpi))
    b = _np(ENTRY[v](X, mu, cov, lpi))
    for u, w in zip(a, b):
        np.testing.assert_array_equal(u, w)       # bitwise run-to-run
    # chunked accumulation == one call (the streaming recipe, README.md:81-103)
    out = L.estep(VARIANT[v], X[:1234], mu, cov, lpi)
    out = (torch.empty(N - 1234, device=DEV),) + out[1:]
    L.estep(VARIANT[v], X[1234:], mu, cov, lpi, out=out, accumulate=True)
    acc = _np(out)
    for u, w in zip(acc[1:], a[1:]):
        assert np.max(np.abs(u - w)) <= 1e-5 * np.max(np.abs(w))


def test_empty_input_gives_zero_stats():
    X = torch.zeros(0, 8, device=DEV)
    mu = torch.randn(5, 8, device=DEV)
    logZ, Nk, mu_acc, sig = flash_gmm.flash_gmm_estep(X, mu, torch.zeros(5, device=DEV),
                                                      torch.zeros(5, device=DEV))
    torch.cuda.synchronize()
    assert logZ.numel() == 0 and float(Nk.abs().sum()) == 0.0
    assert float(mu_acc.abs().sum()) == 0.0 and float(sig.abs().sum()) == 0.0


def test_headline_config_full_size():
    """C2 at full size (N=1M, K=1024, D=128) against the fp64 oracle, plus the
    size-independent invariants sum_k Nk = N and sum_k mu_acc = sum_n x_n."""
    X, mu, lss, lpi = gmm_data.make_config("c2", device=DEV)
    out = flash_gmm.flash_gmm_estep(X, mu, lss, lpi)
    logZ, Nk, mu_acc, sig = _np(out)
    N = X.shape[0]
    assert abs(Nk.astype(np.float64).sum() - N) <= 1e-5 * N
    xs = X.double().sum(0).cpu().numpy()
    np.testing.assert_allclose(mu_acc.astype(np.float64).sum(0), xs,
                               atol=1e-4 * np.abs(mu_acc).max() * 4)
    ref = O.estep_iso(X.cpu().numpy(), mu.cpu().numpy(), lss.cpu().numpy(), lpi.cpu().numpy())
    assert_parity((logZ, Nk, mu_acc, sig), ref, what="C2 full size")


@pytest.mark.parametrize("cfg,n", [("c2", 300_000), ("c3", 140_000)])
def test_chunked_calls_accumulate_and_repeat(cfg, n):
    """Calls of >= 2048 row tiles run in row chunks on two internal streams
    (split of chunk c+1 overlapping the fused kernel of chunk c): bitwise
    run-to-run, accumulation over two such calls equals one call, and the
    caller's stream sees the results (no explicit synchronisation between)."""
    X, mu, cov, lpi = gmm_data.make_config(cfg, device=DEV, N=2 * n)
    v = VARIANT[gmm_data.CONFIGS[cfg]["kind"]]
    one = _np(L.estep(v, X, mu, cov, lpi))
    again = _np(L.estep(v, X, mu, cov, lpi))
    for a, b in zip(one, again):
        np.testing.assert_array_equal(a, b)
    out = L.estep(v, X[:n], mu, cov, lpi)
    out = (torch.empty(n, device=DEV),) + out[1:]
    L.estep(v, X[n:], mu, cov, lpi, out=out, accumulate=True)
    acc = _np(out)
    for u, w in zip(acc[1:], one[1:]):
        assert np.max(np.abs(u - w)) <= 1e-5 * np.max(np.abs(w))
    assert abs(one[1].astype(np.float64).sum() - 2 * n) <= 1e-5 * 2 * n
