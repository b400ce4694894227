"""fgmm_estep_iso_noalloc: the isotropic E-step with library-owned scratch.

Called through the C ABI with ctypes (the argtypes are set here, as a
binding of the header would).  Its results must match the fp64 oracle and
fgmm_estep_iso (with a caller workspace) within the parity tolerances of
tests/parity.py on two calls in a row, whether this file runs alone in a
fresh process or after the rest of the suite.  The file name sorts last on
purpose.
"""

import ctypes

import numpy as np
import pytest
import torch

import _fgmm_lib as L
import gmm_data
from oracle import gmm_oracle as O
from parity import assert_parity

_P, _I64, _I32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32
SCRATCH_BYTES = 64 << 20  # FGMM_NOALLOC_SCRATCH_BYTES


def _noalloc():
    lib = L.load()
    f = lib.fgmm_estep_iso_noalloc
    f.argtypes = [_P, _I64, _I64, _P, _I64, _I64, _P, _P, _I64, _I32, _I32,
                  _P, _P, _P, _P, ctypes.c_uint, _P]
    f.restype = ctypes.c_int
    return lib, f


def _call(f, X, mu, lss, lpi, out, flags=0):
    N, D = X.shape
    K = mu.shape[0]
    logZ, Nk, mu_acc, sig = out
    stream = torch.cuda.current_stream(X.device).cuda_stream if X.is_cuda else None
    return f(X.data_ptr(), X.stride(0), X.stride(1), mu.data_ptr(), mu.stride(0), mu.stride(1),
             lss.data_ptr(), lpi.data_ptr(), N, K, D, logZ.data_ptr(), Nk.data_ptr(),
             mu_acc.data_ptr(), sig.data_ptr(), flags, stream)


def test_oversize_shape_is_rejected_before_any_device_work():
    """The device check comes first (no usable sm_100 device: FGMM_ERR_CUDA
    without a driver, FGMM_ERR_DEVICE on another GPU);
    on a B200 an oversize shape is refused (FGMM_ERR_WORKSPACE) before any
    launch.  The pointers are dummies: neither path touches them."""
    lib, f = _noalloc()
    N, K, D = 200_000, 1024, 128   # tensor-core path needs ~100 MB of scratch
    assert L.workspace_bytes(L.FGMM_VARIANT_ISO, N, K, D) > SCRATCH_BYTES
    before = lib.fgmm_launch_count()
    rc = f(16, D, 1, 16, D, 1, 16, 16, N, K, D, 16, 16, 16, 16, 0, None)
    msg = lib.fgmm_last_error().decode()
    assert "fgmm_estep_iso_noalloc" in msg
    if torch.cuda.is_available():
        assert rc == 2, msg  # FGMM_ERR_WORKSPACE
        assert str(SCRATCH_BYTES) in msg
    else:
        assert rc in (4, 5), msg  # FGMM_ERR_CUDA / FGMM_ERR_DEVICE
    assert lib.fgmm_launch_count() == before


def _inputs(N, K, D, seed, transposed=False):
    X, mu, lss, lpi = gmm_data.iso_mixture(N, K, D, seed=seed)
    dev = "cuda"
    Xd = X.to(dev)
    if transposed:  # same values, column-major storage
        Xd = Xd.t().contiguous().t()
    return Xd, mu.to(dev), lss.to(dev), lpi.to(dev)


def _fresh(N, K, D):
    return (torch.full((N,), float("nan"), device="cuda"),
            torch.full((K,), float("nan"), device="cuda"),
            torch.full((K, D), float("nan"), device="cuda"),
            torch.full((K,), float("nan"), device="cuda"))


def _host(out):
    torch.cuda.synchronize()
    return tuple(t.cpu().numpy() for t in out)


CASES = [
    # (N, K, D, transposed X, flags): tensor-core path with a 4-CTA cluster,
    # single-CTA with ragged D, and the general kernels.
    (20_000, 300, 100, False, 0),
    (7_001, 64, 33, True, 0),
    (5_000, 200, 64, False, L.FGMM_FLAG_FORCE_GENERAL),
]


@pytest.mark.gpu
@pytest.mark.parametrize("N,K,D,transposed,flags", CASES)
def test_noalloc_matches_workspace_entry_on_two_calls(N, K, D, transposed, flags):
    lib, f = _noalloc()
    X, mu, lss, lpi = _inputs(N, K, D, seed=77 + K, transposed=transposed)
    ref = _host(L.estep(L.FGMM_VARIANT_ISO, X, mu, lss, lpi,
                        force_general=bool(flags & L.FGMM_FLAG_FORCE_GENERAL)))
    oracle = O.estep_iso(X.cpu().numpy(), mu.cpu().numpy(), lss.cpu().numpy(),
                         lpi.cpu().numpy())
    for call in range(2):
        out = _fresh(N, K, D)
        rc = _call(f, X, mu, lss, lpi, out, flags)
        assert rc == 0, lib.fgmm_last_error().decode()
        got = _host(out)
        assert_parity(got, oracle, what=f"noalloc call {call + 1} vs the oracle")
        assert_parity(got, ref, what=f"noalloc call {call + 1} vs fgmm_estep_iso")


@pytest.mark.gpu
def test_noalloc_oversize_on_device_launches_nothing():
    lib, f = _noalloc()
    N, K, D = 120_000, 256, 128
    X, mu, lss, lpi = _inputs(N, K, D, seed=5)
    out = _fresh(N, K, D)
    before = L.launch_count()
    rc = _call(f, X, mu, lss, lpi, out)
    assert rc == 2, "shape beyond the fixed scratch must be refused"
    assert L.launch_count() == before
    assert np.isnan(_host(out)[1]).all()  # outputs untouched
