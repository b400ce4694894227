"""Shared tolerance checks and fixture loading for the parity tests.

Tolerances (the contract of the B200 E-step):
  * logZ: elementwise |a - b| <= 1e-5 * max(1, |b|)
  * Nk, mu_acc, sig: normwise  max|a - b| <= 1e-4 * max|b|
"""

from __future__ import annotations

import glob
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
LOGZ_RTOL = 1e-5
STATS_RTOL = 1e-4


def golden_names():
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "*.npz")))


def load_golden(name: str):
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    return {k: z[k] for k in z.files}


def variant_of(name: str) -> str:
    if name.startswith(("iso", "h100")):
        return "iso"
    return "diag" if name.startswith("diag") else "full"


def golden_inputs(name: str, z: dict):
    """(X, mu, cov, log_pi) as numpy arrays; C1's inputs are regenerated."""
    if name == "iso_c1":
        import hashlib
        import gmm_data
        X, mu, lss, lpi = gmm_data.config_c1()
        sha = hashlib.sha256(X.contiguous().numpy().tobytes()).hexdigest()
        assert sha == str(z["meta_sha_X"]), "regenerated C1 inputs differ from the fixture's"
        return X.numpy(), mu.numpy(), lss.numpy(), lpi.numpy()
    X = z["X"]
    if int(z.get("meta_X_transposed", 0)):
        # the fixture was produced from a transposed view: rebuild that layout
        X = np.ascontiguousarray(X.T).T
    return X, z["mu"], z["lss"], z["lpi"]


def rel_errs(out, ref):
    """[logZ elementwise-relative, then normwise errors of the three stats]."""
    o = [np.asarray(t, dtype=np.float64) for t in out]
    r = [np.asarray(t, dtype=np.float64) for t in ref]
    fin = np.isfinite(r[0])
    assert np.array_equal(fin, np.isfinite(o[0])), "logZ finiteness differs"
    e = [float(np.max(np.abs(o[0][fin] - r[0][fin]) / np.maximum(1.0, np.abs(r[0][fin])),
                      initial=0.0))]
    for a, b in zip(o[1:], r[1:]):
        scale = max(float(np.max(np.abs(b), initial=0.0)), 1e-30)
        e.append(float(np.max(np.abs(a - b), initial=0.0)) / scale)
    return e


def assert_parity(out, ref, logz_tol=LOGZ_RTOL, stats_tol=STATS_RTOL, what=""):
    e = rel_errs(out, ref)
    assert e[0] <= logz_tol, f"{what}: logZ rel err {e[0]:.3e} > {logz_tol}"
    for nm, v in zip(("Nk", "mu_acc", "sig"), e[1:]):
        assert v <= stats_tol, f"{what}: {nm} normwise rel err {v:.3e} > {stats_tol}"
    return e
