"""Generate the golden fixtures under tests/golden/ by running the REFERENCE's
own Triton kernels on CPU under ``TRITON_INTERPRET=1``.

Run (needs the reference checkout; not run by the test suite):

    python tests/golden/make_golden.py /path/to/Flash-GMM

What is run:

* ``flash_gmm.py`` (portable fp32 isotropic): its two @triton.jit kernels
  ``_flash_gmm_lse_kernel`` (flash_gmm.py:50-103) and
  ``_flash_gmm_accum_kernel`` (flash_gmm.py:110-166) are launched directly with
  the public wrapper's grid and arguments (flash_gmm.py:192-215); the wrapper
  itself refuses CPU tensors (flash_gmm.py:190).  Under the interpreter
  ``tl.dot`` is an exact fp32 numpy product, so these are faithful fp32 runs.
* ``flash_gmm_h100.py``, ``flash_gmm_diag_h100.py``, ``flash_gmm_full_h100.py``:
  the interpreter does not handle their bf16 operands, and their autotuners
  need a driver.  The module source is loaded in memory with
  ``bfloat16 -> float32`` substituted and the ``is_cuda`` assert dropped, each
  autotuned kernel is called through its ``.fn`` with one fixed config, and the
  public wrapper then runs unchanged on CPU tensors.  These fixtures pin the
  FORMULAS and indexing of each variant (log2 folding, sig reconstruction,
  L^T / L^T mu), not bf16 rounding.  The diag wrapper is run with
  ``_pick_n_split`` forced to 1, which avoids the reference's slab-overlap
  defect (diag:220-236); one extra fixture records that defect as the
  reference computes it.

Nothing here is imported by the product or by the tests; the tests only read
the ``.npz`` files this script writes.
"""

from __future__ import annotations

import hashlib
import linecache
import math
import os
import sys
import types

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "flash-gmm_b200"))
import gmm_data  # noqa: E402


def _load_ref_module(ref_dir: str, fname: str, subs, name: str):
    src = open(os.path.join(ref_dir, fname)).read()
    for a, b in subs:
        assert a in src, (fname, a)
        src = src.replace(a, b)
    mod = types.ModuleType(name)
    # Triton's JIT re-reads kernel source through ``inspect``; register the
    # substituted text under a pseudo file name so it sees that text (nothing
    # is written to disk).
    mod.__file__ = f"<{name}:{fname}>"
    lines = src.splitlines(keepends=True)
    linecache.cache[mod.__file__] = (len(src), None, lines, mod.__file__)
    exec(compile(src, mod.__file__, "exec"), mod.__dict__)
    return mod


class _FixedConfig:
    """Stand-in for a triton Autotuner: launches ``fn`` with one config."""

    def __init__(self, autotuner, **cfg):
        self.fn = autotuner.fn
        self.cfg = cfg

    def __getitem__(self, grid):
        def launch(*args, **kw):
            g = grid(self.cfg) if callable(grid) else grid
            return self.fn[g](*args, **kw, **self.cfg)
        return launch


def _save(name: str, inputs: dict, outputs, meta: dict):
    logZ, Nk, mu_acc, sig = (np.asarray(t.detach().cpu().numpy(), dtype=np.float32)
                             for t in outputs)
    arrays = {k: np.asarray(v.detach().cpu().numpy()) for k, v in inputs.items()}
    arrays.update(out_logZ=logZ, out_Nk=Nk, out_mu_acc=mu_acc, out_sig=sig)
    for k, v in meta.items():
        arrays["meta_" + k] = np.asarray(v)
    path = os.path.join(HERE, name + ".npz")
    np.savez_compressed(path, **arrays)
    print(f"wrote {path}  Nk.sum={Nk.sum():.4f}")


def _sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().numpy().tobytes()).hexdigest()


def run_iso_fp32(fg, X, mu, lss, lpi, BLOCK_N=64, BLOCK_K=16, BLOCK_D=128):
    """The launch sequence of flash_gmm.py:187-215 on CPU tensors."""
    N, D = X.shape
    K = mu.shape[0]
    assert D <= BLOCK_D
    logZ = torch.empty(N)
    Nk = torch.zeros(K)
    mu_acc = torch.zeros(K, D)
    sig = torch.zeros(K)
    grid = ((N + BLOCK_N - 1) // BLOCK_N,)
    fg._flash_gmm_lse_kernel[grid](
        X, mu, lss, lpi, logZ, N, K, D, X.stride(0), X.stride(1),
        mu.stride(0), mu.stride(1), BLOCK_N=BLOCK_N, BLOCK_K=BLOCK_K, BLOCK_D=BLOCK_D)
    fg._flash_gmm_accum_kernel[grid](
        X, mu, lss, lpi, logZ, Nk, mu_acc, sig, N, K, D, X.stride(0), X.stride(1),
        mu.stride(0), mu.stride(1), mu_acc.stride(0), mu_acc.stride(1),
        BLOCK_N=BLOCK_N, BLOCK_K=BLOCK_K, BLOCK_D=BLOCK_D)
    return logZ, Nk, mu_acc, sig


def main(ref_dir: str):
    sys.path.insert(0, ref_dir)
    import flash_gmm as fg  # the reference's portable module, unmodified

    g = torch.Generator().manual_seed(20261201)

    def rnd(*s):
        return torch.randn(*s, generator=g)

    # ---- C1 through the fp32 reference kernels (inputs regenerated from seed)
    X, mu, lss, lpi = gmm_data.config_c1()
    out = run_iso_fp32(fg, X, mu, lss, lpi)
    _save("iso_c1", {}, out, dict(N=10000, K=64, D=32, sha_X=_sha(X), sha_mu=_sha(mu),
                                  source="flash_gmm.py fp32 kernels, TRITON_INTERPRET=1"))

    # ---- isotropic edge cases (inputs stored)
    cases = {}
    cases["iso_tiny"] = (rnd(1, 1), rnd(1, 1), torch.zeros(1), torch.zeros(1))
    cases["iso_ragged"] = (rnd(77, 3), rnd(5, 3), 0.3 * rnd(5),
                           torch.log_softmax(rnd(5), 0))
    lp = torch.log_softmax(rnd(20), 0)
    lp[7] = float("-inf")
    cases["iso_neginf_pi"] = (rnd(300, 33), rnd(20, 33), 0.5 * rnd(20), lp)
    Xt = rnd(16, 200)
    cases["iso_strided_X"] = (Xt.t(), rnd(17, 16), 0.2 * rnd(17),
                              torch.full((17,), -math.log(17)))
    cases["iso_fullD"] = (rnd(130, 128), rnd(130, 128), torch.zeros(130),
                          torch.full((130,), -math.log(130)))
    cases["iso_single_comp"] = (rnd(513, 64), rnd(1, 64), torch.zeros(1), torch.zeros(1))
    Xs, mus, lsss, lpis = gmm_data.iso_mixture(600, 64, 128, seed=7)
    cases["iso_separated"] = (Xs, mus, lsss, lpis)
    for name, (X, mu, lss, lpi) in cases.items():
        out = run_iso_fp32(fg, X, mu, lss, lpi)
        _save(name, dict(X=X, mu=mu, lss=lss, lpi=lpi), out,
              dict(source="flash_gmm.py fp32 kernels, TRITON_INTERPRET=1",
                   X_transposed=int(X.stride(0) == 1 and X.shape[1] > 1)))

    subs_common = [("torch.bfloat16", "torch.float32"), ("tl.bfloat16", "tl.float32"),
                   ("assert X.is_cuda and mu.is_cuda", "pass")]

    # ---- h100 isotropic wrapper, fp32-substituted
    h = _load_ref_module(ref_dir, "flash_gmm_h100.py", subs_common, "ref_h100_f32")
    h._gmm_lse_kernel = _FixedConfig(h._gmm_lse_kernel, BLOCK_N=64, BLOCK_K=64)
    h._gmm_atomic_accum = _FixedConfig(h._gmm_atomic_accum, BLOCK_N=64, BLOCK_K=64)
    for name, (N, K, D) in {"h100_iso_a": (500, 40, 24), "h100_iso_kexact": (256, 256, 64)}.items():
        X, mu = 1.5 * rnd(N, D), 1.5 * rnd(K, D)
        lss, lpi = 0.3 * rnd(K), torch.log_softmax(rnd(K), 0)
        out = h.flash_gmm_estep(X, mu, lss, lpi)
        _save(name, dict(X=X, mu=mu, lss=lss, lpi=lpi), out,
              dict(source="flash_gmm_h100.py wrapper, bf16->fp32 substituted, interpreter"))

    # ---- diag wrapper, fp32-substituted, N_SPLIT forced to 1
    dg = _load_ref_module(ref_dir, "flash_gmm_diag_h100.py", subs_common, "ref_diag_f32")
    dg._diag_lse_kernel = _FixedConfig(dg._diag_lse_kernel, BLOCK_N=64, BLOCK_K=64)
    dg._diag_split_k_accum = _FixedConfig(dg._diag_split_k_accum, BLOCK_N=64, BLOCK_K=32)
    dg._pick_n_split = lambda N: 1
    for name, (N, K, D) in {"diag_a": (700, 30, 12), "diag_kexact": (256, 256, 16),
                            "diag_d96": (600, 64, 96)}.items():
        X, mu = rnd(N, D), rnd(K, D)
        lss, lpi = 2.0 * torch.rand(K, D, generator=g) - 1.0, torch.log_softmax(rnd(K), 0)
        out = dg.flash_gmm_estep_diag(X, mu, lss, lpi)
        _save(name, dict(X=X, mu=mu, lss=lss, lpi=lpi), out,
              dict(source="flash_gmm_diag_h100.py wrapper, fp32-substituted, N_SPLIT=1"))

    # ---- the reference's diag slab-overlap defect, recorded as computed
    dg._pick_n_split = lambda N: 16
    dg._diag_split_k_accum = _FixedConfig(dg._diag_split_k_accum, BLOCK_N=128, BLOCK_K=32)
    X, mu = rnd(3000, 8), rnd(16, 8)
    lss, lpi = torch.zeros(16, 8), torch.full((16,), -math.log(16))
    out = dg.flash_gmm_estep_diag(X, mu, lss, lpi)
    _save("diag_slab_overlap_defect", dict(X=X, mu=mu, lss=lss, lpi=lpi), out,
          dict(source="flash_gmm_diag_h100.py, N_SPLIT=16, BLOCK_N=128: rows re-counted"))

    # ---- full-covariance wrapper, fp32-substituted
    fu = _load_ref_module(ref_dir, "flash_gmm_full_h100.py", subs_common, "ref_full_f32")
    for name, (N, K, D) in {"full_pad": (300, 8, 10), "full_d16": (256, 64, 16),
                            "full_d32": (200, 5, 32)}.items():
        X, mu = rnd(N, D), rnd(K, D)
        off = 0.1 * torch.tril(rnd(K, D, D), diagonal=-1)
        L = off + torch.diag_embed(torch.exp(torch.rand(K, D, generator=g) - 0.5))
        lpi = torch.log_softmax(rnd(K), 0)
        out = fu.flash_gmm_estep_full(X, mu, L, lpi)
        _save(name, dict(X=X, mu=mu, lss=L, lpi=lpi), out,
              dict(source="flash_gmm_full_h100.py wrapper, fp32-substituted, interpreter"))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ["FLASH_GMM_REF"])
