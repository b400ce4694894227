"""Small profiling case for ncu captures of the E-step kernels (not a test).

    python tests/profile_case.py [N] [config] [K] [D]
        config c2 (default), c3 or c4: N rows of its seeded recipe, 2 E-steps;
        K and D, when given, replace the config's component count and
        dimension (same recipe), e.g. 260000 c2 1024 256 for the wide
        isotropic kernel.
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "flash-gmm_b200"))
import torch  # noqa: E402

import _fgmm_lib as L  # noqa: E402
import gmm_data  # noqa: E402

dev = torch.device("cuda")
N = int(sys.argv[1]) if len(sys.argv) > 1 else 400_000
cfg = sys.argv[2] if len(sys.argv) > 2 else "c2"
variant = {"iso": L.FGMM_VARIANT_ISO, "diag": L.FGMM_VARIANT_DIAG,
           "full": L.FGMM_VARIANT_FULL}[gmm_data.CONFIGS[cfg]["kind"]]
if len(sys.argv) > 4:
    K, D = int(sys.argv[3]), int(sys.argv[4])
    make = {"iso": gmm_data.iso_mixture, "diag": gmm_data.diag_mixture,
            "full": gmm_data.full_mixture}[gmm_data.CONFIGS[cfg]["kind"]]
    X, mu, cov, lpi = make(N, K, D, device=dev)
else:
    X, mu, cov, lpi = gmm_data.make_config(cfg, device=dev, N=N)
for _ in range(2):
    out = L.estep(variant, X, mu, cov, lpi)
torch.cuda.synchronize()
print("ok", cfg, N, out[1].sum().item())
