"""Small profiling case for ncu captures of the E-step kernels (not a test).

    python tests/profile_case.py [N] [config]   # config c2 (default), c3 or c4;
                                                # N rows of its seeded recipe, 2 E-steps
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
X, mu, cov, lpi = gmm_data.make_config(cfg, device=dev, N=N)
for _ in range(2):
    out = L.estep(variant, X, mu, cov, lpi)
torch.cuda.synchronize()
print("ok", cfg, N, out[1].sum().item())
