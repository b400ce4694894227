"""Small profiling case for ncu captures of the fused kernel (not a test).

    python tests/profile_case.py [N]     # C2 mixture with N rows, 2 E-steps
"""
import sys
import os
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT); sys.path.insert(0, os.path.join(ROOT, "flash-gmm_b200"))
import torch, _fgmm_lib as L, gmm_data
dev = torch.device("cuda")
N = int(sys.argv[1]) if len(sys.argv) > 1 else 400_000
X, mu, lss, lpi = gmm_data.make_config("c2", device=dev, N=N)
for _ in range(2): out = L.estep(0, X, mu, lss, lpi)
torch.cuda.synchronize()
print("ok", out[1].sum().item())
