"""Microbenchmarks for the E-step kernel design on one B200.

    python tests/microbench/microbench.py [--json out.json]

Builds fgmm_microbench.cu into tests/microbench/libfgmm_microbench.so (nvcc,
sm_100a) and prints, per measurement, cycles per tcgen05.mma and MACs per
clock per SM (many MMAs in flight, one wait at the end), MUFU / FMA issue
rates, co-resident cluster counts, and the dense TF32 and BF16 matmul rates
of torch (same method as the bf16 peak: 8192^3, best of 10, CUDA events).
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "fgmm_microbench.cu")
LIB = os.path.join(HERE, "libfgmm_microbench.so")


def build(force: bool = False) -> str:
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    nvcc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    if not os.path.exists(nvcc):
        nvcc = "nvcc"
    tmp = LIB + ".tmp"
    subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo",
                    "-std=c++17", "-Xcompiler", "-fPIC", "-shared", "-cudart", "static",
                    "-o", tmp, SRC], check=True)
    os.replace(tmp, LIB)
    return LIB


def _lib():
    lib = ctypes.CDLL(build())
    p, i = ctypes.c_void_p, ctypes.c_int
    lib.fgmm_mb_mma_rate.argtypes = [i, i, i, i, i, i, p, p, p]
    lib.fgmm_mb_mma_rate_2cta.argtypes = [i, i, i, p, p, p]
    lib.fgmm_mb_issue_rate.argtypes = [i, i, i, i, p, p, p]
    lib.fgmm_mb_max_clusters.argtypes = [i, i, i]
    return lib


KIND_NAMES = {0: "f16 A=smem", 1: "f16 A=tmem", 2: "tf32 A=smem", 3: "tf32 A=tmem"}


def mma_rate(lib, kind, M, N, ctas=1, iters=4096, hammer=0):
    import torch
    out = torch.zeros(3 * ctas, dtype=torch.int64, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    for _ in range(2):  # first launch warms up
        out.zero_()
        rc = lib.fgmm_mb_mma_rate(kind, ctas, iters, M, N, hammer, out.data_ptr(),
                                  err.data_ptr(), s)
        assert rc == 0, f"launch failed: {rc}"
        torch.cuda.synchronize()
    assert int(err.item()) == 0, "MMA wait timed out"
    o = out.view(ctas, 3).cpu().tolist()
    cyc = statistics.median(r[0] for r in o) / iters
    k = 8 if kind >= 2 else 16
    res = {"what": f"mma {KIND_NAMES[kind]} M={M} N={N}", "ctas": ctas,
           "cycles_per_mma": round(cyc, 2),
           "mac_per_clk_sm": round(M * N * k / cyc, 1),
           "issue_cycles_per_mma": round(statistics.median(r[1] for r in o) / iters, 2)}
    if hammer:
        tot = statistics.median(r[0] for r in o)
        res["hammer_bytes_per_clk"] = round(statistics.median(r[2] for r in o) / tot, 1)
    return res


def mma_rate_2cta(lib, N, pairs=1, iters=4096):
    import torch
    out = torch.zeros(3 * pairs, dtype=torch.int64, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        rc = lib.fgmm_mb_mma_rate_2cta(pairs, iters, N, out.data_ptr(), err.data_ptr(), s)
        assert rc == 0, f"launch failed: {rc}"
        torch.cuda.synchronize()
    assert int(err.item()) == 0, "MMA wait timed out"
    o = out.view(pairs, 3).cpu().tolist()
    cyc = statistics.median(r[0] for r in o) / iters
    return {"what": f"mma f16 cta_group::2 M=256 N={N}", "ctas": 2 * pairs,
            "cycles_per_mma": round(cyc, 2),
            "mac_per_clk_sm": round(128 * N * 16 / cyc, 1)}


OPS = {0: "ex2.approx.ftz.f32", 1: "ex2.approx.f16x2", 2: "fma.rn.f32",
       3: "2 ex2.f32 + 6 fma.f32", 4: "redux.sync.add.u32", 5: "redux.sync.max.f32",
       6: "shfl.sync.bfly.b32", 7: "ex2.approx.ftz.f32, 1 lane of 32 active",
       8: "ex2.approx.ftz.f32, predicated off"}


def issue_rate(lib, op, ctas=148, threads=1024, iters=2048):
    import torch
    out = torch.zeros(ctas, dtype=torch.int64, device="cuda")
    sink = torch.zeros(threads, dtype=torch.float32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        rc = lib.fgmm_mb_issue_rate(ctas, threads, iters, op, out.data_ptr(), sink.data_ptr(), s)
        assert rc == 0
        torch.cuda.synchronize()
    cyc = statistics.median(out.cpu().tolist())
    ops = threads * iters * 8
    return {"what": f"issue {OPS[op]}", "ctas": ctas, "threads": threads,
            "lane_ops_per_clk_sm": round(ops / cyc, 2),
            "warp_instr_per_clk_sm": round(ops / 32 / cyc, 3)}


def matmul_tflops(dtype, tf32=False, n=8192, reps=10):
    import torch
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = tf32
    try:
        a = torch.randn(n, n, device="cuda", dtype=dtype)
        b = torch.randn(n, n, device="cuda", dtype=dtype)
        for _ in range(3):
            torch.matmul(a, b)
        best = 1e9
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
            e0.record()
            torch.matmul(a, b)
            e1.record()
            torch.cuda.synchronize()
            best = min(best, e0.elapsed_time(e1) / 1e3)
        return 2 * n ** 3 / best / 1e12
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old


def run_all(quick: bool = False):
    lib = _lib()
    rows = []
    Ns = [64, 128, 256] if quick else [32, 64, 80, 96, 112, 128, 192, 256]
    for N in Ns:
        rows.append(mma_rate(lib, 0, 128, N))
    for N in Ns:
        rows.append(mma_rate(lib, 1, 128, N))
    if not quick:
        for N in (128, 256):
            rows.append(mma_rate(lib, 0, 64, N))
        for N in (128, 256):
            rows.append(mma_rate(lib, 0, 128, N, ctas=148))
            rows.append(mma_rate(lib, 1, 128, N, ctas=148))
            rows.append(mma_rate(lib, 0, 128, N, ctas=148, hammer=1))
            rows.append(mma_rate(lib, 1, 128, N, ctas=148, hammer=1))
        rows.append(mma_rate(lib, 2, 128, 256))
        rows.append(mma_rate(lib, 3, 128, 256))
        rows.append(mma_rate(lib, 2, 128, 128))
    for N in ((128, 256) if quick else (64, 128, 256)):
        rows.append(mma_rate_2cta(lib, N))
    if not quick:
        rows.append(mma_rate_2cta(lib, 256, pairs=74))
    for op in (0, 1, 2, 3, 4, 5, 6, 7, 8):
        rows.append(issue_rate(lib, op, ctas=148 if not quick else 8))
    clusters = {}
    for smem in (100 * 1024, 200 * 1024):
        for cl in (1, 2, 4, 8, 16):
            clusters[f"cluster={cl} smem={smem // 1024}KB"] = lib.fgmm_mb_max_clusters(
                cl, 256, smem)
    rows.append({"what": "co-resident clusters (occupancy query)", **clusters})
    if not quick:
        import torch
        rows.append({"what": "torch.matmul 8192^3 best of 10",
                     "tf32_tflops": round(matmul_tflops(torch.float32, tf32=True), 1),
                     "bf16_tflops": round(matmul_tflops(torch.bfloat16), 1)})
    return rows


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--json", default=None)
    ap.add_argument("--quick", action="store_true")
    a = ap.parse_args()
    import torch
    rows = run_all(quick=a.quick)
    for r in rows:
        print(json.dumps(r))
    if a.json:
        with open(a.json, "w") as f:
            json.dump({"device": torch.cuda.get_device_name(), "rows": rows}, f, indent=1)


if __name__ == "__main__":
    sys.exit(main())
