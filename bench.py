"""Benchmark of the B200 GMM E-step (contract: one JSON line from rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c2|c3|c4|c5]

Metric: E-step (sample x component)/s = N*K / seconds per E-step, the
reference's headline shape N=1M, K=1024, D=128.

* ``--workload c2`` (default): every rank holds 1M rows of the C2 mixture
  (generated on the device by the row-keyed generator; rows of rank r are
  global rows [r*1M, (r+1)*1M)), so per-GPU work is fixed as N grows
  ("scaling": "weak").  One step = the E-step on each rank + ONE NCCL
  all-reduce of the packed [Nk | mu_acc | sig_acc] statistics.
  The same line carries ``c5``: the C5 strong-scaling step (100M rows in
  total, each rank streaming its shard in 10M-row chunks, then the
  all-reduce), timed the same way (``--no-c5`` skips it), and
  ``allreduce_ms_per_step`` (N>1).
* ``--workload c3`` / ``c4``: the diagonal (N=1M, K=1024, D=96) and full
  covariance (N=250K, K=256, D=64) configurations per rank, from the seeded
  recipes of ``gmm_data`` (weak scaling; the same rows on every rank).
* ``--workload c5``: N = 100M rows in total (config 5), split across the ranks
  ("scaling": "strong"); each rank runs the E-step over its rows in 10M-row
  chunks with FGMM_FLAG_ACCUMULATE, then one all-reduce.
* ``--impl reference``: the reference's algorithm on the host cores -- the
  CPU restatement in oracle/ (the reference itself is Triton-only and has no
  CPU implementation of the path), fp32 torch-CPU, chunked, all physical
  cores, the workload's full row count per step (C2: 1M rows).  Rank 0 runs
  it; other ranks exit.

Timing: W untimed warm-up steps, then K steps between a barrier +
cuda.synchronize on both sides, CUDA events on the launching stream (one
pair per step); ms_per_step is the median step (the mean is reported too),
max over ranks.  Inputs of C2/C3/C5 (384-512 MB of X per
rank) exceed the 126 MB L2; for C4 (64 MB) a 256 MB buffer is rewritten
between the timed steps.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "flash-gmm_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "estep_pairs_per_s"
UNIT = "(sample x component)/s"
ROWS_C5 = 100_000_000
C5_CHUNK = 10_000_000
E2E_CHUNK = 131_072        # rows per host->device piece in the end-to-end timing
SEED = 1234

# Benchmark workloads.  flops_per_pair is the
# algorithmic work per (row, component) pair: iso 4D, diag 8D, full 4D^2 + 2D.
WORKLOADS = {
    "c2": dict(kind="iso", rows=1_000_000, K=1024, D=128, scaling="weak",
               title="C2 isotropic E-step N=1M K=1024 D=128 per GPU",
               profile="tc_iso_c2.txt", kernel="tc_iso_kernel "
               "(fused distance/LSE/statistics, tcgen05)"),
    "c3": dict(kind="diag", rows=1_000_000, K=1024, D=96, scaling="weak",
               title="C3 diagonal-covariance E-step N=1M K=1024 D=96 per GPU",
               profile="tc_fused_diag_c3.txt", kernel="tc_fused_kernel<diag> "
               "(fused distance/LSE/statistics, tcgen05)"),
    "c4": dict(kind="full", rows=250_000, K=256, D=64, scaling="weak",
               title="C4 full-covariance E-step N=250K K=256 D=64 per GPU",
               profile="full_passes_c4.txt", kernel="full_ll_kernel + full_resp_kernel + "
               "full_stats_kernel (the two tensor-core passes and the responsibilities between)"),
    "c5": dict(kind="iso", rows=ROWS_C5, K=1024, D=128, scaling="strong",
               title="C5 streaming isotropic E-step N=100M K=1024 D=128 total",
               profile="tc_iso_c2.txt", kernel="tc_iso_kernel "
               "(fused distance/LSE/statistics, tcgen05), the last row chunk of a step"),
}


def flops_per_pair(kind: str, D: int) -> float:
    return {"iso": 4.0 * D, "diag": 8.0 * D, "full": 4.0 * D * D + 2.0 * D}[kind]


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "bf16_tflops_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])),
                "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
                "source": "fallback"}


def measured_tf32_tflops():
    """Dense TF32 matmul rate measured on this pool's B200 by
    tests/microbench/microbench.py (committed summary profiles/mma_cost.txt),
    or None."""
    v = profile_traffic("mma_cost.txt", "tf32_tflops")
    return v if v and v > 0 else None


def host_cores():
    """(physical, logical) host cores."""
    logical = os.cpu_count() or 1
    try:
        import psutil
        phys = psutil.cpu_count(logical=False) or logical
    except Exception:
        phys = logical
    return phys, logical


def profile_traffic(profile: str, name: str = "dram_bytes_per_launch"):
    """dram bytes per launch from a committed ncu summary (``key: value``)."""
    path = os.path.join(ROOT, "profiles", profile)
    try:
        for line in open(path):
            if line.startswith(name + ":"):
                return float(line.split(":", 1)[1].split()[0])
    except Exception:
        pass
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region.

    One sampler per job (rank 0) queries every GPU the job runs on: one
    nvidia-smi per rank polling every few ms slowed 8-rank steps ~2x."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices):
        self.gpus = ",".join(str(g) for g in gpu_indices)
        self.proc = None
        self.tmp = None
        self.skip = 0

    def start(self):
        try:
            self.tmp = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpus, f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=self.tmp, stderr=subprocess.DEVNULL)
            # the timed region starts once the sampler is producing lines
            t0 = time.time()
            while time.time() - t0 < 5.0 and os.path.getsize(self.tmp.name) == 0:
                time.sleep(0.02)
            self.skip = sum(1 for _ in open(self.tmp.name))
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.05)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.tmp.flush()
        self.tmp.seek(0)
        rows = [r.split(",") for r in self.tmp.read().strip().splitlines() if r.strip()]
        rows = rows[self.skip:] or rows[-1:]  # samples taken after the timed region began
        os.unlink(self.tmp.name)
        sm = []
        smax = None
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                smax = float(r[2])
                for nm, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(nm)
            except Exception:
                continue
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


CPU_PORT = {"iso": "estep_iso_cpu_fp32", "diag": "estep_diag_cpu_fp32",
            "full": "estep_full_cpu_fp32"}


def cpu_port(kind: str):
    from oracle import gmm_oracle as O
    return getattr(O, CPU_PORT[kind])


def cpu_reference_rate(kind, X, mu, cov, lpi, budget_s: float, chunk: int = 16384,
                       threads: int = 0):
    """Pairs/s of the CPU restatement (fp32 torch-CPU) over a bounded sample."""
    import torch
    fn = cpu_port(kind)
    torch.set_num_threads(threads or os.cpu_count() or 1)
    n_done = 0
    t0 = time.perf_counter()
    start = 0
    while True:
        xs = X[start:start + chunk]
        fn(xs, mu, cov, lpi, chunk=chunk)
        n_done += xs.shape[0]
        start = (start + chunk) % max(1, X.shape[0] - chunk)
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    return n_done * mu.shape[0] / dt, n_done, dt


def host_sample(w: dict, rows: int):
    """CPU rows of the workload's mixture (same recipe, seeded)."""
    import gmm_data
    if w["kind"] == "iso":
        return gmm_data.iso_mixture(rows, w["K"], w["D"], seed=SEED)
    if w["kind"] == "diag":
        return gmm_data.diag_mixture(rows, w["K"], w["D"])
    return gmm_data.full_mixture(rows, w["K"], w["D"])


def run_reference(args):
    """The reference arm: the reference's algorithm on the host cores (the
    reference is Triton-only), the full workload of --workload per step (C2:
    all 1M rows), all physical cores.  Warm-up steps run on a 16K-row slice
    (they only load the code paths); the K timed steps are full."""
    world, rank, _ = dist_setup()
    if rank != 0:
        return 0
    import torch
    w = WORKLOADS[args.workload]
    K = w["K"]
    phys, logical = host_cores()
    torch.set_num_threads(phys)
    rows = w["rows"] if args.workload != "c5" else 1_000_000
    if args.ref_rows > 0:
        rows = min(rows, args.ref_rows)
    X, mu, cov, lpi = host_sample(w, rows)
    fn = cpu_port(w["kind"])
    for _ in range(max(args.warmup, 0)):
        fn(X[:16384], mu, cov, lpi)
    times = []
    for s in range(args.steps):
        t0 = time.perf_counter()
        fn(X, mu, cov, lpi)
        times.append(time.perf_counter() - t0)
    sec = statistics.median(times)
    value = rows * K / sec
    title = w["title"] if args.workload != "c5" else (
        "C5 streaming isotropic E-step; the host runs 1M of its rows per step")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3,
        "ms_per_step_mean": sum(times) / len(times) * 1e3,
        "higher_is_better": True, "scaling": w["scaling"], "vs_baseline": None, "dtype": "f32",
        "data": f"synthetic (seeded {args.workload.upper()} mixture rows on the host)",
        "config": {"workload": title, "K": K, "D": w["D"], "rows_per_step": rows},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": phys, "cores_physical": phys,
                         "cores_logical": logical, "kind": "port",
                         "sample": f"all {rows:,} rows x {K} components per step, torch-CPU "
                                   f"fp32, {phys} threads"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference is Triton-only (GPU); this arm runs its algorithm's CPU "
                "restatement from oracle/ on the host's physical cores",
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="c2")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-c5", action="store_true",
                    help="c2 only: skip the C5 strong-scaling measurement on the same line")
    ap.add_argument("--ref-rows", type=int, default=0,
                    help="reference arm only: rows per step (default: the full workload)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        return run_reference(args)

    import torch
    import torch.distributed as dist

    import _fgmm_lib as L
    import gmm_data
    import gmm_stream as GS

    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    w = WORKLOADS[args.workload]
    kind, K, D = w["kind"], w["K"], w["D"]
    variant = {"iso": L.FGMM_VARIANT_ISO, "diag": L.FGMM_VARIANT_DIAG,
               "full": L.FGMM_VARIANT_FULL}[kind]
    if args.workload == "c5":
        n_global = ROWS_C5
        lo, hi = GS.shard_rows(n_global, rank, world)
        chunk = C5_CHUNK
    else:
        n_global = w["rows"] * world
        lo, hi = rank * w["rows"], (rank + 1) * w["rows"]
        chunk = hi - lo
    n_local = hi - lo
    if kind == "iso":
        # rows of the C2 mixture keyed by global row index (rank r owns its own rows)
        centres = GS.mixture_centres(K, D, SEED, dev)
        X = torch.empty(n_local, D, device=dev, dtype=torch.float32)
        for s in range(0, n_local, C5_CHUNK):
            GS.generate_rows(lo + s, min(C5_CHUNK, n_local - s), centres, SEED,
                             out=X[s:s + C5_CHUNK])
        mu = GS.generate_row_ids(GS.pick_mean_rows(min(n_global, 1_000_000), K, SEED).to(dev),
                                 centres, SEED)
        cov = torch.zeros(K, device=dev)
        lpi = torch.full((K,), -math.log(K), device=dev)
        data = ("synthetic: C2 mixture (centres ~ N(0,4I), rows = centre + N(0,I)) generated "
                "on device by row-keyed counter RNG; mu = 1024 rows of X")
    else:
        # the seeded config recipe (gmm_data), the same rows on every rank
        X, mu, cov, lpi = gmm_data.make_config(args.workload, device=dev)
        data = (f"synthetic: seeded {args.workload.upper()} recipe (gmm_data.make_config) "
                "generated on device; every rank holds the same rows")

    buf, (Nk, mu_acc, sig) = GS.packed_stats(kind, K, D, dev)
    logZ = torch.empty(n_local, device=dev)

    ar_ev = []   # (start, end) of each timed step's all-reduce

    def step(ar_events=None):
        for s in range(0, n_local, chunk):
            e = min(n_local, s + chunk)
            L.estep(variant, X[s:e], mu, cov, lpi,
                    out=(logZ[s:e], Nk, mu_acc, sig), accumulate=s > 0)
        if world > 1:
            if ar_events is not None:
                ar_events[0].record(torch.cuda.current_stream(dev))
            dist.all_reduce(buf)
            if ar_events is not None:
                ar_events[1].record(torch.cuda.current_stream(dev))

    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)

    # profiling events around the dominant kernel of each E-step call
    ev_pairs = []
    # rank 0 samples the clocks of all of this job's GPUs (nvidia-smi indices)
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    vis_ids = [v for v in vis.split(",") if v.strip() != ""]
    gpu_ids = [vis_ids[i] if i < len(vis_ids) else str(i) for i in range(world)]
    sampler = ClockSampler(gpu_ids) if rank == 0 else None
    launches0 = L.launch_count()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    if sampler is not None:
        sampler.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    # X smaller than L2 (C4: 64 MB): each step is timed on its own and a
    # 256 MB buffer is rewritten between steps, outside the timed spans
    flush = None
    if n_local * D * 4 < (192 << 20):
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    step_ev = []
    for _ in range(args.steps):
        if flush is not None:
            flush.fill_(1)
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        b.record(stream)  # materialise both events before handing them to the library
        t0.record(stream)
        L.set_profile_events(a, b)
        ar = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        step(ar if world > 1 else None)
        L.set_profile_events(None, None)
        if world > 1:
            ar_ev.append(ar)
        t1.record(stream)
        ev_pairs.append((a, b))
        step_ev.append((t0, t1))
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    clocks = sampler.stop() if sampler is not None else None
    launches = L.launch_count() - launches0
    step_ms = [t0.elapsed_time(t1) for t0, t1 in step_ev]
    kern_ms = [a.elapsed_time(b) for a, b in ev_pairs]
    ms_mean = sum(step_ms) / args.steps
    ms_step = statistics.median(step_ms)  # the median of the K timed steps
    kern_avg = statistics.median(kern_ms)
    ar_ms = statistics.median([x.elapsed_time(y) for x, y in ar_ev]) if ar_ev else 0.0
    if world > 1:
        t = torch.tensor([ms_step, kern_avg, ms_mean, ar_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_step, kern_avg, ms_mean, ar_ms = float(t[0]), float(t[1]), float(t[2]), float(t[3])

    pairs_step = n_global * K
    value = pairs_step / (ms_step * 1e-3)

    # ---- end to end through the public API: host X (pinned) -> device ->
    # the reference-named entry point -> results read back, every step
    e2e = None
    if not args.no_e2e and args.workload != "c5":
        Xh = X.cpu().pin_memory()
        n_sig = {"iso": K, "diag": K * D, "full": K * D * D}[kind]
        out_host = [torch.empty(n_local, pin_memory=True), torch.empty(K, pin_memory=True),
                    torch.empty(K * D, pin_memory=True), torch.empty(n_sig, pin_memory=True)]
        # host rows stream to the device in E2E_CHUNK-row pieces on a copy stream,
        # overlapped with the E-step of the previous piece (gmm_stream.stream_estep,
        # the reference's chunk-summing recipe); all outputs are read back
        host_chunks = [Xh[s:s + E2E_CHUNK] for s in range(0, n_local, E2E_CHUNK)]

        def e2e_step():
            res = GS.stream_estep(host_chunks, mu, cov, lpi, variant=kind, device=dev,
                                  keep_logZ=True)
            if world > 1:
                packed = torch.cat([res[1], res[2].reshape(-1), res[3].reshape(-1)])
                dist.all_reduce(packed)
            for h, r in zip(out_host, res):
                h.copy_(r.reshape(-1), non_blocking=True)

        for _ in range(max(3, args.warmup)):
            e2e_step()
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        n_e2e = max(10, min(3 * args.steps, 60))  # host-driven: more steps dilute a host stall
        e2e_ev = [torch.cuda.Event(enable_timing=True) for _ in range(n_e2e + 1)]
        e2e_ev[0].record(stream)
        for i in range(n_e2e):
            e2e_step()
            e2e_ev[i + 1].record(stream)
        torch.cuda.synchronize(dev)
        e2e_ms_each = [e2e_ev[i].elapsed_time(e2e_ev[i + 1]) for i in range(n_e2e)]
        ms_e2e = sum(e2e_ms_each) / n_e2e
        if world > 1:
            t = torch.tensor([ms_e2e], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms_e2e = float(t[0])
        h2d = X.numel() * 4
        d2h = (n_local + K + K * D + n_sig) * 4
        e2e = {"value": pairs_step / (ms_e2e * 1e-3), "unit": UNIT, "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": ms_e2e,
               "ms_per_step_min_max": [min(e2e_ms_each), max(e2e_ms_each)],
               "ms_per_step_median": statistics.median(e2e_ms_each),
               "path": f"pinned host X in {E2E_CHUNK}-row pieces -> device (copy stream, "
                       "overlapped) -> gmm_stream.stream_estep (the library E-step per piece, "
                       "statistics accumulated) -> logZ and statistics -> host"}

    # ---- C5 strong scaling beside the C2 line: 100M rows in total, this rank's
    # share streamed through the E-step in 10M-row chunks, then the all-reduce
    c5 = None
    if args.workload == "c2" and not args.no_c5:
        lo5, hi5 = GS.shard_rows(ROWS_C5, rank, world)
        n5 = hi5 - lo5
        X5 = torch.empty(n5, D, device=dev, dtype=torch.float32)
        for s0 in range(0, n5, C5_CHUNK):
            GS.generate_rows(lo5 + s0, min(C5_CHUNK, n5 - s0), centres, SEED,
                             out=X5[s0:s0 + C5_CHUNK])
        logZ5 = torch.empty(n5, device=dev)

        def step5(ar_events=None):
            for s0 in range(0, n5, C5_CHUNK):
                e0 = min(n5, s0 + C5_CHUNK)
                L.estep(variant, X5[s0:e0], mu, cov, lpi,
                        out=(logZ5[s0:e0], Nk, mu_acc, sig), accumulate=s0 > 0)
            if world > 1:
                if ar_events is not None:
                    ar_events[0].record(stream)
                dist.all_reduce(buf)
                if ar_events is not None:
                    ar_events[1].record(stream)

        step5()
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        c5_ms, c5_ar = [], []
        for _ in range(3):
            e5 = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
            e5[0].record(stream)
            step5((e5[2], e5[3]) if world > 1 else None)
            e5[1].record(stream)
            torch.cuda.synchronize(dev)
            c5_ms.append(e5[0].elapsed_time(e5[1]))
            c5_ar.append(e5[2].elapsed_time(e5[3]) if world > 1 else 0.0)
        t5 = torch.tensor([statistics.median(c5_ms), statistics.median(c5_ar)], device=dev)
        if world > 1:
            dist.all_reduce(t5, op=dist.ReduceOp.MAX)
        c5 = {"workload": WORKLOADS["c5"]["title"], "scaling": "strong",
              "ms_per_step": float(t5[0]), "value": ROWS_C5 * K / (float(t5[0]) * 1e-3),
              "unit": UNIT, "rows_per_rank": n5, "steps": 3, "warmup": 1,
              "allreduce_ms": float(t5[1]) if world > 1 else None,
              "how": "every rank streams its shard of the 100M C2-mixture rows (generated on "
                     "device, 10M-row chunks, FGMM_FLAG_ACCUMULATE), then one NCCL all-reduce "
                     "of the packed statistics; CUDA events, median of 3 steps, max over ranks"}
        del X5, logZ5

    # ---- roofline of the dominant kernel
    peaks = load_peaks()
    fpp = flops_per_pair(kind, D)
    # the events bracket the dominant kernels of the last E-step call of each
    # step (one call per step, except c5: the call on the last row chunk)
    last_rows = n_local - ((n_local - 1) // chunk) * chunk
    flops_launch = fpp * last_rows * K
    kern_launch_ms = kern_avg
    achieved = flops_launch / (kern_launch_ms * 1e-3) / 1e12
    traffic = profile_traffic(w["profile"])
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"],
                "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"],
                "traffic": traffic, "peak_source": peaks["source"] + " bf16 burst",
                "kernel": w["kernel"],
                "algorithmic_flops_per_launch": flops_launch,
                "kernel_ms_per_launch": kern_launch_ms, "rows_per_launch": last_rows}
    # north-star roofline: max(tensor time at the measured dense TF32 rate,
    # exp time at the MUFU rate: 16 ex2 per clock per SM, measured by the
    # microbenchmark, at the 1965 MHz maximum clock)
    tf32 = measured_tf32_tflops()
    p_tf32 = tf32 if tf32 else peaks["bf16_tflops"] / 2
    tf32_basis = (f"TF32 {p_tf32:.1f} TFLOP/s measured (torch.matmul 8192^3, "
                  "profiles/mma_cost.txt)" if tf32 else "TF32 = bf16/2 of measured")
    p_mufu = 148 * 16 * 1.965e9
    t_tc = fpp * pairs_step / world / (p_tf32 * 1e12)
    t_exp = pairs_step / world / p_mufu
    t_roof = max(t_tc, t_exp)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        ncpu = min(n_local, 262144)
        Xc, muc, covc, lpic = X[:ncpu].cpu(), mu.cpu(), cov.cpu(), lpi.cpu()
        phys, logical = host_cores()
        rate, nrows, secs = cpu_reference_rate(kind, Xc, muc, covc, lpic, budget_s=12.0,
                                               chunk=65536 if kind != "full" else 4096,
                                               threads=phys)
        cpu = {"value": rate, "unit": UNIT, "cores": phys, "cores_physical": phys,
               "cores_logical": logical, "kind": "port",
               "sample": f"{nrows} rows x {K} components of the same workload in {secs:.1f} s, "
                         f"torch-CPU fp32 restatement (oracle/), {phys} threads"}

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "ms_per_step_mean": ms_mean,
        "higher_is_better": True,
        "scaling": w["scaling"], "vs_baseline": None, "dtype": "f32",
        "data": data,
        "config": {"workload": w["title"], "N_global": n_global, "N_per_rank": n_local, "K": K,
                   "D": D, "covariance": kind,
                   "parallelism": f"dp{world} (rows sharded, one NCCL all-reduce of stats)",
                   "l2": ("inputs larger than L2 (X = %d MB per rank)" % (n_local * D * 4 >> 20)
                          if flush is None else
                          "X = %d MB fits L2: 256 MB buffer rewritten between timed steps"
                          % (n_local * D * 4 >> 20))},
        "roofline": roofline,
        "north_star_roofline": {"t_tensor_ms": t_tc * 1e3, "t_exp_ms": t_exp * 1e3,
                                "t_roof_ms": t_roof * 1e3, "frac": t_roof / (ms_step * 1e-3),
                                "basis": tf32_basis + ", MUFU 148x16/clk @1965 MHz",
                                "frac_bf16_half_basis": (max(fpp * pairs_step / world /
                                                             (peaks["bf16_tflops"] / 2 * 1e12),
                                                             t_exp) / (ms_step * 1e-3))},
        "clocks": clocks,
        "allreduce_ms_per_step": ar_ms if world > 1 else None,
        "c5": c5,
        "e2e": e2e,
        "gpu_launches": launches,
        "cpu_baseline": cpu,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
