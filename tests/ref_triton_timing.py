"""Times the reference's own Triton E-step kernels on this GPU beside this
library's drop-ins, on the benchmark configurations (not a test).

    python tests/ref_triton_timing.py [c2 c3 c4]

The reference modules (flash_gmm.py, flash_gmm_h100.py,
flash_gmm_diag_h100.py, flash_gmm_full_h100.py) are loaded unmodified from
baseline/_ref/ (the reference's install location, not part of this
repository) and called through their public entry points with their default
arguments; Triton compiles them for this GPU, and the autotuned ones pick
their configuration during the untimed warm-up calls.  Both sides are timed
the same way: CUDA events around one entry-point call on the current stream,
median of 5 calls after 2 warm-up calls, inputs resident on the device.

Note on the diagonal reference: its split-K pass re-counts rows of
neighbouring slabs when ceil(N / N_SPLIT) % BLOCK_N != 0
(flash_gmm_diag_h100.py:220-236); its time is reported, its outputs are not
a parity target.
"""
import importlib.util
import os
import statistics
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "flash-gmm_b200"))
import torch  # noqa: E402

import flash_gmm  # noqa: E402
import flash_gmm_diag_h100  # noqa: E402
import flash_gmm_full_h100  # noqa: E402
import gmm_data  # noqa: E402

REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def load_ref(name):
    spec = importlib.util.spec_from_file_location("ref_" + name, os.path.join(REF_DIR, name + ".py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def time_call(fn, *args, reps=5, warm=2):
    for _ in range(warm):
        fn(*args)
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        fn(*args)
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    return statistics.median(ts)


def main():
    cfgs = sys.argv[1:] or ["c2", "c3", "c4"]
    if not os.path.isdir(REF_DIR):
        print(f"reference modules not found under {REF_DIR}")
        return 1
    print(f"device: {torch.cuda.get_device_name()}")
    print(f"{'config':6s} {'implementation':44s} {'ms/E-step':>10s} {'pairs/s':>10s} "
          f"{'ours faster by':>14s}")
    for cfg in cfgs:
        c = gmm_data.CONFIGS[cfg]
        X, mu, cov, lpi = gmm_data.make_config(cfg, device="cuda")
        pairs = X.shape[0] * mu.shape[0]
        if c["kind"] == "iso":
            rows = [("reference flash_gmm.flash_gmm_estep (fp32)", load_ref("flash_gmm").flash_gmm_estep),
                    ("reference flash_gmm_h100.flash_gmm_estep (bf16)",
                     load_ref("flash_gmm_h100").flash_gmm_estep)]
            ours = ("this library, flash_gmm.flash_gmm_estep", flash_gmm.flash_gmm_estep)
        elif c["kind"] == "diag":
            rows = [("reference flash_gmm_diag_h100.flash_gmm_estep_diag",
                     load_ref("flash_gmm_diag_h100").flash_gmm_estep_diag)]
            ours = ("this library, flash_gmm_estep_diag", flash_gmm_diag_h100.flash_gmm_estep_diag)
        else:
            rows = [("reference flash_gmm_full_h100.flash_gmm_estep_full",
                     load_ref("flash_gmm_full_h100").flash_gmm_estep_full)]
            ours = ("this library, flash_gmm_estep_full", flash_gmm_full_h100.flash_gmm_estep_full)
        t_ours = time_call(ours[1], X, mu, cov, lpi)
        for name, fn in rows:
            try:
                t = time_call(fn, X, mu, cov, lpi)
            except Exception as exc:  # e.g. a Triton compile failure for this GPU
                print(f"{cfg:6s} {name:44s} failed: {type(exc).__name__}: "
                      f"{str(exc).splitlines()[-1][:80]}", flush=True)
                continue
            print(f"{cfg:6s} {name:44s} {t:10.3f} {pairs / t * 1e3:10.3e} {t / t_ours:13.1f}x",
                  flush=True)
        print(f"{cfg:6s} {ours[0]:44s} {t_ours:10.3f} {pairs / t_ours * 1e3:10.3e}", flush=True)
        del X, mu, cov, lpi
        torch.cuda.empty_cache()
    return 0


if __name__ == "__main__":
    sys.exit(main())
