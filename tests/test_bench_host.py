"""Host-side parts of bench.py, on the CPU: the reference arm's JSON line
(every key of the benchmark contract), its silence on ranks other than 0, the
clock sampler's parsing of nvidia-smi lines, and the peak fallback."""

import json
import os
import subprocess
import sys
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402

CONTRACT = ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
            "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config")


def _run_bench(*args, env_extra=None):
    env = dict(os.environ)
    env.update(env_extra or {})
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args],
                          capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)


def test_reference_arm_prints_one_contract_line():
    r = _run_bench("--impl", "reference", "--workload", "c4", "--steps", "2", "--warmup", "0",
                   "--ref-rows", "8192")
    assert r.returncode == 0, r.stderr
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    line = json.loads(lines[0])
    for key in CONTRACT:
        assert key in line, key
    assert line["impl"] == "reference"
    assert line["metric"] == bench.METRIC and line["unit"] == bench.UNIT
    assert line["value"] > 0 and line["higher_is_better"] is True
    assert line["steps"] == 2 and line["warmup"] >= 3 and line["n_gpus"] == 1
    assert line["vs_baseline"] is None and "workload" in line["config"]
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["kind"] in ("port", "reference")
    assert cb["cores"] >= 1 and cb["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"],
                           "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    expect_ms = 8192 * 256 / line["value"] * 1e3
    assert line["ms_per_step"] == pytest.approx(expect_ms, rel=1e-6)


def test_reference_arm_other_ranks_exit_silently():
    r = _run_bench("--impl", "reference", "--steps", "2", "--warmup", "3",
                   env_extra={"RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == ""


class _FakeProc:
    def terminate(self):
        pass

    def wait(self, timeout=None):
        return 0


def _sampler_over(lines, skip):
    s = bench.ClockSampler([0, 1])
    s.tmp = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
    s.tmp.write("".join(ln + "\n" for ln in lines))
    s.proc = _FakeProc()
    s.skip = skip
    return s


def test_clock_sampler_median_and_reasons_after_skip():
    na, act = "Not Active", "Active"
    lines = [
        f"0, 900, 1965, 100.0, 0x1, {na}, {na}, {act}, {na}",     # before the timed region
        f"0, 1965, 1965, 700.0, 0x4, {na}, {na}, {na}, {act}",
        f"1, 1950, 1965, 710.0, 0x4, {na}, {na}, {na}, {act}",
        f"0, 1900, 1965, 720.0, 0x0, {na}, {na}, {na}, {na}",
        "garbage line",
    ]
    s = _sampler_over(lines, skip=1)
    name = s.tmp.name
    out = bench.ClockSampler.stop(s)
    assert out == {"sm_mhz": 1950.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"],
                   "samples": 3}
    assert not os.path.exists(name)


def test_clock_sampler_reports_throttle_and_keeps_last_line_when_nothing_new():
    na, act = "Not Active", "Active"
    lines = [f"0, 1200, 1965, 990.0, 0x8, {act}, {act}, {na}, {na}"]
    out = _sampler_over(lines, skip=1).stop()
    assert out["sm_mhz"] == 1200.0
    assert out["reasons"] == ["hw_slowdown", "hw_thermal_slowdown"]


def test_clock_sampler_without_nvidia_smi_returns_none():
    s = bench.ClockSampler([0])
    assert s.stop() is None


def test_flops_per_pair_and_peak_fallback(monkeypatch, tmp_path):
    assert bench.flops_per_pair("iso", 128) == 512.0
    assert bench.flops_per_pair("diag", 96) == 768.0
    assert bench.flops_per_pair("full", 64) == 4 * 64 * 64 + 128.0
    monkeypatch.setattr(bench, "ROOT", str(tmp_path))
    p = bench.load_peaks()
    assert p["source"] == "fallback" and p["hbm_gbs"] == 6650.0 and p["bf16_tflops"] == 1590.0
    (tmp_path / "MEASURED_PEAKS.json").write_text(json.dumps({"hbm_gbs": 6544.0,
                                                               "bf16_tflops": 1675.7}))
    p = bench.load_peaks()
    assert p["source"] == "measured" and p["bf16_tflops_sustained"] == 1675.7


def test_profile_traffic_reads_committed_summaries():
    for w in bench.WORKLOADS.values():
        t = bench.profile_traffic(w["profile"])
        assert t is not None and t > 0, w["profile"]
    assert bench.profile_traffic("no_such_profile.txt") is None
