"""Host-side logic of bench.py, on CPU: the roofline denominators, the traffic table's
scaling, the clock record's parsing (only the job's GPUs, only the timed region, throttle
reasons), the all-reduce bucket layout of the config-5 stack and the argument defaults."""

from __future__ import annotations

import importlib.util
import json
import re
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def test_measured_peaks_and_fallback(bench, tmp_path, monkeypatch):
    data = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    for key in ("hbm_gbs", "bf16_tflops", "bf16_tflops_sustained"):
        assert bench.measured_peaks(key) == (float(data[key]), "measured")
    monkeypatch.setattr(bench, "ROOT", tmp_path)  # no MEASURED_PEAKS.json there
    assert bench.measured_peaks("hbm_gbs") == (6650.0, "fallback")
    assert bench.measured_peaks("bf16_tflops") == (1590.0, "fallback")
    assert bench.measured_peaks("bf16_tflops_sustained") == (1400.0, "fallback")


def test_traffic_table_scaling(bench):
    table = json.loads((ROOT / "profiles" / "traffic.json").read_text())["kernels"]
    for kernel, entry in table.items():
        base = entry["params"] if "params" in entry else entry["tokens"]
        t, ratio = bench.traffic_per_launch(kernel, base)
        assert t == pytest.approx(entry["traffic_bytes_per_launch"])
        assert ratio == entry["traffic_over_algorithmic"]
        # Every kernel moves at least its algorithmic bytes (ncu DRAM reads + SM stores).
        assert entry["traffic_over_algorithmic"] >= 0.99, kernel
    # Proportional scaling by tokens, except the GEMM's weights, read once per launch.
    t1, _ = bench.traffic_per_launch("swiglu_bwd", 16384)
    t2, _ = bench.traffic_per_launch("swiglu_bwd", 2 * 16384)
    assert t2 == pytest.approx(2 * t1)
    fixed = 2 * bench.INTER * bench.HIDDEN * bench.BF16
    g1, _ = bench.traffic_per_launch("swiglu_gemm", table["swiglu_gemm"]["tokens"])
    g2, _ = bench.traffic_per_launch("swiglu_gemm", 2 * table["swiglu_gemm"]["tokens"])
    assert g2 - fixed == pytest.approx(2 * (g1 - fixed))
    assert bench.traffic_per_launch("no_such_kernel", 1) == (None, None)


def _sampler(bench, tmp_path, uuids, lines, skip=0):
    s = bench.ClockSampler(uuids)
    path = tmp_path / "clocks.csv"
    path.write_text("".join(line + "\n" for line in lines))
    s.out_path = str(path)
    s.proc = object()  # a sampler that ran
    s.skip = skip
    return s


def test_clock_record_counts_only_the_jobs_gpus_in_the_timed_region(bench, tmp_path):
    busy, idle = "GPU-aaaa", "GPU-bbbb"
    row = "{u}, {mhz}, 1965, {w}, 0x0, Not Active, Not Active, Not Active, {cap}"
    lines = [row.format(u=busy, mhz=300, w=100, cap="Not Active")]  # before mark(): skipped
    lines += [row.format(u=busy, mhz=m, w=900, cap="Active") for m in (1800, 1850, 1900)]
    lines += [row.format(u=idle, mhz=120, w=80, cap="Not Active") for _ in range(5)]
    summary = _sampler(bench, tmp_path, [busy.lower()], lines, skip=1).summary()
    assert summary["sm_mhz"] == 1850 and summary["sm_max_mhz"] == 1965
    assert summary["reasons"] == ["sw_power_cap"] and summary["samples"] == 3
    assert summary["power_w_max"] == 900


def test_clock_record_reports_throttling_and_absence(bench, tmp_path):
    row = "GPU-aaaa, 1400, 1965, 990, 0x0, Active, Not Active, Active, Not Active"
    summary = _sampler(bench, tmp_path, ["aaaa"], [row, row]).summary()
    assert summary["reasons"] == ["hw_slowdown", "sw_thermal_slowdown"]
    assert _sampler(bench, tmp_path, ["aaaa"], []).summary()["reasons"] == ["no samples"]
    assert bench.ClockSampler([]).summary()["reasons"] == ["nvidia-smi unavailable"]


def test_stack_bucket_layout_leaves_only_layer_0_last():
    # Buckets start at every 8th layer and layer 0 is a bucket of its own, issued last (the
    # backward runs from the last layer down): only a 2-norm all-reduce can remain after the
    # last kernel of a step. The expression is taken from Stack.__init__ (which needs a GPU).
    src = (ROOT / "bench.py").read_text()
    m = re.search(r"self\.bucket_starts = (.+)\n", src)
    assert m is not None
    for layers, want in ((32, [0, 1, 8, 16, 24]), (2, [0, 1]), (9, [0, 1, 8]), (1, [0])):
        starts = eval(m.group(1), {"layers": layers})  # noqa: S307 - a set expression
        assert starts == want, layers
        ends = starts[1:] + [layers]
        assert (starts[0], ends[0]) == (0, 1)  # layer 0 alone
        assert all(a < b for a, b in zip(starts, ends))  # no empty bucket


def test_argument_defaults(bench, monkeypatch):
    monkeypatch.setattr(sys, "argv", ["bench.py", "--help"])
    with pytest.raises(SystemExit) as info:
        bench.main()
    assert info.value.code == 0
    src = (ROOT / "bench.py").read_text()
    # NVLink SHARP off for the small dweight all-reduces unless the environment says otherwise.
    assert 'os.environ.setdefault("NCCL_NVLS_ENABLE", "0")' in src
    assert '300 if args.workload in ("mlpup", "mlpact") else 30' in src
