"""CPU checks of bench.py's reporting logic (the GPU runs are checked by the driver): the
headline metric name, the roofline's algorithmic bytes and ncu traffic per edge, and the
parsing of nvidia-smi clock samples into clocks and throttle reasons."""
import importlib.util
import subprocess
import sys

import pytest

from conftest import ROOT


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def test_metric_names(bench):
    assert bench.metric_for("C3") == bench.METRIC == "atoms*evals/s (E+F+virial), MH1-shape, C3 10k-atom cell"
    assert bench.metric_for("C1").endswith("C1 64-atom cell")
    assert bench.metric_for("C5").endswith("C5 ~200k-atom cell")


def test_roofline_bytes(bench):
    # R and dR rows (2 x 10 paths x 128 fp32), Y and dY, geometry, cutoff and density pairs,
    # sender index, edge force, and the edge's up-gradient row (4 x 128 fp32) written out.
    assert bench.edge_backward1_bytes(1) == 10548 + 2048
    assert bench.edge_backward1_bytes(846394, paths=10) == 846394 * 12596
    # The measured DRAM traffic is within 5% of the algorithmic bytes (no re-reads).
    assert 0.95 < bench.TRAFFIC_PER_EDGE / bench.edge_backward1_bytes(1) < 1.05


def test_roofline_flops(bench, archive_path):
    # 674 FP32 operations per channel and edge: 20 (w) + 408 (terms) + 110 (groups) + 40 (dE/dr)
    # + 96 (dE/dd), over 128 channels.
    assert bench.edge_backward1_flops(1) == 128 * 674
    # Layer-0 linear_2 of the MH1-shaped archive: 4 paths of 512 x 512 over 1 + 3 + 5 + 7
    # components.
    assert bench.linear_flops(archive_path, "layer0.linear_2", 10) == 10 * 2 * 512 * 512 * 16


def test_workload_config_is_shared(bench):
    # The reference arm and this build print the same config object at N = 1.
    assert bench.workload_config("C3", 10000, 1, False) == bench.workload_config("C3", 10000, 1, False)
    assert bench.workload_config("C3", 10000, 1, False)["parallelism"] == "one GPU"
    assert "decomposition" in bench.workload_config("C3", 10000, 4, True)["parallelism"]
    assert bench.io_bytes(10) == (196, 204)


def test_clock_summary(bench):
    sampler = bench.ClockSampler(0)
    t0 = "2026/12/02 10:00:00"
    sampler.lines = [
        t0 + ".000, 0, 1965, 1965, 700.1, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active",
        t0 + ".200, 0, 1890, 1965, 998.7, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
        t0 + ".400, 0, 1900, 1965, 990.0, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
        "garbage",
        t0 + ".600, 0, [N/A], 1965, 0, 0x0, Not Active, Not Active, Not Active, Not Active",
    ]
    s = sampler.summary()
    assert s == {"sm_mhz": 1900.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"], "samples": 3}
    # A marked region keeps the samples within one period (0.2 s) of it.
    base = bench.datetime.datetime.strptime(t0 + ".000", "%Y/%m/%d %H:%M:%S.%f").timestamp()
    sampler.start, sampler.end = base + 0.45, base + 0.46  # window [0.25, 0.66]: the .400 sample
    assert sampler.summary() == {"sm_mhz": 1900.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"], "samples": 1}
    sampler.start, sampler.end = base + 0.05, base + 0.10  # window [-0.15, 0.30]: .000 and .200
    assert sampler.summary()["samples"] == 2
    sampler = bench.ClockSampler(0)
    sampler.lines = [t0 + ".000, 0, 1200, 1965, 500, 0x8, Active, Not Active, Active, Not Active"]
    assert sampler.summary()["reasons"] == ["hw_slowdown", "sw_thermal_slowdown"]
    assert bench.ClockSampler(0).summary() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}


def test_help_runs_without_a_gpu():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--help"], capture_output=True, text=True)
    assert r.returncode == 0 and "--impl" in r.stdout and "--host" in r.stdout
