"""bench.py's reading of the nvidia-smi clock samples taken during the timed
region (host logic only): the median SM clock under load, the maximum, and
every throttle reason that was active in any sample."""
import importlib.util
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _bench():
    spec = importlib.util.spec_from_file_location("bench_module", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _summary(tmp_path, lines):
    bench = _bench()
    c = bench.Clocks(0, str(tmp_path))
    c.path.write_text("\n".join(lines) + "\n")
    c.proc = object()  # as if nvidia-smi had been started
    return c.summary()


def test_median_clock_and_no_reasons(tmp_path):
    s = _summary(tmp_path, [
        "1965, 1965, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active",
        "1950, 1965, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active",
        "1965, 1965, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active",
    ])
    assert s["sm_mhz"] == 1965.0 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == [] and s["samples"] == 3


def test_active_reasons_are_reported(tmp_path):
    s = _summary(tmp_path, [
        "1300, 1965, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
        "1200, 1965, 0x0000000000000020, Not Active, Not Active, Active, Not Active",
        "garbage line",
        "[N/A], 1965, 0x0, Not Active, Not Active, Not Active, Not Active",
    ])
    assert s["reasons"] == ["sw_power_cap", "sw_thermal_slowdown"]
    assert s["samples"] == 2 and s["sm_mhz"] == 1250.0


def test_no_sampler_reports_unavailable(tmp_path):
    bench = _bench()
    s = bench.Clocks(0, str(tmp_path)).summary()
    assert s["sm_mhz"] is None and s["reasons"] == ["nvidia-smi unavailable"]
