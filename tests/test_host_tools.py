"""Host-side pieces that need no GPU: the bench's clock summary and the library-path
override of the package."""

import importlib.util
import pathlib

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]


def _bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_clock_summary_from_nvml_samples():
    b = _bench()
    c = b.ClockSampler(0)
    # (SM MHz, max MHz, NVML clocks-event reason bits): power cap in one sample,
    # hardware slowdown in another.
    c.samples = [(1965, 1965, 0), (1800, 1965, 0x4), (1500, 1965, 0x8), (1965, 1965, 0)]
    s = c.summary()
    assert s["sm_mhz"] == pytest.approx(1882.5) and s["sm_max_mhz"] == 1965
    assert s["reasons"] == ["hw_slowdown", "sw_power_cap"]
    assert s["samples"] == 4 and s["source"] == "nvml"


def test_clock_summary_from_nvidia_smi_rows():
    b = _bench()
    c = b.ClockSampler(0)
    c.rows = [["0", "1965", "1965", "700.1", "0x0", "Not Active", "Not Active", "Not Active",
               "Active"],
              ["0", "1900", "1965", "980.0", "0x4", "Not Active", "Not Active", "Active",
               "Active"],
              ["garbled"]]
    s = c.summary()
    assert s["sm_mhz"] == pytest.approx(1932.5) and s["samples"] == 2
    assert s["reasons"] == ["sw_power_cap", "sw_thermal_slowdown"]
    assert s["source"] == "nvidia-smi"


def test_empty_clock_summary():
    s = _bench().ClockSampler(0).summary()
    assert s["sm_mhz"] is None and s["samples"] == 0 and s["source"] is None


def test_library_path_override(pkg, monkeypatch, tmp_path):
    monkeypatch.setenv("MOE_B200_LIBRARY", str(tmp_path / "absent.so"))
    with pytest.raises(RuntimeError, match="not a file"):
        pkg.get_library_path()
    other = tmp_path / "libother.so"
    other.write_bytes(b"")
    monkeypatch.setenv("MOE_B200_LIBRARY", str(other))
    assert pkg.get_library_path() == str(other)
    monkeypatch.delenv("MOE_B200_LIBRARY")
    assert pkg.get_library_path().endswith("libmoe_b200.so")
