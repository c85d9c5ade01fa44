"""Clock-sample summaries used by the benchmarks' `clocks` record (nvidia-smi CSV rows; read-only
sampling, nothing on the GPU is changed)."""
from my_muon_fsdp2_b200.utils.clocks import physical_gpu_index, summarize


def _row(sm, reasons=("Not Active",) * 4, mx=1965, power=900.0, idx=0, active="0x0000000000000000"):
    return ", ".join([str(idx), str(sm), str(mx), str(power), active] + list(reasons))


def test_median_under_load_and_reasons():
    rows = [_row(345), _row(1500), _row(1605), _row(1650),
            _row(1620, ("Not Active", "Not Active", "Not Active", "Active"))]
    s = summarize(rows)
    assert s["samples"] == 5 and s["sm_max_mhz"] == 1965
    assert s["sm_mhz"] == 1612.5  # median of the samples at or above the 25th percentile (1500 MHz): the idle 345 MHz edge drops
    assert s["reasons"] == ["sw_power_cap"] and s["power_w_max"] == 900.0


def test_thermal_reason_and_bad_rows():
    rows = ["garbage", "0, N/A, 1965, 10, x, a, b, c, d",
            _row(1200, ("Not Active", "Active", "Not Active", "Not Active"))]
    s = summarize(rows)
    assert s["samples"] == 1 and s["reasons"] == ["hw_thermal_slowdown"]


def test_no_samples():
    assert summarize([])["reasons"] == ["no samples"]


def test_physical_index_follows_visible_devices(monkeypatch):
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "3,5")
    assert physical_gpu_index(1) == 5
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "GPU-abc")
    assert physical_gpu_index(0) == 0
    monkeypatch.delenv("CUDA_VISIBLE_DEVICES")
    assert physical_gpu_index(2) == 2
