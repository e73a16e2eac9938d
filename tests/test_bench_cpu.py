"""CPU checks of bench.py's roofline helpers (no GPU): the peak follows the
clocks seen (burst at full clock, sustained under the power cap, and ranks
that sampled no clocks), and the DRAM traffic comes from the committed ncu
summary."""
import bench

PEAKS = {"bf16_tflops": 1682.1, "bf16_tflops_sustained": 1383.8, "hbm_gbs": 6541.8, "source": "measured"}


def test_tensor_peak_follows_clocks():
    burst, kind = bench._tensor_peak(PEAKS, {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": []})
    assert abs(burst - 1682.1 / 6) < 1e-9 and kind.startswith("burst")
    capped, kind = bench._tensor_peak(PEAKS, {"sm_mhz": 1485.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"]})
    assert abs(capped - 1383.8 / 6) < 1e-9 and kind.startswith("sustained")
    # ranks other than 0 sample no clocks
    assert bench._tensor_peak(PEAKS, None)[0] == burst
    assert bench._tensor_peak(PEAKS, {})[0] == burst


def test_traffic_from_committed_profile():
    traffic, src = bench._traffic_from_profiles()
    assert traffic is not None and 1e9 < traffic < 1e11
    assert "ncu" in src
