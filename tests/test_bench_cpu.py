"""CPU checks of bench.py's helpers (no GPU): the peak follows the clocks
seen (burst at full clock, sustained under the power cap, and ranks that
sampled no clocks); both arms name the same workload; the sharded parity
sample covers every rank's blocks."""
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


def test_both_arms_share_the_workload_string():
    assert bench.workload(1).startswith("config3")
    assert "M=65536" in bench.workload(8) and bench.workload(2) != bench.workload(4)


def test_sharded_parity_sample_covers_every_rank():
    from jstorch_b200 import dist as jdist

    for world, per in ((2, 8), (8, 4)):
        rows = bench._sample_rows(world, 8192, 1024, per)
        assert len(rows) == world * per and rows == sorted(rows)
        owners = []
        for g in rows:
            for r in range(world):
                if any(b.global_row0 <= g < b.global_row0 + b.rows for b in jdist.row_plan(world, r, 8192, 1024)):
                    owners.append(r)
        assert sorted(set(owners)) == list(range(world))
        assert all(owners.count(r) == per for r in range(world))
