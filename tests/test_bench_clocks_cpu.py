"""The bench's clock record: samples of one or several GPUs reduce to the median SM clock,
the highest max clock and every throttle reason seen (NVML reason bits)."""

import bench


def test_clock_summary_merges_ranks_and_reasons():
    S = bench.ClockSampler
    rank0 = [(1900.0, 1965.0, 0x4), (1910.0, 1965.0, 0x0)]
    rank1 = [(1950.0, 1965.0, 0x4 | 0x8), (1890.0, 1965.0, 0x1)]  # 0x1 (idle) is not reported
    got = S.summary(rank0 + rank1)
    assert got == {"sm_mhz": 1905.0, "sm_max_mhz": 1965.0, "reasons": ["hw_slowdown", "sw_power_cap"],
                   "samples": 4}
    assert S.summary([]) is None
    assert S.summary([(1965.0, 1965.0, 0x20 | 0x40)])["reasons"] == ["hw_thermal_slowdown", "sw_thermal_slowdown"]
