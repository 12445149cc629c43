"""Host helpers of bench.py (no GPU): the DRAM-traffic ratios it reads from the
committed ncu summaries, keyed by workload and by the cascade mode."""

from __future__ import annotations

import bench


def test_traffic_ratios_come_from_the_profiles():
    cfg3 = bench._traffic_ratio_from_profiles("cfg3-llama3-8b")
    cascade = bench._traffic_ratio_from_profiles("cfg4-prefix-verify+cascade")
    assert cfg3 is not None and 1.0 <= cfg3 < 1.05  # the KV cache is read once
    assert cascade is not None and 1.0 <= cascade < 1.2
    # the plain call on config 4 reads the shared prefix from L2: no ratio applies
    assert bench._traffic_ratio_from_profiles("cfg4-prefix-verify") is None
    assert bench._traffic_ratio_from_profiles("no-such-workload") is None
