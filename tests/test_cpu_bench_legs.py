"""The bench's CPU baselines for configurations 0, 1, 3 and 4 (bench.cpu_legs: the oracle port on the host
cores) run on a small budget and report a positive figure for each configuration."""
from __future__ import annotations


def test_cpu_legs_report_every_configuration():
    import bench

    r = bench.cpu_legs(budget_s=1.0)
    assert r["cfg0"]["gemv_us"] > 0 and r["cfg0"]["gemm_m128_us"] > 0
    assert r["cfg1"]["value"] > 0 and r["cfg3"]["us_per_step"] > 0
    assert r["cfg4"]["value"] > 0 and r["cfg4"]["extrapolated"] is True
    assert all(v["kind"] == "port" and v["cores"] >= 1 for v in r.values())
