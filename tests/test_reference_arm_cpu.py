"""The CPU baseline / reference arm runs the reference's own classes
(oracle/ref_fleet.py over baseline/_ref, installed by oracle/ref_install.py):
a tiny workload through the same function bench.py calls.  Skipped when the
reference is not installed."""
import pytest

from oracle import ref_fleet

pytestmark = pytest.mark.skipif(ref_fleet.reference_dir() is None,
                                reason="reference not installed (python oracle/ref_install.py)")

TINY = dict(layers=2, hq=4, hkv=2, d=128, sessions=2, prompt=64, sink=4, recent=16, important=20,
            dtype="float32", decay=0.99)


def test_reference_fleet_runs_the_reference_cache():
    r = ref_fleet.measure(dict(TINY), budget_s=1.0, max_steps=5, ref_dir=ref_fleet.reference_dir())
    assert r["value"] > 0 and 1 <= r["steps"] <= 5
    assert r["workers"] == 2 and r["cores"] >= 2
    assert isinstance(r["cpu_model"], str) and r["host_cores"] >= 1


def test_bench_reference_cpu_reports_kind_reference():
    import bench
    line = bench.reference_cpu(dict(TINY), 1.0, 3)
    assert line["kind"] == "reference" and line["unit"] == bench.UNIT
    assert "HierarchicalKVCache" in line["sample"]
