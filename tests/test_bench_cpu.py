"""bench.py's reference arm (the reference's CPU code on this host's cores) and its output contract.

The reference arm needs no GPU: it times the compiled reference C (C1 round trip) on host
threads and prints exactly one JSON line with the same metric, unit and config as the
repository's own arm.
"""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def ref_line():
    from oracle import oracle as O
    if not O.ref_available():
        pytest.skip("compiled reference library not built")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload", "tq4",
                        "--steps", "1", "--warmup", "0"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, r.stdout
    return json.loads(lines[0])


def test_reference_arm_contract(ref_line):
    import bench
    d = ref_line
    assert d["impl"] == "reference" and d["metric"] == bench.METRIC and d["unit"] == "GB/s"
    assert d["higher_is_better"] is True and d["value"] > 0
    assert d["config"]["workload"] == bench.WORKLOAD["tq4"] and d["config"]["input"] == bench.INPUT["tq4"]
    assert d["cpu_baseline"]["kind"] == "reference" and d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["warmup"] >= 3
