"""bench.py's output contract, checked on the CPU through its reference arm (the reference's own
kernels from oracle/_ref on the host cores): exactly one JSON line on stdout with the keys and
types the benchmark driver reads."""
import json
import os
import subprocess
import sys

import pytest

import oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(not oracle.ref_available(), reason="reference library not built")
def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0",
                        "--no-decode"],
                       cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for key, typ in [("metric", str), ("value", (int, float)), ("unit", str), ("n_gpus", int), ("steps", int),
                     ("warmup", int), ("ms_per_step", (int, float)), ("higher_is_better", bool), ("scaling", str),
                     ("dtype", str), ("data", str), ("config", dict)]:
        assert isinstance(d[key], typ), key
    assert d["steps"] == 1 and d["warmup"] == 0 and d["n_gpus"] == 1
    assert d["value"] > 0 and d["scaling"] in ("weak", "strong")
    assert "vs_baseline" in d and "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["sample"] and cb["value"] == d["value"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert cb["cores"] <= (os.cpu_count() or 1)


def test_cpu_baselines_use_the_cpus_this_process_may_run_on():
    """The CPU baselines' thread count: at least one, at most the CPUs the process may run on."""
    sys.path.insert(0, ROOT)
    import bench
    n = bench.host_cores()
    assert 1 <= n <= len(os.sched_getaffinity(0))
