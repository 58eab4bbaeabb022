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
def test_reference_arm_prints_one_contract_line(tmp_path):
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0",
                        "--no-decode"],
                       cwd=ROOT, capture_output=True, text=True, timeout=600,
                       env=dict(os.environ, SARDYNE_MODEL_DIR=str(tmp_path)))  # caches stay in the test's directory
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


def test_sweep_inputs_are_cached_and_rebuilt_when_damaged(tmp_path, monkeypatch):
    """bench.make_inputs keeps the quantized matrices in the model cache directory: a second call
    returns the same bytes from the cache, and a truncated cache file is rebuilt."""
    monkeypatch.setenv("SARDYNE_MODEL_DIR", str(tmp_path))
    sys.path.insert(0, ROOT)
    import numpy as np

    import bench
    monkeypatch.setattr(bench, "SHAPES", [(16, 256), (40, 512)])  # small matrices: the same code
    first, xs = bench.make_inputs(only="Q4_K:16")
    path = bench.inputs_cache_path(only="Q4_K:16")
    assert path.exists() and [p.name for p in tmp_path.iterdir()] == [path.name]
    again, _ = bench.make_inputs(only="Q4_K:16")
    assert [m[:3] for m in again] == [m[:3] for m in first] == [("Q4_K", 16, 256)]
    assert all(np.array_equal(a[3], b[3]) for a, b in zip(first, again))
    path.write_bytes(path.read_bytes()[:100])
    rebuilt, _ = bench.make_inputs(only="Q4_K:16")
    assert np.array_equal(rebuilt[0][3], first[0][3]) and path.stat().st_size > 100
    full, _ = bench.make_inputs()  # every format and shape, one file each set
    assert [m[:3] for m in full] == [(f, n, k) for f in bench.FORMATS for n, k in bench.SHAPES]
    assert all(np.array_equal(a[3], b[3]) for a, b in zip(full, bench.make_inputs()[0]))
