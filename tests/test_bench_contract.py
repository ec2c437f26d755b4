"""bench.py's output contract, checked on the CPU.

The reference arm (the reference's own cagra::search through oracle/_ref, or
the C restatement when that library is absent) runs at a small size and must
print exactly one JSON line on stdout with the keys the driver reads.  The
engine arm needs a GPU and is exercised by the GPU test run and the bench.
"""
import json
import os
import subprocess
import sys

from conftest import ROOT

REQUIRED = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
            "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
            "cpu_baseline", "e2e", "impl"}


def test_reference_arm_prints_one_contract_line():
    cmd = [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
           "--n", "20000", "--dim", "64", "--q", "16", "--k", "10", "--centres", "100",
           "--steps", "3", "--warmup", "3"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout
    line = json.loads(lines[0])
    assert REQUIRED <= set(line), REQUIRED - set(line)
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["steps"] == 3 and line["warmup"] >= 3 and line["higher_is_better"] is True
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]
    cfg = line["config"]
    assert (cfg["n_rows"], cfg["dim"], cfg["n_queries"], cfg["k"]) == (20000, 64, 16, 10)
    assert cfg["metric"] == "L2Expanded" and cfg["exact_fp32_rerank"] is False
    assert line["cpu_baseline"]["kind"] in ("reference", "port")
    assert line["cpu_baseline"]["cores"] >= 1


def test_roofline_traffic_comes_from_the_matching_capture():
    # the committed ncu figures are per (dim, k, query count) and scale with
    # the rows a launch scans; a configuration without a capture reports None
    import types

    sys.path.insert(0, ROOT)
    import bench

    with open(os.path.join(ROOT, "profiles", "knn_scan_traffic.json")) as f:
        caps = json.load(f)["captures"]
    for c in caps:
        a = types.SimpleNamespace(dim=c["captured_dim"], k=c["captured_k"],
                                  q=c["captured_queries"])
        assert c["traffic_bytes_per_launch"] == c["dram_bytes_read"] + c["dram_bytes_write"]
        t = bench.profile_traffic(a, 5 * c["captured_rows"])
        assert t == 5 * c["traffic_bytes_per_launch"]
        # every row is read about once: traffic within 3% of the fp16 rows
        assert abs(c["dram_bytes_read"] / (2 * c["captured_rows"] * c["captured_dim"]) - 1) < 0.03
    assert bench.profile_traffic(types.SimpleNamespace(dim=96, k=10, q=100), 1000) is None
