"""bench.py's host-side logic on CPU: which library path a workload takes (the label
and arithmetic type of its line), and the reference arm's JSON line."""
import json
import subprocess
import sys
from pathlib import Path

import bench
from prism_test_b200 import workloads as W

ROOT = Path(__file__).resolve().parents[1]


def test_path_of_follows_the_dispatch():
    wl = W.WORKLOADS
    assert bench.path_of(wl["prefill-chunk-128k"]) == "prefill"
    assert bench.path_of(wl["decode-128k"]) == "decode"
    assert bench.path_of(wl["decode-1m-sharded"]) == "decode"
    # 8 query positions x 28 heads over one 256K cache: the queries-as-M tensor-core pass
    assert bench.path_of(wl["shared-context-256k"]) == "wide"
    # the same workload split over 8 ranks: each shard holds fewer than 16 k keys
    assert bench.path_of(wl["shared-context-256k"], "qk", wl["shared-context-256k"].Sk // 8) == "decode"
    # the value-weighted recall takes the score-matrix path
    assert bench.path_of(wl["shared-context-256k"], "qkv") == "decode"
    assert "tcgen05" in bench.dtype_of(wl["shared-context-256k"])
    assert "tcgen05" in bench.dtype_of(wl["prefill-chunk-128k"])


def test_reference_arm_line():
    # the reference arm times the oracle port on the host cores: no GPU needed
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--workload", "cpu-ref-16k",
                          "--steps", "1", "--warmup", "1"], cwd=ROOT, capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads([x for x in out.stdout.splitlines() if x.startswith("{")][-1])
    assert line["impl"] == "reference" and line["n_gpus"] == 1 and line["steps"] == 1
    assert line["value"] > 0 and line["unit"] == bench.UNIT and line["metric"] == bench.METRIC
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"], "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert line["config"]["workload"] == "cpu-ref-16k"
