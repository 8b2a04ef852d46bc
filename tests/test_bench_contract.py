"""bench.py's reference arm on the host (it needs no GPU): one JSON line with
the keys the driver reads, BASELINE.json's metric, the CPU baseline it ran
and an end-to-end figure with no host-device copies; at least 3 warm-up
steps whatever is asked; under torchrun only rank 0 prints."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
REF_LIB = ROOT / "oracle" / "_ref" / "libzest_ref.so"

pytestmark = pytest.mark.skipif(not REF_LIB.exists(), reason="oracle/_ref not built (needs the reference sources)")


def lines(stdout: str) -> list[dict]:
    return [json.loads(s) for s in stdout.splitlines() if s.startswith("{")]


def test_reference_arm_line():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "0"],
                       capture_output=True, text=True, timeout=600, cwd=ROOT,
                       env=dict(os.environ, ZEST_REF_SECONDS="4"))
    assert r.returncode == 0, r.stderr[-2000:]
    (d,) = lines(r.stdout)
    baseline = json.loads((ROOT / "BASELINE.json").read_text())
    assert d["impl"] == "reference" and d["metric"] == baseline["metric"]
    assert d["warmup"] == 3, "at least 3 untimed warm-up steps"
    assert d["steps"] == 1 and d["n_gpus"] == 1 and d["value"] > 0 and d["higher_is_better"] is True
    for key in ("unit", "ms_per_step", "scaling", "vs_baseline", "dtype", "data"):
        assert key in d, key
    assert d["config"]["workload"] == "qwen3-4b-layer"
    sys.path[:0] = [str(ROOT), str(ROOT / "ggml-xdna_b200")]
    import bench
    # the same config as our arm's line, so the two arms compare like with like
    assert d["config"] == bench.layer_config(bench.WORKLOADS["qwen3-4b-layer"], "qwen3-4b-layer", 1, None)
    assert d["scaling"] == "none"
    assert "all 8192 token rows" in d["cpu_baseline"]["sample"]
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["sample"] and cb["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_under_torchrun_prints_once():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
           "127.0.0.1", "--master-port", "29541", str(ROOT / "bench.py"), "--impl", "reference", "--gpus", "2",
           "--steps", "1", "--warmup", "3"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, cwd=ROOT,
                       env=dict(os.environ, OMP_NUM_THREADS="1", ZEST_REF_SECONDS="4"))
    assert r.returncode == 0, r.stderr[-2000:]
    (d,) = lines(r.stdout)
    assert d["impl"] == "reference" and d["n_gpus"] == 2
    assert d["scaling"] == "strong" and d["config"]["parallelism"].startswith("n-shard2")
