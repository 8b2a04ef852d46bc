"""The service's host thread pool and bf16 widening (csrc/host_copy.cpp) on
the CPU: a stress test with late-waking workers, every piece of every job
run exactly once, and the widening exact at every alignment. No GPU."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
CSRC = ROOT / "ggml-xdna_b200" / "csrc"


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_host_pool_and_widening(tmp_path):
    exe = tmp_path / "host_pool_stress"
    subprocess.run(["g++", "-O2", "-std=c++17", "-pthread", f"-I{CSRC}", str(ROOT / "tests" / "host_pool_stress.cpp"),
                    str(CSRC / "host_copy.cpp"), "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "POOL OK" in r.stdout, r.stdout + r.stderr
