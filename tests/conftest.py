"""Test setup: import paths and the `gpu` marker.

`-m "not gpu"` runs on any host: the oracle against the golden vectors and
the reference build, the host logic, and that the C-ABI libraries load and
export what include/*.h declares. `-m gpu` runs on a B200 and checks every
kernel through the C ABI against the oracle.
"""
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "ggml-xdna_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
