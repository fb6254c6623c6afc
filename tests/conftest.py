"""pytest configuration: import paths and the `gpu` marker.

Tests marked `gpu` need a CUDA device (a B200); everything else runs on the
CPU and exercises the oracle, the golden vectors, the host-side logic and the
C ABI's exported symbols.
"""
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "web-xpu-ops_b200", ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (runs on the B200 box)")
