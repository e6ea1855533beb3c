"""pytest configuration: the `gpu` marker and import paths.

Tests marked `gpu` need a B200 (sm_100a) and call librustane_cuda.so through
its C ABI; everything else runs on the CPU (oracle, golden vectors, host-side
logic, library symbol checks, gloo multi-process tests).
"""
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "oracle"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU (sm_100a)")
