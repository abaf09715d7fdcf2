"""Shared pytest setup: import paths and the `gpu` marker.

`-m "not gpu"` runs everywhere (oracle vs golden vectors, host logic, C-ABI
exports, argument validation). `-m gpu` needs a B200 and calls the CUDA path
through the C-ABI.
"""
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]
for p in (REPO, REPO / "tilemix-cuda_b200", REPO / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU; calls the CUDA kernels")
