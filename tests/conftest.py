"""pytest configuration: the `gpu` marker and import paths.

`-m "not gpu"` runs on a CPU-only machine (oracle vs golden vectors, host
logic, C-ABI exports, gloo multi-process tests); `-m gpu` runs the parity
tests of the CUDA kernels on a B200.
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "ouroboros-kernelsmith_b200")
for p in (ROOT, PKG, os.path.dirname(os.path.abspath(__file__))):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
