"""Shared test setup: import paths and the `gpu` marker.

Tests marked `gpu` need a B200 and call the CUDA path through the C ABI;
everything else runs on CPU (the oracle against the golden fixtures, host
logic, and the C-ABI library's load/export surface).
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "diffuse-rs_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (sm_100a)")
