"""Shared test setup: marker registration and import paths.

`-m "not gpu"` runs everywhere (oracle vs golden vectors, host logic, C-ABI
symbol checks); `-m gpu` needs an sm_100 device and calls libemx through its
C ABI, checking it against the CPU oracle.
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "engine-mlx_b200"), os.path.join(ROOT, "oracle"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and the built libemx.so")
    config.addinivalue_line("markers", "slow: full-size configuration (minutes)")
