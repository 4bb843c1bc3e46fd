"""pytest configuration: the `gpu` marker and import paths.

`-m "not gpu"` runs on any machine (oracle vs golden fixtures, host logic,
C-ABI exports); `-m gpu` needs a B200 and calls the kernels through the C ABI.
"""
import os
import sys

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
for p in (ROOT, os.path.join(ROOT, "sen-mlx_b200"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU (runs the sm_100a kernels)")
