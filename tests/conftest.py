"""Shared pytest setup: marker registration and import paths.

`-m "not gpu"` runs the oracle, host-logic and library-load tests on any CPU
machine; `-m gpu` runs the CUDA parity tests (they call through the C-ABI
library, directly via ctypes or through the `llmik_cuda` torch glue).
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "llm-inference-kernels_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
