"""Test configuration: import paths and the ``gpu`` marker.

``-m "not gpu"`` runs everywhere (the oracle against the golden fixtures, the
API contract, the ABI surface, the multi-process host logic on gloo);
``-m gpu`` needs a B200 and the built library, and compares the CUDA kernels
with the CPU oracle through the C ABI.
"""

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "oko-xpu-kernels_b200"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built libxpuint8.so")
