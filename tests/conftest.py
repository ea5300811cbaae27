"""Test configuration: import paths and the ``gpu`` marker.

``-m "not gpu"`` runs on a CPU-only machine: the oracle against the golden
vectors, the host-side Python logic, and the C-ABI library's exports.
``-m gpu`` runs the parity tests proper on a B200; they call the kernels through
the C ABI (directly via ctypes, or via the thin torch binding over it).
"""

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "ash-quant-kernels_b200")
for p in (ROOT, PKG_DIR):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (B200); run with -m gpu")
