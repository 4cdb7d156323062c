"""Test configuration: the `gpu` marker and the repository root on sys.path.

`-m "not gpu"` runs on any machine (oracle known-answer tests, host logic, the C-ABI library's
exports). `-m gpu` runs the parity tests proper on a B200: every one calls the CUDA kernels
through the C ABI and checks them against the CPU oracle.
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
