"""pytest configuration: the `gpu` marker and import paths.

Tests marked `gpu` need a CUDA device and the built CUDA library; everything
else runs on the CPU (oracle vs golden vectors, GGUF and host logic, and the
C-ABI library's exported symbols).
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a) and the built libcuq.so")
