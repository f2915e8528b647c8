"""Test configuration: the `gpu` marker and import paths.

Tests marked `gpu` need a B200 and call libstade_b200 through its C ABI;
everything else runs on the CPU (oracle pins, ABI exports, host logic,
multi-rank host paths over gloo).
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "stade.jl_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); parity tests of the CUDA path")
