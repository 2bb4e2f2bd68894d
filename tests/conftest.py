"""Shared pytest setup: the `gpu` marker and import paths.

Tests marked `gpu` need a CUDA device and the built libiris_b200.so; the rest
run on a CPU-only machine (oracle known-answer tests, host logic, the C-ABI
symbol check, and multi-process gloo tests).
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built CUDA library")
