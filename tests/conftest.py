"""Shared pytest setup: the `gpu` marker and import paths.

Tests marked `gpu` need a CUDA device and the built native library; every
other test runs on a CPU-only machine.
"""
import pathlib
import sys

ROOT = pathlib.Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a) and the built libtitan_b200.so")
