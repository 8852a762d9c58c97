"""Test configuration: registers the `gpu` and `slow` markers and puts the repo
root on sys.path so `oracle` (the checker) and `zynfer_b200` import."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA backend)")
    config.addinivalue_line("markers", "slow: full-size parity run, minutes of oracle CPU time")
