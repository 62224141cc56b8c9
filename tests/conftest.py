"""Test configuration: registers the `gpu` marker and puts the repo root on sys.path.

`-m "not gpu"` runs everywhere (oracle vs golden vectors, host logic, C-ABI exports, gloo ranks);
`-m gpu` needs a B200 and calls the CUDA path through the C-ABI library."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
