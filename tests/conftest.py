"""Shared pytest setup: the ``gpu`` marker and import paths for the package and the oracle."""

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("", "onnxruntime-ep-mlx_b200", os.path.join("tests", "golden")):
    path = os.path.join(ROOT, sub)
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built extension")
