"""pytest configuration: import paths and the `gpu` marker.

Tests marked `gpu` need a CUDA device (a B200) and the built native libraries; everything
else runs on CPU (`pytest -m "not gpu"`).
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "rdna4-vllm_b200"), os.path.join(ROOT, "oracle"),
          os.path.join(ROOT, "tests", "golden"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built libraries")
