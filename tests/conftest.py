"""Test configuration: import paths, the `gpu` marker, shared fixtures.

The package lives in rdna4-conv3d-wmma_b200/ (the reference keeps its package
under src/, tests/conftest.py:1-6 of the reference); the oracle (test
infrastructure only) lives in oracle/.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "rdna4-conv3d-wmma_b200"), os.path.join(ROOT, "oracle"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN_DIR = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) CUDA device")


@pytest.fixture(scope="session")
def cuda_ready():
    """Fail (not skip) when a GPU test runs without the native library."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from rdna4_conv3d import _native
    _native.lib()  # raises if libr4c_conv3d.so is missing
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    return True
