"""Test configuration.

Markers: ``gpu`` (needs a B200; run with ``-m gpu``).  Everything else runs
on CPU.  The package directory ``ltx-2-mlx_b200`` is put on sys.path so that
``import ltxq`` resolves to the in-tree package (and its in-tree libltxq.so).
"""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "ltx-2-mlx_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a visible CUDA device")
    return torch.device("cuda:0")
